// Token-embedding gather: out[t, :] = bf16_rn(f32(table[clamp(id[t]), :]) * scale).
//
// One warp per token row: the id is read once per warp (one broadcast
// transaction; the reference re-reads it for every 8-element chunk,
// src/kernels/embedding_lookup.cu:33), then each lane moves 16-byte chunks
// lane, lane+32, ... with up to 8 loads in flight before the first store.
// Table rows are loaded with normal caching (ids repeat, and a 2048-wide bf16
// row is 4 KB of reusable L2 data); the output is streamed (evict-first).
// CTAs have 8 warps, or fewer when there are fewer than 8 tokens per SM, so a
// decode-size gather runs on as many SMs as it has warps; a launch of few
// tokens also splits each row over up to 8 warps (below), so 64 ids run as 512
// warps (171 CTAs of 3) of one 32-chunk block each: 1.55 -> 1.50 us per call inside a
// CUDA graph on B200, 8 ids 1.50 -> 1.38 us, 1 id 1.52 -> 1.30 us.
// Arithmetic per element: one fp32 multiply and one RNE rounding, exactly
// src/kernels/embedding_lookup.cu:44-47, so the result is bit-exact.
#include "common.cuh"
#include "launch.h"

namespace hrm {
namespace {

// Launch shape (compile-time; defaults tuned):
//   HRM_EMB_INFLIGHT  16-byte loads per lane issued before the first store
//   HRM_EMB_WAVES     grid cap in waves of 8 CTAs per SM (0: one warp per token)
#ifndef HRM_EMB_INFLIGHT
#define HRM_EMB_INFLIGHT 8
#endif
#ifndef HRM_EMB_WAVES
#define HRM_EMB_WAVES 0
#endif
//   HRM_EMB_SPLIT_SMS warps per SM that a launch of few tokens is spread to by
//                     splitting rows (0: one warp per token always)
#ifndef HRM_EMB_SPLIT_SMS
#define HRM_EMB_SPLIT_SMS 4
#endif

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kInFlight = HRM_EMB_INFLIGHT;

// split = 2^lg_split > 1 (decode-size launches): `split` warps share a token
// row, warp part p moving the 32-chunk blocks p, p + split, ... of it, so that
// a launch of few tokens spreads each row's loads, conversions and stores over
// more SMs.
__global__ void __launch_bounds__(kThreads) embedding_warp_kernel(const uint32_t* ids, const uint4* table,
                                                                  uint4* out, int64_t tokens, int nchunks,
                                                                  uint32_t vocab, float scale, int lg_split) {
  grid_dependency_begin();
  const int lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int split = 1 << lg_split;
  const int64_t warp_stride = (int64_t)gridDim.x * nwarps;
  const int64_t units = tokens << lg_split;
  for (int64_t wi = (int64_t)blockIdx.x * nwarps + (threadIdx.x >> 5); wi < units; wi += warp_stride) {
    const int64_t t = wi >> lg_split;
    const int part = (int)(wi & (split - 1));
    uint32_t id = ids[t];
    if (id >= vocab) id = vocab - 1;
    const uint4* src = table + (int64_t)id * nchunks + 32 * part;
    uint4* dst = out + t * nchunks + 32 * part;
    const int n = nchunks - 32 * part;  // chunks from this part's first block on
    for (int c0 = 0; c0 < n; c0 += 32 * split * kInFlight) {
      uint4 v[kInFlight];
#pragma unroll
      for (int u = 0; u < kInFlight; ++u) {
        const int c = c0 + lane + 32 * split * u;
        if (c < n) v[u] = ld_keep(src + c);
      }
#pragma unroll
      for (int u = 0; u < kInFlight; ++u) {
        const int c = c0 + lane + 32 * split * u;
        if (c < n) {
          uint4 o;
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const uint32_t wa = vget(v[u], w);
            vset(o, w, pack_bf16x2(bf16_lo(wa) * scale, bf16_hi(wa) * scale));
          }
          st_stream(dst + c, o);
        }
      }
    }
  }
}

// Any hidden size / alignment: one element per thread per step.
__global__ void __launch_bounds__(kThreads) embedding_scalar_kernel(const uint32_t* ids, const uint16_t* table,
                                                                    uint16_t* out, int64_t tokens,
                                                                    int64_t hidden, uint32_t vocab,
                                                                    float scale) {
  grid_dependency_begin();
  const int64_t n = tokens * hidden;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride) {
    const int64_t t = i / hidden, j = i - t * hidden;
    uint32_t id = ids[t];
    if (id >= vocab) id = vocab - 1;
    out[i] = f32_to_bf16(bf16_to_f32(table[(int64_t)id * hidden + j]) * scale);
  }
}

}  // namespace

cudaError_t launch_embedding(const uint32_t* ids, const void* table, void* out, int64_t tokens, int64_t hidden,
                             int64_t vocab, float scale, cudaStream_t s) {
  cudaError_t err = cudaSuccess;
  const int64_t wave = (int64_t)device_sm_count() * (2048 / kThreads);
  // (rows of at most 2^30 chunks keep every chunk index of the loops in int)
  if (hidden % 8 == 0 && hidden / 8 <= ((int64_t)1 << 30) && aligned16(table) && aligned16(out)) {
    // decode-size launches: split rows over warps until there are about
    // HRM_EMB_SPLIT_SMS x SMs warps, at most one 32-chunk block per warp
    const int64_t nchunks = hidden / 8;
    int lg_split = 0;
    while (HRM_EMB_SPLIT_SMS > 0 && (tokens << (lg_split + 1)) <= (int64_t)device_sm_count() * HRM_EMB_SPLIT_SMS &&
           (int64_t)32 << (lg_split + 1) <= nchunks)
      ++lg_split;
    const int64_t split = (int64_t)1 << lg_split;
    const int nw = warps_per_cta(tokens * split, kWarps);
    int64_t blocks = (tokens * split + nw - 1) / nw;
    if (HRM_EMB_WAVES > 0 && blocks > wave * HRM_EMB_WAVES) blocks = wave * HRM_EMB_WAVES;
    if (blocks > INT32_MAX) blocks = INT32_MAX;
    err = launch_kernel(embedding_warp_kernel, blocks, 32 * nw, 0, s, ids, static_cast<const uint4*>(table),
        static_cast<uint4*>(out), tokens,
        (int)(hidden / 8), (uint32_t)vocab, scale, lg_split);
  } else {
    int64_t blocks = (tokens * hidden + kThreads - 1) / kThreads;
    if (blocks > wave) blocks = wave;
    err = launch_kernel(embedding_scalar_kernel, blocks, kThreads, 0, s, ids, static_cast<const uint16_t*>(table),
        static_cast<uint16_t*>(out), tokens, hidden,
        (uint32_t)vocab, scale);
  }
  return err;
}

}  // namespace hrm
