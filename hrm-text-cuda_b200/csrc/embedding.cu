// Token-embedding gather: out[t, :] = bf16_rn(f32(table[clamp(id[t]), :]) * scale).
//
// One warp per token row: the id is read once per warp (one broadcast
// transaction; the reference re-reads it for every 8-element chunk,
// src/kernels/embedding_lookup.cu:33), then each lane moves 16-byte chunks
// lane, lane+32, ... with up to 8 loads in flight before the first store.
// Table rows are loaded with normal caching (ids repeat, and a 2048-wide bf16
// row is 4 KB of reusable L2 data); the output is streamed (evict-first).
// CTAs have 8 warps, or fewer when there are fewer than 8 tokens per SM, so a
// decode-size gather (64 ids) runs on 64 SMs.
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

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kInFlight = HRM_EMB_INFLIGHT;

__global__ void __launch_bounds__(kThreads) embedding_warp_kernel(const uint32_t* ids, const uint4* table,
                                                                  uint4* out, int64_t tokens, int nchunks,
                                                                  uint32_t vocab, float scale) {
  grid_dependency_begin();
  const int lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int64_t warp_stride = (int64_t)gridDim.x * nwarps;
  for (int64_t t = (int64_t)blockIdx.x * nwarps + (threadIdx.x >> 5); t < tokens; t += warp_stride) {
    uint32_t id = ids[t];
    if (id >= vocab) id = vocab - 1;
    const uint4* src = table + (int64_t)id * nchunks;
    uint4* dst = out + t * nchunks;
    for (int c0 = 0; c0 < nchunks; c0 += 32 * kInFlight) {
      uint4 v[kInFlight];
#pragma unroll
      for (int u = 0; u < kInFlight; ++u) {
        const int c = c0 + lane + 32 * u;
        if (c < nchunks) v[u] = ld_keep(src + c);
      }
#pragma unroll
      for (int u = 0; u < kInFlight; ++u) {
        const int c = c0 + lane + 32 * u;
        if (c < nchunks) {
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
  if (hidden % 8 == 0 && hidden / 8 <= INT32_MAX && aligned16(table) && aligned16(out)) {
    const int nw = warps_per_cta(tokens, kWarps);
    int64_t blocks = (tokens + nw - 1) / nw;
    if (HRM_EMB_WAVES > 0 && blocks > wave * HRM_EMB_WAVES) blocks = wave * HRM_EMB_WAVES;
    if (blocks > INT32_MAX) blocks = INT32_MAX;
    err = launch_kernel(embedding_warp_kernel, blocks, 32 * nw, 0, s, ids, static_cast<const uint4*>(table),
        static_cast<uint4*>(out), tokens,
        (int)(hidden / 8), (uint32_t)vocab, scale);
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
