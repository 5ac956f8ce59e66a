// Row-normalising kernels: RMSNorm, residual-add + RMSNorm, embedding gather
// + RMSNorm (bf16 I/O) and RMSNorm with fp32 I/O.
//
// Fast path (hidden % vector width == 0, hidden <= 4096 bf16 / 2048 fp32,
// 16-byte aligned pointers): one warp per row, the whole row held in
// registers, so the row is read from HBM exactly once (the reference reads it
// twice, src/kernels/rms_norm.cu:28 and :62).  Lane l holds the 16-byte chunks
// l, l+32, l+64, ... of its row, so every warp-wide access is one contiguous
// 512-byte span.  A CTA of 4 warps (fewer for a launch with fewer than 4 rows
// per SM, so that small launches spread over more SMs) copies the optional
// weight vector into shared memory with cp.async while its first rows load;
// the grid has one warp per row (measured on B200: 6.7 TB/s for add + RMSNorm
// vs 6.05 TB/s with a persistent one-wave grid), and the warps still loop if a
// launch exceeds the grid limit.  4-warp CTAs, against 8, refill an SM at a
// finer grain when a launch ends in a partial wave: RMSNorm [4096 x 2048]
// 7.22 -> 7.05 us (bf16) and 12.14 -> 11.91 us (fp32) in back-to-back
// launches, add + RMSNorm [16384 x 2048] 6283 -> 6390 GB/s; 2 and 16 warps
// were slower.  A plain bf16 RMSNorm launch that fits in one wave of 8-warp
// CTAs at 64 registers takes that shape instead (see rownorm_max_regs), and a
// decode-size launch of wide rows gives each row a CTA (rownorm_cta_kernel).
//
// Reduction order.  rms_norm_kernel runs 256 threads per row: thread t
// accumulates x[t], x[t+256], ... with fused multiply-add (src/kernels/
// rms_norm.cu:28-31), then a shuffle-down tree in each warp (:34-37) and a
// shuffle-down tree over the 8 warp sums (:44-55).  In the register layout a
// lane's chunk j holds elements 8*lane + e + 256*j (bf16), i.e. exactly the
// elements reference thread t = 8*lane + e accumulates, in the same order.
// The lane keeps those 8 partial sums and replays the reference's two trees
// with shuffles, so the sum of squares -- and with it every output -- is
// bit-identical to the reference kernel's.  The fp32 variant follows the same
// 256-thread order (4 elements per chunk; reference threads 4*lane + e and
// 128 + 4*lane + e).
//
// Fallback (any hidden, any alignment): one 256-thread CTA per row with the
// reference's own structure and two passes over the row.
#include <atomic>

#include "common.cuh"
#include "launch.h"

namespace hrm {
namespace {

// Launch shape of the warp-per-row kernels (compile-time; defaults tuned):
//   HRM_RN_WARPS      warps per CTA
//   HRM_RN_WAVES      grid cap in waves of resident CTAs (0: one warp per row)
//   HRM_RN_MAXREGS    register cap per thread (128: no spills, and 2048-wide
//                     rows keep 16-24 warps per SM), enforced through the
//                     __launch_bounds__ minimum of resident CTAs
#ifndef HRM_RN_WARPS
#define HRM_RN_WARPS 4
#endif
#ifndef HRM_RN_WAVES
#define HRM_RN_WAVES 0
#endif
#ifndef HRM_RN_MAXREGS
#define HRM_RN_MAXREGS 128
#endif
// Grid cap of the fp32 kernel, in waves (0: one warp per row), and its
// register cap.
#ifndef HRM_RN_F32_WAVES
#define HRM_RN_F32_WAVES HRM_RN_WAVES
#endif
#ifndef HRM_RN_F32_MAXREGS
#define HRM_RN_F32_MAXREGS HRM_RN_MAXREGS
#endif
// fp32 launches of one to two waves run two rows per warp in one wave (1) or
// one row per warp (0, the default).  [4096 x 2048] back to back on B200:
// with evict-first accesses two rows per warp won (12.0 -> 11.4 us); with the
// default-priority accesses in use now one row per warp wins (11.26 -> 11.09
// us in-process, 5967-5992 -> 6139-6158 GB/s in bench.py).
#ifndef HRM_RN_F32_TWO_ROWS
#define HRM_RN_F32_TWO_ROWS 0
#endif

constexpr int kWarps = HRM_RN_WARPS;          // warp-per-row kernels
constexpr int kThreads = 32 * kWarps;
// __launch_bounds__ minimum resident CTAs that caps a thread at max_regs.
constexpr int min_blocks_for(int max_regs, int threads = kThreads) {
  return 65536 / (threads * max_regs) < 1 ? 1 : 65536 / (threads * max_regs);
}
constexpr int kBlockThreads = 256;            // reference-shaped fallback: 8 warps per row
constexpr int kBlockWarps = kBlockThreads / 32;
constexpr int kMaxVpl = 16;

enum Mode { kRms = 0, kAdd = 1, kEmbed = 2 };

struct RowArgs {
  const uint4* x;        // kRms: input rows; kAdd: x rows; kEmbed: table rows
  const uint4* b;        // kAdd: branch rows
  const uint32_t* ids;   // kEmbed: token ids, one per row
  uint4* r;              // kAdd: residual out; kEmbed: gathered rows out (may be null)
  uint4* y;              // normed out
  const uint4* w;        // weight (null: parameterless)
  int64_t rows;
  int nchunks;           // 16-byte chunks per row
  int hidden;            // elements per row
  uint32_t vocab;        // kEmbed
  float scale;           // kEmbed
  float eps;
};

// ---------------------------------------------------------------- reductions
// bf16 layout: p[e] is the partial sum of reference thread 8*lane + e.
// Reference warp w covers threads 32w..32w+31 = lanes 4w..4w+3, element
// slot m = 8*(lane%4) + e.  Returns the row total in every lane.
__device__ __forceinline__ float ref_tree_bf16(float (&p)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) p[e] += __shfl_down_sync(0xffffffffu, p[e], 2);  // m + 16
#pragma unroll
  for (int e = 0; e < 8; ++e) p[e] += __shfl_down_sync(0xffffffffu, p[e], 1);  // m + 8
  const float q0 = p[0] + p[4], q1 = p[1] + p[5], q2 = p[2] + p[6], q3 = p[3] + p[7];  // m + 4
  const float r0 = q0 + q2, r1 = q1 + q3;                                               // m + 2
  float s = r0 + r1;                                                                    // m + 1
  // lane 4w now holds warp w's sum; tree over the 8 warps (offsets 4, 2, 1).
  s += __shfl_down_sync(0xffffffffu, s, 16);
  s += __shfl_down_sync(0xffffffffu, s, 8);
  s += __shfl_down_sync(0xffffffffu, s, 4);
  return __shfl_sync(0xffffffffu, s, 0);
}

// fp32 layout: a[e] = reference thread 4*lane + e (chunks j even),
// c[e] = reference thread 128 + 4*lane + e (chunks j odd).  Reference warp
// w < 4 covers lanes 8w..8w+7 of a, warp w + 4 the same lanes of c, element
// slot m = 4*(lane%8) + e.
__device__ __forceinline__ float ref_tree_f32(float (&a)[4], float (&c)[4]) {
#pragma unroll
  for (int off = 4; off >= 1; off >>= 1) {  // m + 16, m + 8, m + 4
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      a[e] += __shfl_down_sync(0xffffffffu, a[e], off);
      c[e] += __shfl_down_sync(0xffffffffu, c[e], off);
    }
  }
  const float ra = (a[0] + a[2]) + (a[1] + a[3]);  // m + 2, m + 1
  const float rc = (c[0] + c[2]) + (c[1] + c[3]);
  float s = ra + rc;                               // warp w + warp w+4
  s += __shfl_down_sync(0xffffffffu, s, 16);       // + warp w+2
  s += __shfl_down_sync(0xffffffffu, s, 8);        // + warp w+1
  return __shfl_sync(0xffffffffu, s, 0);
}

// inv = 1 / sqrtf(ss / hidden + eps), as src/kernels/rms_norm.cu:58-59.
__device__ __forceinline__ float inv_rms(float ss, int hidden, float eps) {
  const float rms = sqrtf(ss / (float)hidden + eps);
  return 1.0f / rms;
}

__device__ __forceinline__ uint4 add8(const uint4& a, const uint4& b) {
  uint4 o;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t wa = vget(a, w), wb = vget(b, w);
    vset(o, w, pack_bf16x2(bf16_lo(wa) + bf16_lo(wb), bf16_hi(wa) + bf16_hi(wb)));
  }
  return o;
}

__device__ __forceinline__ uint4 scale8(const uint4& a, float scale) {
  uint4 o;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t wa = vget(a, w);
    vset(o, w, pack_bf16x2(bf16_lo(wa) * scale, bf16_hi(wa) * scale));
  }
  return o;
}

template <bool HAS_W>
__device__ __forceinline__ uint4 norm8(const uint4& v, float inv, const uint4& wv) {
  uint4 o;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t wa = vget(v, w);
    float lo = bf16_lo(wa) * inv, hi = bf16_hi(wa) * inv;
    if (HAS_W) {
      const uint32_t ww = vget(wv, w);
      lo = lo * bf16_lo(ww);
      hi = hi * bf16_hi(ww);
    }
    vset(o, w, pack_bf16x2(lo, hi));
  }
  return o;
}

// Row inputs and outputs (x, branch, residual, normed) move with the default
// L2 priority (ld_l2 / st_l2): RMSNorm bf16 [4096 x 2048] 6.40 -> 5.80 us and
// add + RMSNorm [16384 x 2048] 6.50 -> 6.71 TB/s against evict-first on B200.
// Embed + RMSNorm keeps evict-first stores, so that its outputs do not push
// the repeating table rows out of L2 (the chain's embed + RMSNorm measured
// 6.73 -> 6.62 TB/s with default-priority stores).
template <int MODE>
__device__ __forceinline__ void st_row(uint4* p, const uint4& v) {
  if (MODE == kEmbed)
    st_stream(p, v);
  else
    st_l2(p, v);
}

__device__ __forceinline__ void accum8(float (&p)[8], const uint4& v) {
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t wa = vget(v, w);
    const float lo = bf16_lo(wa), hi = bf16_hi(wa);
    p[2 * w] = fmaf(lo, lo, p[2 * w]);
    p[2 * w + 1] = fmaf(hi, hi, p[2 * w + 1]);
  }
}

// ------------------------------------------------------------ bf16 fast path
// Weight staging.  The CTA's cp.async copies of the weight stay in flight while
// its warps load and reduce their first rows; the CTA waits for them (and
// publishes them with a barrier) only before the first normalisation, so a CTA
// start does not serialise a weight fetch before its row loads.  Every warp
// runs the first iteration of the row loop -- a warp without a row does no
// memory work -- so that all threads reach that barrier.
__device__ __forceinline__ void issue_weight(uint4* s_w, const uint4* w, int nchunks) {
  for (int c = threadIdx.x; c < nchunks; c += blockDim.x) cp_async16(&s_w[c], w + c);
  cp_async_commit();
}
__device__ __forceinline__ void publish_weight() {
  cp_async_wait_all();
  __syncthreads();
}

// Register cap of plain RMSNorm over rows of 1544-2048 elements (7-8 chunks
// per lane; 64 holds the row without spilling) and its warps per CTA, used
// where the launch then fits in one wave; and the cap of embed + RMSNorm there.
#ifndef HRM_RN_NORM8_MAXREGS
#define HRM_RN_NORM8_MAXREGS 64
#endif
#ifndef HRM_RN_NORM8_WARPS
#define HRM_RN_NORM8_WARPS 8
#endif
#ifndef HRM_RN_EMBED8_MAXREGS
#define HRM_RN_EMBED8_MAXREGS HRM_RN_MAXREGS
#endif

// Register cap: HRM_RN_MAXREGS, except
// - add + RMSNorm over rows of more than 2048 elements, whose x and branch
//   chunks (2 x 16 per lane) need more registers than that without spilling;
// - plain and embed + RMSNorm over rows of at most 1536 elements (<= 6 chunks
//   per lane), capped at 64 registers for more warps per SM: embed + RMSNorm
//   at the reference model's hidden 1536 measured 6.36 -> 6.46 TB/s with it;
// - plain RMSNorm over rows of 1544-2048 elements, capped at 64 in 8-warp CTAs
//   when the launch then fits in one wave (4 CTAs per SM): a [4096 x 2048]
//   launch (512 CTAs) is one wave on 148 SMs, against 1.15 waves in the
//   default shape (80 registers, 4-warp CTAs).  Back to back on B200: 7.00 us
//   default, 6.39 us capped in 4-warp CTAs (1024 of them, also one wave), 6.23
//   us capped in 8-warp CTAs.  Larger launches keep the default shape (65536
//   rows: 79.0 us, against 79.4 us capped).  The choice is made per launch.
template <int VPL, int MODE>
constexpr int rownorm_max_regs() {
  return MODE == kAdd ? (VPL > 8 ? 255 : HRM_RN_MAXREGS)
         : VPL <= 6   ? 64
         : VPL <= 8   ? (MODE == kRms ? HRM_RN_MAXREGS : HRM_RN_EMBED8_MAXREGS)
                      : HRM_RN_MAXREGS;
}

// Embedding-table rows of embed + RMSNorm loaded evict-last in L2 (1) or with
// normal caching (0, the default).  Evict-last took the 65536-token embed +
// RMSNorm from 119-120 to 117 us on B200 (the chain +0.4%), but the table's
// lines keep that priority after the kernel returns, which would leave less
// L2 to the GEMMs that follow it in a model; so it is an opt-in build.
#ifndef HRM_EMB_EVICT_LAST
#define HRM_EMB_EVICT_LAST 0
#endif

// L2 prefetch of each warp's first row(s) before the grid dependency wait
// (1) or none (0).
#ifndef HRM_RN_PREFETCH
#define HRM_RN_PREFETCH 1
#endif
// Rows of a warp prefetched before the wait: its rows r and r + G of a grid of
// G warps (one row per warp except in the HRM_RN_F32_TWO_ROWS build).
constexpr int kPrefetchRows = 2;

// Issues the L2 prefetches (lane 0) of this warp's first kPrefetchRows rows of
// x (and b) for a grid whose warp w takes rows w, w + G, ...
template <typename T>
__device__ __forceinline__ void prefetch_warp_rows(const T* x, const T* b, int64_t rows, int nchunks) {
  if ((threadIdx.x & 31) != 0) return;
  const int64_t stride = (int64_t)gridDim.x * (blockDim.x >> 5);
  int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  for (int k = 0; k < kPrefetchRows && r < rows; ++k, r += stride) {
    prefetch_l2(x + r * nchunks, (uint32_t)nchunks * 16u);
    if (b != nullptr) prefetch_l2(b + r * nchunks, (uint32_t)nchunks * 16u);
  }
}

template <int VPL, int MODE, bool HAS_W, int REGS = rownorm_max_regs<VPL, MODE>(), int WARPS = kWarps>
__global__ void __launch_bounds__(32 * WARPS, min_blocks_for(REGS, 32 * WARPS))
    rownorm_warp_kernel(const RowArgs a) {
  if (HRM_RN_PREFETCH && MODE != kEmbed) prefetch_warp_rows(a.x, MODE == kAdd ? a.b : nullptr, a.rows, a.nchunks);
  grid_dependency_begin();
  extern __shared__ uint4 s_w[];
  const int lane = threadIdx.x & 31;
  if (HAS_W) issue_weight(s_w, a.w, a.nchunks);

  const int nwarps = blockDim.x >> 5;  // WARPS, or fewer for a small launch
  const int64_t warp_stride = (int64_t)gridDim.x * nwarps;
  int64_t row = (int64_t)blockIdx.x * nwarps + (threadIdx.x >> 5);
  for (bool first = true; first || row < a.rows; first = false, row += warp_stride) {
    const bool active = row < a.rows;  // uniform across the warp
    const uint4* src = a.x;
    if (active) {
      if (MODE == kEmbed) {
        uint32_t id = a.ids[row];
        if (id >= a.vocab) id = a.vocab - 1;  // src/kernels/embedding_lookup.cu:35
        src = a.x + (int64_t)id * a.nchunks;
      } else {
        src = a.x + row * a.nchunks;
      }
    }
    const int64_t base = row * a.nchunks;

    uint4 v[VPL];
    uint4 vb[MODE == kAdd ? VPL : 1];
    // All loads first (r may alias x / b, so no store may precede a load).
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (active && c < a.nchunks) {
        if (MODE == kEmbed) {
#if HRM_EMB_EVICT_LAST
          v[j] = ld_keep_last(src + c, l2_evict_last_policy());  // table rows may repeat: keep them in L2
#else
          v[j] = ld_keep(src + c);  // table rows may repeat: keep them in L2
#endif
        } else {
          v[j] = ld_l2(src + c);
          if (MODE == kAdd) vb[j] = ld_l2(a.b + base + c);
        }
      }
    }
    float p[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) p[e] = 0.0f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (active && c < a.nchunks) {
        if (MODE == kAdd) {
          v[j] = add8(v[j], vb[j]);
          st_row<MODE>(a.r + base + c, v[j]);
        } else if (MODE == kEmbed) {
          v[j] = scale8(v[j], a.scale);
          if (a.r != nullptr) st_stream(a.r + base + c, v[j]);
        }
        accum8(p, v[j]);
      }
    }
    const float inv = inv_rms(ref_tree_bf16(p), a.hidden, a.eps);
    if (HAS_W && first) publish_weight();
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (active && c < a.nchunks) {
        uint4 wv = make_uint4(0, 0, 0, 0);
        if (HAS_W) wv = s_w[c];
        st_row<MODE>(a.y + base + c, norm8<HAS_W>(v[j], inv, wv));
      }
    }
  }
}

// ------------------------------------------------- bf16 decode-size path
// A launch of at most HRM_RN_CTA_ROWS_PER_SM rows per SM gives each row a CTA
// of nchunks / 32 warps (up to 16): thread c moves the row's 16-byte chunk c
// (the chunk lane c % 32 of the warp kernel holds as its chunk j = c / 32), so
// the loads, the add / scale, the stores and the normalisation of a row spread
// over its warps instead of running one after another in one warp.  The row's
// chunks go to shared memory, and warp 0 replays the warp kernel's summation
// from there -- chunk j = 0, 1, ... per lane, then ref_tree_bf16 -- so the sum
// of squares, and every output, stay bit-identical.  Each thread reads its own
// chunk before writing any output of it (in place use stays safe), and the
// weight chunk comes straight from global memory (L2).
#ifndef HRM_RN_CTA_ROWS_PER_SM
#define HRM_RN_CTA_ROWS_PER_SM 1
#endif
// ... for rows of more than HRM_RN_CTA_MIN_CHUNKS 16-byte chunks: at 6 chunks
// per lane (1536 bf16) the warp kernel is as fast (64 rows of add + RMSNorm:
// 1.93 us, against 1.97 us in CTAs of 6 warps; at 2048 bf16 2.22 -> 2.08 us).
#ifndef HRM_RN_CTA_MIN_CHUNKS
#define HRM_RN_CTA_MIN_CHUNKS 193
#endif
constexpr int kCtaMaxThreads = kMaxVpl * 32;  // 512: a row of 4096 bf16

template <int MODE, bool HAS_W>
__global__ void __launch_bounds__(kCtaMaxThreads) rownorm_cta_kernel(const RowArgs a) {
  if (HRM_RN_PREFETCH && MODE != kEmbed && threadIdx.x == 0 && (int64_t)blockIdx.x < a.rows) {
    prefetch_l2(a.x + (int64_t)blockIdx.x * a.nchunks, (uint32_t)a.nchunks * 16u);
    if (MODE == kAdd) prefetch_l2(a.b + (int64_t)blockIdx.x * a.nchunks, (uint32_t)a.nchunks * 16u);
  }
  grid_dependency_begin();
  __shared__ uint4 s_row[kCtaMaxThreads];
  __shared__ float s_inv;
  const int c = threadIdx.x, lane = c & 31;
  const bool has = c < a.nchunks;
  uint4 wv = make_uint4(0, 0, 0, 0);
  if (HAS_W && has) wv = ld_keep(a.w + c);
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const int64_t base = row * a.nchunks;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (has) {
      if (MODE == kEmbed) {
        uint32_t id = a.ids[row];
        if (id >= a.vocab) id = a.vocab - 1;  // src/kernels/embedding_lookup.cu:35
        v = scale8(ld_keep(a.x + (int64_t)id * a.nchunks + c), a.scale);
        if (a.r != nullptr) st_stream(a.r + base + c, v);
      } else {
        v = ld_l2(a.x + base + c);
        if (MODE == kAdd) {
          v = add8(v, ld_l2(a.b + base + c));
          st_row<MODE>(a.r + base + c, v);
        }
      }
      s_row[c] = v;
    }
    __syncthreads();
    if (c < 32) {
      float p[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) p[e] = 0.0f;
#pragma unroll
      for (int j = 0; j < kMaxVpl; ++j) {
        if (lane + 32 * j < a.nchunks) accum8(p, s_row[lane + 32 * j]);
      }
      const float inv = inv_rms(ref_tree_bf16(p), a.hidden, a.eps);
      if (lane == 0) s_inv = inv;
    }
    __syncthreads();
    if (has) st_row<MODE>(a.y + base + c, norm8<HAS_W>(v, s_inv, wv));
    __syncthreads();  // s_row and s_inv are rewritten by the next row
  }
}

// ---------------------------------------------- bf16 bulk-async (TMA engine) path
// Opt-in build (-DHRM_RN_BULK=1); the register path above is the default.
// Same rows, same lane layout and arithmetic as rownorm_warp_kernel, but the
// input rows reach shared memory through the bulk-copy engine instead of the
// warp's own loads.  Each warp runs its own pipeline over its rows
// (kBkRows contiguous rows, or with kBkRows = 0 rows gw, gw + G, ... of a
// persistent one-CTA-per-SM grid): kBkStages shared-memory stages of one row
// (x, or a gathered table row) or two rows (x and branch), each completed by
// an mbarrier transaction count.  Lane 0 keeps kBkStages rows in flight: as
// soon as the warp has copied stage s into registers it refills s with the
// row kBkStages ahead.  Stores are the warp's usual coalesced 512-byte spans.
//
// Measured on B200, add + RMSNorm over 65536 x 2048 rows in the chain: 6.23
// TB/s at its best shape (4 rows per warp, 8 warps, 2 stages) and 5.79 TB/s
// persistent, against 6.59 TB/s for the register path.  Bytes in flight are
// the limit: the register path holds 16-24 warps x 16 KB per SM (its 117
// registers per thread fill most of the 256 KB register file), while bulk
// staging is capped by 227 KB of shared memory and adds a shared -> register
// hop.  For pure streaming the register file is the larger staging buffer.
//
// In-place use (residual_out == x) stays safe: a row's copy completes before
// any output of that row is written, and every row belongs to one warp.
// Bulk-async path on (1) or off (0, the default: the register path measured
// faster) for the shapes it takes.
#ifndef HRM_RN_BULK
#define HRM_RN_BULK 0
#endif
#if HRM_RN_BULK
#ifndef HRM_BK_WARPS
#define HRM_BK_WARPS 8
#endif
#ifndef HRM_BK_STAGES
#define HRM_BK_STAGES 2
#endif
// Rows per warp (0: persistent grid, one CTA per SM, rows strided by the
// grid's warp count) and resident CTAs per SM the shared memory is sized for.
#ifndef HRM_BK_ROWS
#define HRM_BK_ROWS 4
#endif
#ifndef HRM_BK_CTAS
#define HRM_BK_CTAS 1
#endif
constexpr int kBkMaxWarps = HRM_BK_WARPS;
constexpr int kBkStages = HRM_BK_STAGES;
constexpr int kBkRows = HRM_BK_ROWS;

template <int MODE>
__device__ __forceinline__ void bk_issue(const RowArgs& a, uint4* stage, uint32_t bar, int64_t row,
                                         uint64_t policy) {
  const uint32_t row_bytes = (uint32_t)a.nchunks * 16u;
  mbar_arrive_expect_tx(bar, (MODE == kAdd ? 2u : 1u) * row_bytes);
  if (MODE == kEmbed) {
    uint32_t id = a.ids[row];
    if (id >= a.vocab) id = a.vocab - 1;  // src/kernels/embedding_lookup.cu:35
    bulk_g2s(smem_addr(stage), a.x + (int64_t)id * a.nchunks, row_bytes, bar);  // table rows may repeat
  } else {
    bulk_g2s_hint(smem_addr(stage), a.x + row * a.nchunks, row_bytes, bar, policy);
    if (MODE == kAdd) bulk_g2s_hint(smem_addr(stage + a.nchunks), a.b + row * a.nchunks, row_bytes, bar, policy);
  }
}

template <int VPL, int MODE, bool HAS_W>
__global__ void __launch_bounds__(32 * kBkMaxWarps, 1) rownorm_bulk_kernel(const RowArgs a) {
  grid_dependency_begin();
  extern __shared__ uint4 smem[];
  constexpr int kRowsPerStage = MODE == kAdd ? 2 : 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int w_chunks = HAS_W ? a.nchunks : 0;
  const int stage_chunks = kRowsPerStage * a.nchunks;
  uint4* s_w = smem;
  uint4* s_rows = smem + w_chunks + (int64_t)warp * kBkStages * stage_chunks;
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(smem + w_chunks + (int64_t)nwarps * kBkStages * stage_chunks) + warp * kBkStages;

  if (HAS_W) {
    for (int c = threadIdx.x; c < a.nchunks; c += blockDim.x) cp_async16(&s_w[c], a.w + c);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
  }
  // Row k of this warp: gw + k * G (persistent) or gw * kBkRows + k.
  const int64_t gw = (int64_t)blockIdx.x * nwarps + warp;
  const int64_t G = kBkRows > 0 ? 1 : (int64_t)gridDim.x * nwarps;
  const int64_t row0 = kBkRows > 0 ? gw * kBkRows : gw;
  int64_t K = 0;
  if (row0 < a.rows) {
    K = kBkRows > 0 ? a.rows - row0 : (a.rows - row0 + G - 1) / G;
    if (kBkRows > 0 && K > kBkRows) K = kBkRows;
  }
  if (K == 0) return;
  const uint64_t policy = l2_evict_first_policy();
  if (lane == 0) {
    for (int s = 0; s < kBkStages; ++s) mbar_init(smem_addr(&bars[s]), 1);
    mbar_init_fence();
    for (int s = 0; s < kBkStages && s < K; ++s)
      bk_issue<MODE>(a, s_rows + s * stage_chunks, smem_addr(&bars[s]), row0 + s * G, policy);
  }
  __syncwarp();

  for (int64_t k = 0; k < K; ++k) {
    const int s = (int)(k % kBkStages);
    const uint32_t parity = (uint32_t)((k / kBkStages) & 1);
    if (!warp_wait_bounded(smem_addr(&bars[s]), parity)) {
      // Report, then wait (bounded) for this warp's other copies still in
      // flight so that none lands in shared memory after the CTA is gone.
      if (lane == 0) atomicAdd(&g_wait_timeouts, 1u);
      for (int64_t kk = k + 1; kk < K && kk < k + kBkStages; ++kk)
        warp_wait_bounded(smem_addr(&bars[kk % kBkStages]), (uint32_t)((kk / kBkStages) & 1));
      warp_wait_bounded(smem_addr(&bars[s]), parity);
      return;
    }
    const uint4* sx = s_rows + s * stage_chunks;
    uint4 v[VPL];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (c < a.nchunks) {
        v[j] = sx[c];
        if (MODE == kAdd) v[j] = add8(v[j], sx[a.nchunks + c]);
        if (MODE == kEmbed) v[j] = scale8(v[j], a.scale);
      }
    }
    __syncwarp();  // every lane has read stage s
    if (lane == 0 && k + kBkStages < K) {
      fence_proxy_async_smem();
      bk_issue<MODE>(a, s_rows + s * stage_chunks, smem_addr(&bars[s]), row0 + (k + kBkStages) * G, policy);
    }
    const int64_t base = (row0 + k * G) * a.nchunks;
    float p[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) p[e] = 0.0f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (c < a.nchunks) {
        if (MODE == kAdd || (MODE == kEmbed && a.r != nullptr)) st_stream(a.r + base + c, v[j]);
        accum8(p, v[j]);
      }
    }
    const float inv = inv_rms(ref_tree_bf16(p), a.hidden, a.eps);
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (c < a.nchunks) {
        uint4 wv = make_uint4(0, 0, 0, 0);
        if (HAS_W) wv = s_w[c];
        st_stream(a.y + base + c, norm8<HAS_W>(v[j], inv, wv));
      }
    }
  }
}

#endif  // HRM_RN_BULK

// ------------------------------------------------------------ fp32 fast path
struct RowArgsF32 {
  const float4* x;
  float4* y;
  const float4* w;
  int64_t rows;
  int nchunks;  // hidden / 4
  int hidden;
  float eps;
};

template <int VPL, bool HAS_W>
__global__ void __launch_bounds__(kThreads, min_blocks_for(HRM_RN_F32_MAXREGS)) rms_f32_warp_kernel(const RowArgsF32 a) {
  if (HRM_RN_PREFETCH) prefetch_warp_rows<float4>(a.x, nullptr, a.rows, a.nchunks);
  grid_dependency_begin();
  extern __shared__ uint4 s_w4[];
  float4* s_w = reinterpret_cast<float4*>(s_w4);
  const int lane = threadIdx.x & 31;
  if (HAS_W) issue_weight(s_w4, reinterpret_cast<const uint4*>(a.w), a.nchunks);

  const int nwarps = blockDim.x >> 5;  // kWarps, or fewer for a small launch
  const int64_t warp_stride = (int64_t)gridDim.x * nwarps;
  int64_t row = (int64_t)blockIdx.x * nwarps + (threadIdx.x >> 5);
  for (bool first = true; first || row < a.rows; first = false, row += warp_stride) {
    const bool active = row < a.rows;  // uniform across the warp
    const int64_t base = row * a.nchunks;
    float4 v[VPL];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (active && c < a.nchunks) v[j] = ld_l2(a.x + base + c);
    }
    float pa[4] = {0.f, 0.f, 0.f, 0.f}, pc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (active && c < a.nchunks) {
        float(&p)[4] = (j & 1) ? pc : pa;
        p[0] = fmaf(v[j].x, v[j].x, p[0]);
        p[1] = fmaf(v[j].y, v[j].y, p[1]);
        p[2] = fmaf(v[j].z, v[j].z, p[2]);
        p[3] = fmaf(v[j].w, v[j].w, p[3]);
      }
    }
    const float inv = inv_rms(ref_tree_f32(pa, pc), a.hidden, a.eps);
    if (HAS_W && first) publish_weight();
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int c = lane + 32 * j;
      if (active && c < a.nchunks) {
        float4 o = make_float4(v[j].x * inv, v[j].y * inv, v[j].z * inv, v[j].w * inv);
        if (HAS_W) {
          const float4 wv = s_w[c];
          o.x = o.x * wv.x; o.y = o.y * wv.y; o.z = o.z * wv.z; o.w = o.w * wv.w;
        }
        st_l2(a.y + base + c, o);
      }
    }
  }
}

// ----------------------------------------------------- fallback (any shape)
// One CTA of 256 threads per row, the reference's structure: strided
// accumulation, shuffle-down tree per warp, tree over the warp sums, then a
// second pass that produces the outputs.
struct RowArgsScalar {
  const void* x;         // T rows (kRms / kAdd) or bf16 table (kEmbed)
  const uint16_t* b;     // kAdd
  const uint32_t* ids;   // kEmbed
  uint16_t* r;           // kAdd residual / kEmbed hidden (nullable)
  void* y;               // T rows
  const void* w;         // T [hidden] or null
  int64_t rows;
  int64_t hidden;
  uint32_t vocab;
  float scale, eps;
};

template <typename T> __device__ __forceinline__ float load_t(const void* p, int64_t i);
template <> __device__ __forceinline__ float load_t<uint16_t>(const void* p, int64_t i) {
  return bf16_to_f32(static_cast<const uint16_t*>(p)[i]);
}
template <> __device__ __forceinline__ float load_t<float>(const void* p, int64_t i) {
  return static_cast<const float*>(p)[i];
}
template <typename T> __device__ __forceinline__ void store_t(void* p, int64_t i, float v);
template <> __device__ __forceinline__ void store_t<uint16_t>(void* p, int64_t i, float v) {
  static_cast<uint16_t*>(p)[i] = f32_to_bf16(v);
}
template <> __device__ __forceinline__ void store_t<float>(void* p, int64_t i, float v) {
  static_cast<float*>(p)[i] = v;
}

template <typename T, int MODE, bool HAS_W>
__global__ void __launch_bounds__(kBlockThreads) rownorm_block_kernel(const RowArgsScalar a) {
  grid_dependency_begin();
  __shared__ float s_sums[kBlockWarps];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const int64_t base = row * a.hidden;
    int64_t src = base;
    if (MODE == kEmbed) {
      uint32_t id = a.ids[row];
      if (id >= a.vocab) id = a.vocab - 1;
      src = (int64_t)id * a.hidden;
    }
    float local = 0.0f;
    for (int64_t i = tid; i < a.hidden; i += kBlockThreads) {
      float v;
      if (MODE == kAdd) {
        v = bf16_to_f32(f32_to_bf16(load_t<uint16_t>(a.x, base + i) + bf16_to_f32(a.b[base + i])));
        a.r[base + i] = f32_to_bf16(v);
      } else if (MODE == kEmbed) {
        v = bf16_to_f32(f32_to_bf16(load_t<uint16_t>(a.x, src + i) * a.scale));
        if (a.r != nullptr) a.r[base + i] = f32_to_bf16(v);
      } else {
        v = load_t<T>(a.x, base + i);
      }
      local = fmaf(v, v, local);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) local += __shfl_down_sync(0xffffffffu, local, off);
    if (lane == 0) s_sums[warp] = local;
    __syncthreads();
    if (warp == 0) {
      // Lane 0's result is the reference's tree over the 8 warp sums
      // (offsets 4, 2, 1); lanes >= 8 only feed lanes that are not used.
      float val = lane < kBlockWarps ? s_sums[lane] : 0.0f;
#pragma unroll
      for (int off = kBlockWarps / 2; off > 0; off >>= 1) val += __shfl_down_sync(0xffffffffu, val, off);
      if (lane == 0) s_sums[0] = val;
    }
    __syncthreads();
    const float inv = inv_rms(s_sums[0], (int)a.hidden, a.eps);
    __syncthreads();  // s_sums is rewritten by the next row
    for (int64_t i = tid; i < a.hidden; i += kBlockThreads) {
      float v;
      if (MODE == kAdd) {
        v = bf16_to_f32(a.r[base + i]);  // written above by this same thread
      } else if (MODE == kEmbed) {
        v = bf16_to_f32(f32_to_bf16(load_t<uint16_t>(a.x, src + i) * a.scale));
      } else {
        v = load_t<T>(a.x, base + i);
      }
      float o = v * inv;
      if (HAS_W) o = o * load_t<T>(a.w, i);
      store_t<T>(a.y, base + i, o);
    }
  }
}

// ------------------------------------------------------------ dispatch
template <typename K>
int resident_ctas(K kernel, size_t smem, int threads = kThreads) {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess || n < 1) {
    cudaGetLastError();
    n = 1;
  }
  return n;
}

// Resident CTAs per SM of one warp-kernel instantiation (shared memory of at
// most 8 KB never limits it), cached.
template <int VPL, int MODE, bool HAS_W, int REGS, int WARPS>
int warp_occupancy() {
  static std::atomic<int> occ{0};
  int o = occ.load(std::memory_order_relaxed);
  if (o == 0) {
    o = resident_ctas(rownorm_warp_kernel<VPL, MODE, HAS_W, REGS, WARPS>, (size_t)kMaxVpl * 32 * 16, 32 * WARPS);
    occ.store(o, std::memory_order_relaxed);
  }
  return o;
}

inline int64_t warp_blocks(const RowArgs& a, int max_warps) {
  const int nw = warps_per_cta(a.rows, max_warps);
  return (a.rows + nw - 1) / nw;
}

template <int VPL, int MODE, bool HAS_W, int REGS = rownorm_max_regs<VPL, MODE>(), int WARPS = kWarps>
cudaError_t launch_warp_on(const RowArgs& a, cudaStream_t s) {
  cudaError_t err = cudaSuccess;
  auto kernel = rownorm_warp_kernel<VPL, MODE, HAS_W, REGS, WARPS>;
  const int o = warp_occupancy<VPL, MODE, HAS_W, REGS, WARPS>();
  const size_t smem = HAS_W ? (size_t)a.nchunks * 16 : 0;
  const int nw = warps_per_cta(a.rows, WARPS);
  int64_t blocks = warp_blocks(a, WARPS);
  const int64_t wave = (int64_t)device_sm_count() * o;
  if (HRM_RN_WAVES > 0 && blocks > wave * HRM_RN_WAVES) blocks = wave * HRM_RN_WAVES;
  if (blocks > INT32_MAX) blocks = INT32_MAX;
  err = launch_kernel(kernel, blocks, 32 * nw, smem, s, a);
  return err;
}

template <int MODE, bool HAS_W>
cudaError_t dispatch_vpl(const RowArgs& a, cudaStream_t s) {
  const int need = (a.nchunks + 31) / 32;
  if (need <= 1) return launch_warp_on<1, MODE, HAS_W>(a, s);
  if (need <= 2) return launch_warp_on<2, MODE, HAS_W>(a, s);
  if (need <= 4) return launch_warp_on<4, MODE, HAS_W>(a, s);
  if (need <= 6) return launch_warp_on<6, MODE, HAS_W>(a, s);
  if (need <= 8) {
    if constexpr (MODE == kRms && HRM_RN_NORM8_MAXREGS < HRM_RN_MAXREGS) {
      // the capped shape only where the launch fits in one wave of it
      constexpr int kW = HRM_RN_NORM8_WARPS;
      if (warp_blocks(a, kW) <= (int64_t)device_sm_count() * warp_occupancy<8, MODE, HAS_W, HRM_RN_NORM8_MAXREGS, kW>())
        return launch_warp_on<8, MODE, HAS_W, HRM_RN_NORM8_MAXREGS, kW>(a, s);
    }
    return launch_warp_on<8, MODE, HAS_W>(a, s);
  }
  return launch_warp_on<16, MODE, HAS_W>(a, s);
}

#if HRM_RN_BULK
// Opt-in dynamic shared memory per CTA of the current device, cached per device.
int smem_optin_bytes() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  int v = (dev >= 0 && dev < 64) ? cache[dev].load(std::memory_order_relaxed) : 0;
  if (v > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || v <= 0) {
    cudaGetLastError();
    v = 48 * 1024;
  }
  if (dev >= 0 && dev < 64) cache[dev].store(v, std::memory_order_relaxed);
  return v;
}

// Warps per CTA of the bulk path (as many stage rings as fit, at most
// kBkMaxWarps) and the dynamic shared memory they need; 0 warps: no fit.
int bulk_plan(int nchunks, int rows_per_stage, bool has_w, size_t* smem) {
  size_t cap = (size_t)smem_optin_bytes();
  if (HRM_BK_CTAS > 1) {  // per-SM capacity shared by HRM_BK_CTAS CTAs, 1 KB reserved each
    const size_t per_cta = (233472 - 1024 * (size_t)HRM_BK_CTAS) / HRM_BK_CTAS;
    if (per_cta < cap) cap = per_cta;
  }
  const size_t wbytes = has_w ? (size_t)nchunks * 16 : 0;
  const size_t per_warp = (size_t)kBkStages * ((size_t)rows_per_stage * nchunks * 16 + 8);
  if (cap <= wbytes) return 0;
  size_t w = (cap - wbytes) / per_warp;
  if (w > (size_t)kBkMaxWarps) w = kBkMaxWarps;
  *smem = wbytes + w * per_warp;
  return (int)w;
}

template <int VPL, int MODE, bool HAS_W>
cudaError_t launch_bulk_on(const RowArgs& a, int nwarps, size_t smem, cudaStream_t s) {
  cudaError_t err = cudaSuccess;
  auto kernel = rownorm_bulk_kernel<VPL, MODE, HAS_W>;
  static std::atomic<bool> opted[64];  // per device: the opt-in is per function and device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  if (dev < 0 || dev >= 64 || !opted[dev].load(std::memory_order_relaxed)) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_optin_bytes());
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) opted[dev].store(true, std::memory_order_relaxed);
  }
  int64_t blocks;
  if (kBkRows > 0) {
    const int64_t rows_per_cta = (int64_t)nwarps * kBkRows;
    blocks = (a.rows + rows_per_cta - 1) / rows_per_cta;
  } else {
    blocks = (a.rows + nwarps - 1) / nwarps;
    const int64_t sms = device_sm_count();
    if (blocks > sms) blocks = sms;  // one CTA per SM, warps loop over their rows
  }
  if (blocks > INT32_MAX) blocks = INT32_MAX;
  err = launch_kernel(kernel, blocks, 32 * nwarps, smem, s, a);
  return err;
}

template <int MODE, bool HAS_W>
cudaError_t dispatch_bulk(const RowArgs& a, int nwarps, size_t smem, cudaStream_t s) {
  const int need = (a.nchunks + 31) / 32;
  if (need <= 1) return launch_bulk_on<1, MODE, HAS_W>(a, nwarps, smem, s);
  if (need <= 2) return launch_bulk_on<2, MODE, HAS_W>(a, nwarps, smem, s);
  if (need <= 4) return launch_bulk_on<4, MODE, HAS_W>(a, nwarps, smem, s);
  if (need <= 6) return launch_bulk_on<6, MODE, HAS_W>(a, nwarps, smem, s);
  if (need <= 8) return launch_bulk_on<8, MODE, HAS_W>(a, nwarps, smem, s);
  return launch_bulk_on<16, MODE, HAS_W>(a, nwarps, smem, s);
}

#endif  // HRM_RN_BULK

template <typename T, int MODE, bool HAS_W>
cudaError_t launch_block(const RowArgsScalar& a, cudaStream_t s) {
  cudaError_t err = cudaSuccess;
  int64_t blocks = a.rows;
  const int64_t cap = (int64_t)device_sm_count() * 64;
  if (blocks > cap) blocks = cap;
  err = launch_kernel(rownorm_block_kernel<T, MODE, HAS_W>, blocks, kBlockThreads, 0, s, a);
  return err;
}

template <int MODE>
cudaError_t launch_bf16_rows(const void* x, const void* b, const uint32_t* ids, void* r, void* y, const void* w,
                             int64_t rows, int64_t hidden, int64_t vocab, float scale, float eps, cudaStream_t s) {
  const bool fast = hidden % 8 == 0 && hidden / 8 <= kMaxVpl * 32 && aligned16(x) && aligned16(y) &&
                    (b == nullptr || aligned16(b)) && (r == nullptr || aligned16(r)) &&
                    (w == nullptr || aligned16(w));
  if (fast) {
    RowArgs a;
    a.x = static_cast<const uint4*>(x);
    a.b = static_cast<const uint4*>(b);
    a.ids = ids;
    a.r = static_cast<uint4*>(r);
    a.y = static_cast<uint4*>(y);
    a.w = static_cast<const uint4*>(w);
    a.rows = rows;
    a.nchunks = (int)(hidden / 8);
    a.hidden = (int)hidden;
    a.vocab = (uint32_t)vocab;
    a.scale = scale;
    a.eps = eps;
    if (HRM_RN_CTA_ROWS_PER_SM > 0 && a.nchunks >= HRM_RN_CTA_MIN_CHUNKS &&
        rows <= (int64_t)device_sm_count() * HRM_RN_CTA_ROWS_PER_SM) {
      const int threads = (a.nchunks + 31) / 32 * 32;
      return w ? launch_kernel(rownorm_cta_kernel<MODE, true>, rows, threads, 0, s, a)
               : launch_kernel(rownorm_cta_kernel<MODE, false>, rows, threads, 0, s, a);
    }
#if HRM_RN_BULK
    size_t smem = 0;
    const int nwarps = bulk_plan(a.nchunks, MODE == kAdd ? 2 : 1, w != nullptr, &smem);
    if (nwarps >= 1)
      return w ? dispatch_bulk<MODE, true>(a, nwarps, smem, s) : dispatch_bulk<MODE, false>(a, nwarps, smem, s);
#endif
    return w ? dispatch_vpl<MODE, true>(a, s) : dispatch_vpl<MODE, false>(a, s);
  }
  RowArgsScalar a;
  a.x = x;
  a.b = static_cast<const uint16_t*>(b);
  a.ids = ids;
  a.r = static_cast<uint16_t*>(r);
  a.y = y;
  a.w = w;
  a.rows = rows;
  a.hidden = hidden;
  a.vocab = (uint32_t)vocab;
  a.scale = scale;
  a.eps = eps;
  return w ? launch_block<uint16_t, MODE, true>(a, s) : launch_block<uint16_t, MODE, false>(a, s);
}

template <int VPL, bool HAS_W>
cudaError_t launch_f32_warp(const RowArgsF32& a, cudaStream_t s) {
  cudaError_t err = cudaSuccess;
  auto kernel = rms_f32_warp_kernel<VPL, HAS_W>;
  static std::atomic<int> occ{0};
  int o = occ.load(std::memory_order_relaxed);
  if (o == 0) {
    o = resident_ctas(kernel, (size_t)kMaxVpl * 32 * 16);
    occ.store(o, std::memory_order_relaxed);
  }
  const size_t smem = HAS_W ? (size_t)a.nchunks * 16 : 0;
  const int nw = warps_per_cta(a.rows, kWarps);
  int64_t blocks = (a.rows + nw - 1) / nw;
  const int64_t wave = (int64_t)device_sm_count() * o;
  // Option: a launch of one to two waves takes two rows per warp (rows w and
  // w + G, both prefetched before the dependency wait), which makes it one
  // wave (prefetching only the first row of the two was slower still).
  if (HRM_RN_F32_TWO_ROWS && blocks > wave && (blocks + 1) / 2 <= wave) blocks = (blocks + 1) / 2;
  if (HRM_RN_F32_WAVES > 0 && blocks > wave * HRM_RN_F32_WAVES) blocks = wave * HRM_RN_F32_WAVES;
  if (blocks > INT32_MAX) blocks = INT32_MAX;
  err = launch_kernel(kernel, blocks, 32 * nw, smem, s, a);
  return err;
}

template <bool HAS_W>
cudaError_t dispatch_f32(const RowArgsF32& a, cudaStream_t s) {
  const int need = (a.nchunks + 31) / 32;
  if (need <= 1) return launch_f32_warp<1, HAS_W>(a, s);
  if (need <= 2) return launch_f32_warp<2, HAS_W>(a, s);
  if (need <= 4) return launch_f32_warp<4, HAS_W>(a, s);
  if (need <= 8) return launch_f32_warp<8, HAS_W>(a, s);
  return launch_f32_warp<16, HAS_W>(a, s);
}

}  // namespace

cudaError_t rownorm_wait_timeouts(unsigned int* count, bool reset) {
  cudaError_t e = cudaMemcpyFromSymbol(count, g_wait_timeouts, sizeof(unsigned int));
  if (e == cudaSuccess && reset) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_wait_timeouts, &zero, sizeof(unsigned int));
  }
  return e;
}

cudaError_t launch_rms_norm_bf16(const void* x, void* y, const void* w, int64_t rows, int64_t hidden, float eps,
                                 cudaStream_t s) {
  return launch_bf16_rows<kRms>(x, nullptr, nullptr, nullptr, y, w, rows, hidden, 0, 1.0f, eps, s);
}

cudaError_t launch_add_rms_norm(const void* x, const void* b, void* r, void* y, const void* w, int64_t rows,
                                int64_t hidden, float eps, cudaStream_t s) {
  return launch_bf16_rows<kAdd>(x, b, nullptr, r, y, w, rows, hidden, 0, 1.0f, eps, s);
}

cudaError_t launch_embed_rms_norm(const uint32_t* ids, const void* table, void* h, void* y, const void* w,
                                  int64_t rows, int64_t hidden, int64_t vocab, float scale, float eps,
                                  cudaStream_t s) {
  return launch_bf16_rows<kEmbed>(table, nullptr, ids, h, y, w, rows, hidden, vocab, scale, eps, s);
}

cudaError_t launch_rms_norm_f32(const float* x, float* y, const float* w, int64_t rows, int64_t hidden, float eps,
                                cudaStream_t s) {
  const bool fast = hidden % 4 == 0 && hidden / 4 <= kMaxVpl * 32 && aligned16(x) && aligned16(y) &&
                    (w == nullptr || aligned16(w));
  if (fast) {
    RowArgsF32 a;
    a.x = reinterpret_cast<const float4*>(x);
    a.y = reinterpret_cast<float4*>(y);
    a.w = reinterpret_cast<const float4*>(w);
    a.rows = rows;
    a.nchunks = (int)(hidden / 4);
    a.hidden = (int)hidden;
    a.eps = eps;
    return w ? dispatch_f32<true>(a, s) : dispatch_f32<false>(a, s);
  }
  RowArgsScalar a;
  a.x = x;
  a.b = nullptr;
  a.ids = nullptr;
  a.r = nullptr;
  a.y = y;
  a.w = w;
  a.rows = rows;
  a.hidden = hidden;
  a.vocab = 0;
  a.scale = 1.0f;
  a.eps = eps;
  return w ? launch_block<float, kRms, true>(a, s) : launch_block<float, kRms, false>(a, s);
}

}  // namespace hrm
