// Rotary position embedding, in place on Q and K ([batch, heads, seq, head_dim]
// bf16 as the reference lays them out, or token-major [batch, seq, heads,
// head_dim]), rotate-half pairing (x[i], x[i + head_dim/2]) as in
// src/kernels/rope_embed.cu:36-53.
//
// Fast path (head_dim % 16 == 0, head_dim <= 512, 16-byte aligned): a thread
// owns 8 consecutive pairs of one row -- one 16-byte chunk of the low half and
// the matching chunk of the high half -- so g = head_dim / 16 threads cover a
// row (8 for head_dim 128).  A 128-thread CTA tile is pt positions x ht head
// slices x g; each thread fetches the cos/sin of its 8 pairs at its position
// once and reuses them for every head it visits (h = slice, slice + ht, ...)
// and for both Q and K, so the angle work / table traffic is amortised over
// 2 * heads / ht rows.  Prefill tiles are 4 positions x 4 head slices (a
// thread visits 4 of the 16 heads, two in flight at a time); decode (seq 1)
// tiles are 1 position x 16 slices.  One CTA per tile.  Measured on B200
// (in-place Q/K [16, 16, 4096, 128]): 6.59 TB/s, against 6.47 for 16
// positions x 1 slice and 6.58 for 1 position x 16 slices at 8 CTAs/SM.
// HRM_ROPE_UNROLL heads' worth of loads (4 x 16 B each) are in flight before
// any store.
//
// Angles: either the fp32 table written by rope_table_kernel or, with no
// table, evaluated in the kernel with exactly the reference expression
//   (float)(s + offset) * expf(-2.0f * i * logf(theta) / (float)head_dim)
// and sincosf (src/kernels/rope_embed.cu:41-43), each of a tile's distinct
// angles once, shared through shared memory (tile_angles).  The table is
// built with that same expression, so both ways give the reference's cos/sin
// bit for bit.
// The rotation is written with explicit roundings in the forms nvcc gives the
// reference's source (src/kernels/rope_embed.cu:45-53), established by
// running the reference kernel against every candidate rounding:
//   q: x0' = fma(x0, c, -(x1 * s)),  x1' = fma(x1, c, x0 * s)
//   k: x0' = fma(x0, c, -(x1 * s)),  x1' = fma(x0, s, x1 * c)
// (the identical source expression contracts one way for q and the other for
// k).  Left to contraction, the same expressions compile differently here and
// round differently in ~2e-5 of the outputs.
#include "common.cuh"
#include "launch.h"

namespace hrm {
namespace {

// Launch shape of the tiled kernel (compile-time; defaults tuned):
//   HRM_ROPE_UNROLL     heads whose Q/K chunks are loaded before any is used
//   HRM_ROPE_CAP        grid cap in CTAs per SM (0: one CTA per tile)
//   HRM_ROPE_MINBLOCKS  __launch_bounds__ minimum resident CTAs per SM
#ifndef HRM_ROPE_UNROLL
#define HRM_ROPE_UNROLL 2
#endif
#ifndef HRM_ROPE_CAP
#define HRM_ROPE_CAP 0
#endif
#ifndef HRM_ROPE_MINBLOCKS
#define HRM_ROPE_MINBLOCKS 1
#endif
//   HRM_ROPE_MAX_PT     positions per tile at most (the rest of the 128 threads
//                       become head slices)
#ifndef HRM_ROPE_MAX_PT
#define HRM_ROPE_MAX_PT 4
#endif

constexpr int kThreads = 128;
constexpr int kHeadUnroll = HRM_ROPE_UNROLL;

struct RopeArgs {
  uint4* q;
  uint4* k;
  // 16-byte-chunk strides of a (batch, position, head) row start:
  // [b, h, s, d]: heads * seq * rc, rc, seq * rc; [b, s, h, d]: seq * heads * rc, heads * rc, rc
  int64_t batch_stride, pos_stride, head_stride;
  const float4* table;  // [positions][head_dim] floats: cos in [0, hd/2), sin in [hd/2, hd)
  int64_t seq;
  int tiles_per_batch;  // tile counts fit 31 bits (checked at launch): 32-bit index math
  int ntiles;
  int heads;
  int head_dim;
  int g;   // threads per row (= chunks per half-row), a power of two
  int pt;  // positions per tile, a power of two
  int ht;  // head slices per tile, a power of two
  int lg, lht;  // log2(g), log2(ht)
  int offset;
  float theta;
};

__device__ __forceinline__ float rope_angle(int pos, int i, int head_dim, float theta) {
  return (float)pos * expf(-2.0f * i * logf(theta) / (float)head_dim);
}

// x0' and x1' of one pair, rounded as the reference kernel rounds them.
__device__ __forceinline__ float rot_lo(float x0, float x1, float c, float s) {
  return __fmaf_rn(x0, c, -__fmul_rn(x1, s));
}
__device__ __forceinline__ float rot_hi_q(float x0, float x1, float c, float s) {
  return __fmaf_rn(x1, c, __fmul_rn(x0, s));
}
__device__ __forceinline__ float rot_hi_k(float x0, float x1, float c, float s) {
  return __fmaf_rn(x0, s, __fmul_rn(x1, c));
}

template <bool IS_K>
__device__ __forceinline__ void rotate8(uint4& lo, uint4& hi, const float (&c)[8], const float (&s)[8]) {
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t wl = vget(lo, w), wh = vget(hi, w);
    const float x0a = bf16_lo(wl), x0b = bf16_hi(wl);
    const float x1a = bf16_lo(wh), x1b = bf16_hi(wh);
    const float ca = c[2 * w], sa = s[2 * w], cb = c[2 * w + 1], sb = s[2 * w + 1];
    vset(lo, w, pack_bf16x2(rot_lo(x0a, x1a, ca, sa), rot_lo(x0b, x1b, cb, sb)));
    if (IS_K)
      vset(hi, w, pack_bf16x2(rot_hi_k(x0a, x1a, ca, sa), rot_hi_k(x0b, x1b, cb, sb)));
    else
      vset(hi, w, pack_bf16x2(rot_hi_q(x0a, x1a, ca, sa), rot_hi_q(x0b, x1b, cb, sb)));
  }
}

// cos/sin of pairs 8j..8j+7 at position pos from the table.
__device__ __forceinline__ void table_cos_sin(const float4* table, int pos, int j, int head_dim, float (&c)[8],
                                              float (&sn)[8]) {
  const float4* row = table + (int64_t)pos * (head_dim / 4);
  const float4 c0 = ld_keep(row + 2 * j), c1 = ld_keep(row + 2 * j + 1);
  const float4 s0 = ld_keep(row + head_dim / 8 + 2 * j), s1 = ld_keep(row + head_dim / 8 + 2 * j + 1);
  c[0] = c0.x; c[1] = c0.y; c[2] = c0.z; c[3] = c0.w; c[4] = c1.x; c[5] = c1.y; c[6] = c1.z; c[7] = c1.w;
  sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w; sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
}

// In-kernel angles (no table): the tile's distinct (position, pair) angles
// are shared out -- each of the CTA's threads evaluates one at a time, with
// the reference expression and sincosf, into shared memory -- instead of every
// thread evaluating the 8 of its own pairs, which all the tile's head slices
// repeat.  A decode tile (1 position, 64 pairs for head_dim 128) thus costs
// one sincosf per thread instead of 8.  Positions past seq are skipped.
constexpr int kMaxAngles = HRM_ROPE_MAX_PT * 256;  // tile positions x pairs (head_dim <= 512)

__device__ __forceinline__ void tile_angles(float* s_cos, float* s_sin, int64_t s_base, int64_t seq, int pt,
                                            int lhalf, int offset, int head_dim, float theta) {
  const int half = 1 << lhalf;
  for (int idx = threadIdx.x; idx < (pt << lhalf); idx += blockDim.x) {
    const int p = idx >> lhalf, i = idx & (half - 1);
    if (s_base + p < seq) sincosf(rope_angle((int)(s_base + p) + offset, i, head_dim, theta), &s_sin[idx], &s_cos[idx]);
  }
}

__device__ __forceinline__ void shared_cos_sin(const float* s_cos, const float* s_sin, int pl, int j, int lhalf,
                                               float (&c)[8], float (&sn)[8]) {
  const float4* cr = reinterpret_cast<const float4*>(s_cos + (pl << lhalf) + 8 * j);
  const float4* sr = reinterpret_cast<const float4*>(s_sin + (pl << lhalf) + 8 * j);
  const float4 c0 = cr[0], c1 = cr[1], s0 = sr[0], s1 = sr[1];
  c[0] = c0.x; c[1] = c0.y; c[2] = c0.z; c[3] = c0.w; c[4] = c1.x; c[5] = c1.y; c[6] = c1.z; c[7] = c1.w;
  sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w; sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
}

// First position of a tile and its batch index (32-bit: tile counts fit 31 bits).
template <typename Args>
__device__ __forceinline__ int64_t tile_first_pos(const Args& a, int tile, int& bi) {
  bi = tile / a.tiles_per_batch;
  return (int64_t)(tile - bi * a.tiles_per_batch) * a.pt;
}

// In-kernel angles of the CTA's first tile, evaluated before the grid
// dependency wait: they depend on the launch arguments only (positions,
// offset, theta), so their expf / logf / sincosf latency overlaps the previous
// kernel's drain instead of preceding this kernel's loads.  Published by the
// barrier at the top of the first tile.
template <typename Args>
__device__ __forceinline__ void first_tile_angles(const Args& a, float* s_cos, float* s_sin) {
  if ((int)blockIdx.x >= a.ntiles) return;
  int bi;
  const int64_t s_base = tile_first_pos(a, (int)blockIdx.x, bi);
  tile_angles(s_cos, s_sin, s_base, a.seq, a.pt, a.lg + 3, a.offset, a.head_dim, a.theta);
}

// Thread layout within a tile (g, ht powers of two): lane j of its row, head
// slice, position in the tile.  Shifts and masks, and 32-bit tile arithmetic:
// at decode sizes a launch is a handful of CTAs whose time is latency, where a
// 64-bit division costs a visible fraction.
template <bool TABLE>
__global__ void __launch_bounds__(kThreads, HRM_ROPE_MINBLOCKS) rope_tile_kernel(const RopeArgs a) {
  __shared__ __align__(16) float s_cos[TABLE ? 1 : kMaxAngles], s_sin[TABLE ? 1 : kMaxAngles];
  if (!TABLE) first_tile_angles(a, s_cos, s_sin);
  grid_dependency_begin();
  const int j = threadIdx.x & (a.g - 1);
  const int rest = threadIdx.x >> a.lg;
  const int slice = rest & (a.ht - 1);
  const int pl = rest >> a.lht;

  for (int tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x) {
    int bi;
    const int64_t s_base = tile_first_pos(a, tile, bi);
    const int64_t b = bi;
    const int64_t s = s_base + pl;
    if (!TABLE) {
      if (tile != (int)blockIdx.x) {
        __syncthreads();  // the previous tile's angles are no longer read
        tile_angles(s_cos, s_sin, s_base, a.seq, a.pt, a.lg + 3, a.offset, a.head_dim, a.theta);
      }
      __syncthreads();
    }
    if (s >= a.seq) continue;
    const int pos = (int)s + a.offset;

    float c[8], sn[8];
    if (TABLE)
      table_cos_sin(a.table, pos, j, a.head_dim, c, sn);
    else
      shared_cos_sin(s_cos, s_sin, pl, j, a.lg + 3, c, sn);

    const int64_t head_step = a.head_stride;
    const int64_t row0 = b * a.batch_stride + s * a.pos_stride + j;
    int h = slice;
    for (; h + (kHeadUnroll - 1) * a.ht < a.heads; h += kHeadUnroll * a.ht) {
      uint4 ql[kHeadUnroll], qh[kHeadUnroll], kl[kHeadUnroll], kh[kHeadUnroll];
#pragma unroll
      for (int u = 0; u < kHeadUnroll; ++u) {
        const int64_t lo = row0 + (int64_t)(h + u * a.ht) * head_step;
        ql[u] = ld_stream(a.q + lo);
        qh[u] = ld_stream(a.q + lo + a.g);
        kl[u] = ld_stream(a.k + lo);
        kh[u] = ld_stream(a.k + lo + a.g);
      }
#pragma unroll
      for (int u = 0; u < kHeadUnroll; ++u) {
        const int64_t lo = row0 + (int64_t)(h + u * a.ht) * head_step;
        rotate8<false>(ql[u], qh[u], c, sn);
        rotate8<true>(kl[u], kh[u], c, sn);
        st_stream(a.q + lo, ql[u]);
        st_stream(a.q + lo + a.g, qh[u]);
        st_stream(a.k + lo, kl[u]);
        st_stream(a.k + lo + a.g, kh[u]);
      }
    }
    for (; h < a.heads; h += a.ht) {
      const int64_t lo = row0 + (int64_t)h * head_step;
      uint4 ql = ld_stream(a.q + lo), qh = ld_stream(a.q + lo + a.g);
      uint4 kl = ld_stream(a.k + lo), kh = ld_stream(a.k + lo + a.g);
      rotate8<false>(ql, qh, c, sn);
      rotate8<true>(kl, kh, c, sn);
      st_stream(a.q + lo, ql);
      st_stream(a.q + lo + a.g, qh);
      st_stream(a.k + lo, kl);
      st_stream(a.k + lo + a.g, kh);
    }
  }
}

// Any even head_dim / alignment: one thread per pair, as the reference maps
// its threads (src/kernels/rope_embed.cu:22-37), with 64-bit indexing.
// Rows enumerate (b, h, s) for [b, h, s, d] (heads_inner = 1) or (b, s, h)
// for [b, s, h, d] (heads_inner = heads).
__global__ void __launch_bounds__(256) rope_scalar_kernel(uint16_t* q, uint16_t* k, int64_t rows, int64_t seq,
                                                          int64_t heads_inner, int head_dim, int offset,
                                                          float theta, const float* table) {
  grid_dependency_begin();
  const int half = head_dim / 2;
  const int64_t total = rows * half;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    const int i = (int)(idx % half);
    const int64_t row = idx / half;
    const int pos = (int)((row / heads_inner) % seq) + offset;
    float c, s;
    if (table != nullptr) {
      c = table[(int64_t)pos * head_dim + i];
      s = table[(int64_t)pos * head_dim + half + i];
    } else {
      sincosf(rope_angle(pos, i, head_dim, theta), &s, &c);
    }
    const int64_t i0 = row * head_dim + i, i1 = i0 + half;
    const float x0 = bf16_to_f32(q[i0]), x1 = bf16_to_f32(q[i1]);
    q[i0] = f32_to_bf16(rot_lo(x0, x1, c, s));
    q[i1] = f32_to_bf16(rot_hi_q(x0, x1, c, s));
    const float k0 = bf16_to_f32(k[i0]), k1 = bf16_to_f32(k[i1]);
    k[i0] = f32_to_bf16(rot_lo(k0, k1, c, s));
    k[i1] = f32_to_bf16(rot_hi_k(k0, k1, c, s));
  }
}

__global__ void __launch_bounds__(256) rope_table_kernel(float* table, int64_t positions, int head_dim,
                                                         float theta) {
  grid_dependency_begin();
  const int half = head_dim / 2;
  const int64_t total = positions * half;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    const int i = (int)(idx % half);
    const int64_t p = idx / half;
    float s, c;
    sincosf(rope_angle((int)p, i, head_dim, theta), &s, &c);
    table[p * head_dim + i] = c;
    table[p * head_dim + half + i] = s;
  }
}

// ---------------------------------------------------- split + RoPE + cache
// The attention prologue of the reference reads the projection output
// [batch, seq, 4*heads*head_dim] three times over three kernels (split_gqkv,
// rope_embed, kv_cache_update).  Here one thread moves, per head it visits,
// the 8 pairs it owns of all four segments: gate and v are copied, q and k
// rotated with the cos/sin it fetched once, and k / v also go to the cache.
// Same tile shape as rope_tile_kernel.
struct SplitArgs {
  const uint4* gqkv;
  uint4* gate;
  uint4* q;
  uint4* k;
  uint4* v;
  uint4* kc;  // k cache or null
  uint4* vc;  // v cache or null
  const float4* table;
  int64_t seq;
  int tiles_per_batch;  // 31-bit tile counts, as RopeArgs
  int ntiles;
  int64_t cache_len;
  int64_t cache_offset;
  int heads;
  int head_dim;
  int g, pt, ht;
  int lg, lht;  // log2(g), log2(ht)
  int offset;
  float theta;
};

// Loads and stores with the default L2 priority (ld_l2 / st_l2): 6.42 -> 6.48
// TB/s over 65536 tokens with the cache on B200 against evict-first (the
// stores alone with default priority measured 6.34).
template <bool TABLE, bool CACHE>
__global__ void __launch_bounds__(kThreads, HRM_ROPE_MINBLOCKS) split_rope_tile_kernel(const SplitArgs a) {
  __shared__ __align__(16) float s_cos[TABLE ? 1 : kMaxAngles], s_sin[TABLE ? 1 : kMaxAngles];
  if (!TABLE) first_tile_angles(a, s_cos, s_sin);
  grid_dependency_begin();
  const int j = threadIdx.x & (a.g - 1);
  const int rest = threadIdx.x >> a.lg;
  const int slice = rest & (a.ht - 1);
  const int pl = rest >> a.lht;
  const int row_chunks = 2 * a.g;                       // 16-byte chunks per head row
  const int64_t seg = (int64_t)a.heads * row_chunks;   // chunks per gqkv segment

  for (int tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x) {
    int bi;
    const int64_t s_base = tile_first_pos(a, tile, bi);
    const int64_t b = bi;
    const int64_t s = s_base + pl;
    if (!TABLE) {
      if (tile != (int)blockIdx.x) {
        __syncthreads();  // the previous tile's angles are no longer read
        tile_angles(s_cos, s_sin, s_base, a.seq, a.pt, a.lg + 3, a.offset, a.head_dim, a.theta);
      }
      __syncthreads();
    }
    if (s >= a.seq) continue;
    float c[8], sn[8];
    if (TABLE)
      table_cos_sin(a.table, (int)s + a.offset, j, a.head_dim, c, sn);
    else
      shared_cos_sin(s_cos, s_sin, pl, j, a.lg + 3, c, sn);

    const int64_t tok = b * a.seq + s;
    const int64_t in0 = tok * 4 * seg + j;                              // + h * row_chunks
    const int64_t gate0 = tok * seg + j;                                // + h * row_chunks
    const int64_t out0 = ((b * a.heads) * a.seq + s) * row_chunks + j;  // + h * out_step
    const int64_t out_step = a.seq * row_chunks;
    const int64_t c0 = ((b * a.heads) * a.cache_len + a.cache_offset + s) * row_chunks + j;
    const int64_t c_step = a.cache_len * row_chunks;
    for (int h = slice; h < a.heads; h += a.ht) {
      const int64_t src = in0 + (int64_t)h * row_chunks;
      const uint4 gl = ld_l2(a.gqkv + src), gh = ld_l2(a.gqkv + src + a.g);
      uint4 ql = ld_l2(a.gqkv + src + seg), qh = ld_l2(a.gqkv + src + seg + a.g);
      uint4 kl = ld_l2(a.gqkv + src + 2 * seg), kh = ld_l2(a.gqkv + src + 2 * seg + a.g);
      const uint4 vl = ld_l2(a.gqkv + src + 3 * seg), vh = ld_l2(a.gqkv + src + 3 * seg + a.g);
      rotate8<false>(ql, qh, c, sn);
      rotate8<true>(kl, kh, c, sn);
      const int64_t go = gate0 + (int64_t)h * row_chunks, o = out0 + (int64_t)h * out_step;
      st_l2(a.gate + go, gl);
      st_l2(a.gate + go + a.g, gh);
      st_l2(a.q + o, ql);
      st_l2(a.q + o + a.g, qh);
      st_l2(a.k + o, kl);
      st_l2(a.k + o + a.g, kh);
      st_l2(a.v + o, vl);
      st_l2(a.v + o + a.g, vh);
      if (CACHE) {
        const int64_t co = c0 + (int64_t)h * c_step;
        st_l2(a.kc + co, kl);
        st_l2(a.kc + co + a.g, kh);
        st_l2(a.vc + co, vl);
        st_l2(a.vc + co + a.g, vh);
      }
    }
  }
}

// Any even head_dim / alignment: one thread per (b, h, s, pair).
__global__ void __launch_bounds__(256) split_rope_scalar_kernel(
    const uint16_t* gqkv, uint16_t* gate, uint16_t* q, uint16_t* k, uint16_t* v, uint16_t* kc, uint16_t* vc,
    int64_t batch, int64_t seq, int heads, int head_dim, int offset, float theta, const float* table,
    int64_t cache_len, int64_t cache_offset) {
  grid_dependency_begin();
  const int half = head_dim / 2;
  const int64_t total = batch * heads * seq * half;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    const int i = (int)(idx % half);
    const int64_t r = idx / half;
    const int64_t s = r % seq;
    const int64_t bh = r / seq;
    const int h = (int)(bh % heads);
    const int64_t b = bh / heads;
    const int pos = (int)s + offset;
    float c, sn;
    if (table != nullptr) {
      c = table[(int64_t)pos * head_dim + i];
      sn = table[(int64_t)pos * head_dim + half + i];
    } else {
      sincosf(rope_angle(pos, i, head_dim, theta), &sn, &c);
    }
    const int64_t tok = b * seq + s;
    const int64_t in = tok * 4 * heads * head_dim + (int64_t)h * head_dim + i;
    const int64_t segd = (int64_t)heads * head_dim;
    const int64_t go = (tok * heads + h) * head_dim + i;
    const int64_t o = ((b * heads + h) * seq + s) * head_dim + i;
    gate[go] = gqkv[in];
    gate[go + half] = gqkv[in + half];
    const float x0 = bf16_to_f32(gqkv[in + segd]), x1 = bf16_to_f32(gqkv[in + segd + half]);
    q[o] = f32_to_bf16(rot_lo(x0, x1, c, sn));
    q[o + half] = f32_to_bf16(rot_hi_q(x0, x1, c, sn));
    const float k0 = bf16_to_f32(gqkv[in + 2 * segd]), k1 = bf16_to_f32(gqkv[in + 2 * segd + half]);
    const uint16_t klo = f32_to_bf16(rot_lo(k0, k1, c, sn)), khi = f32_to_bf16(rot_hi_k(k0, k1, c, sn));
    k[o] = klo;
    k[o + half] = khi;
    const uint16_t vlo = gqkv[in + 3 * segd], vhi = gqkv[in + 3 * segd + half];
    v[o] = vlo;
    v[o + half] = vhi;
    if (kc != nullptr) {
      const int64_t co = ((b * heads + h) * cache_len + cache_offset + s) * head_dim + i;
      kc[co] = klo;
      kc[co + half] = khi;
      vc[co] = vlo;
      vc[co + half] = vhi;
    }
  }
}

int pow2_ceil(int64_t x) {
  int p = 1;
  while (p < x && p < (1 << 30)) p <<= 1;
  return p;
}

int log2_of(int p) {  // p a power of two
  int l = 0;
  while ((1 << l) < p) ++l;
  return l;
}

// Tile counts the tiled kernels take: their 32-bit tile loop needs
// ntiles + gridDim.x < 2^31.
constexpr int64_t kMaxTiles = (int64_t)1 << 30;

}  // namespace

cudaError_t launch_rope(void* q, void* k, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                        int64_t offset, float theta, const float* table, bool token_major, cudaStream_t s) {
  cudaError_t err = cudaSuccess;
  const int64_t sms = device_sm_count();
  const int g = (int)(head_dim / 16);
  int pt = pow2_ceil(seq);
  if (pt > kThreads / (g > 0 ? g : 1)) pt = kThreads / (g > 0 ? g : 1);
  if (pt > HRM_ROPE_MAX_PT) pt = HRM_ROPE_MAX_PT;
  const int64_t tiles_per_batch = (seq + pt - 1) / pt;
  const bool fast = head_dim % 16 == 0 && head_dim <= 512 && (g & (g - 1)) == 0 && aligned16(q) &&
                    aligned16(k) && (table == nullptr || aligned16(table)) &&
                    batch <= kMaxTiles / tiles_per_batch;
  if (fast) {
    RopeArgs a;
    a.q = static_cast<uint4*>(q);
    a.k = static_cast<uint4*>(k);
    const int64_t rc = 2 * g;
    a.batch_stride = heads * seq * rc;
    a.pos_stride = token_major ? heads * rc : rc;
    a.head_stride = token_major ? rc : seq * rc;
    a.table = reinterpret_cast<const float4*>(table);
    a.seq = seq;
    a.heads = (int)heads;
    a.head_dim = (int)head_dim;
    a.g = g;
    a.pt = pt;
    a.ht = kThreads / (g * a.pt);
    a.lg = log2_of(g);
    a.lht = log2_of(a.ht);
    a.tiles_per_batch = (int)tiles_per_batch;
    a.ntiles = (int)(batch * tiles_per_batch);
    a.offset = (int)offset;
    a.theta = theta;
    int64_t blocks = a.ntiles;
    if (HRM_ROPE_CAP > 0 && blocks > sms * HRM_ROPE_CAP) blocks = sms * HRM_ROPE_CAP;
    if (blocks > INT32_MAX) blocks = INT32_MAX;
    if (table != nullptr)
      err = launch_kernel(rope_tile_kernel<true>, blocks, kThreads, 0, s, a);
    else
      err = launch_kernel(rope_tile_kernel<false>, blocks, kThreads, 0, s, a);
  } else {
    const int64_t rows = batch * heads * seq;
    int64_t blocks = (rows * (head_dim / 2) + 255) / 256;
    if (blocks > sms * 8) blocks = sms * 8;
    err = launch_kernel(rope_scalar_kernel, blocks, 256, 0, s, static_cast<uint16_t*>(q), static_cast<uint16_t*>(k),
        rows, seq, token_major ? heads : 1, (int)head_dim, (int)offset, theta, table);
  }
  return err;
}

cudaError_t launch_rope_table(float* table, int64_t positions, int64_t head_dim, float theta, cudaStream_t s) {
  cudaError_t err = cudaSuccess;
  int64_t blocks = (positions * (head_dim / 2) + 255) / 256;
  const int64_t cap = (int64_t)device_sm_count() * 8;
  if (blocks > cap) blocks = cap;
  err = launch_kernel(rope_table_kernel, blocks, 256, 0, s, table, positions, (int)head_dim, theta);
  return err;
}

cudaError_t launch_split_rope(const void* gqkv, void* gate, void* q, void* k, void* v, void* kc, void* vc,
                              int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, int64_t offset,
                              float theta, const float* table, int64_t cache_len, int64_t cache_offset,
                              cudaStream_t s) {
  cudaError_t err = cudaSuccess;
  const int64_t sms = device_sm_count();
  const int g = (int)(head_dim / 16);
  int pt = pow2_ceil(seq);
  if (pt > kThreads / (g > 0 ? g : 1)) pt = kThreads / (g > 0 ? g : 1);
  if (pt > HRM_ROPE_MAX_PT) pt = HRM_ROPE_MAX_PT;
  const int64_t tiles_per_batch = (seq + pt - 1) / pt;
  const bool fast = head_dim % 16 == 0 && head_dim <= 512 && (g & (g - 1)) == 0 && aligned16(gqkv) &&
                    aligned16(gate) && aligned16(q) && aligned16(k) && aligned16(v) &&
                    (kc == nullptr || (aligned16(kc) && aligned16(vc))) && (table == nullptr || aligned16(table)) &&
                    batch <= kMaxTiles / tiles_per_batch;
  if (fast) {
    SplitArgs a;
    a.gqkv = static_cast<const uint4*>(gqkv);
    a.gate = static_cast<uint4*>(gate);
    a.q = static_cast<uint4*>(q);
    a.k = static_cast<uint4*>(k);
    a.v = static_cast<uint4*>(v);
    a.kc = static_cast<uint4*>(kc);
    a.vc = static_cast<uint4*>(vc);
    a.table = reinterpret_cast<const float4*>(table);
    a.seq = seq;
    a.heads = (int)heads;
    a.head_dim = (int)head_dim;
    a.g = g;
    a.pt = pt;
    a.ht = kThreads / (g * a.pt);
    a.lg = log2_of(g);
    a.lht = log2_of(a.ht);
    a.tiles_per_batch = (int)tiles_per_batch;
    a.ntiles = (int)(batch * tiles_per_batch);
    a.cache_len = cache_len;
    a.cache_offset = cache_offset;
    a.offset = (int)offset;
    a.theta = theta;
    int64_t blocks = a.ntiles;
    if (HRM_ROPE_CAP > 0 && blocks > sms * HRM_ROPE_CAP) blocks = sms * HRM_ROPE_CAP;
    if (blocks > INT32_MAX) blocks = INT32_MAX;
    if (table != nullptr) {
      if (kc != nullptr)
        err = launch_kernel(split_rope_tile_kernel<true, true>, blocks, kThreads, 0, s, a);
      else
        err = launch_kernel(split_rope_tile_kernel<true, false>, blocks, kThreads, 0, s, a);
    } else {
      if (kc != nullptr)
        err = launch_kernel(split_rope_tile_kernel<false, true>, blocks, kThreads, 0, s, a);
      else
        err = launch_kernel(split_rope_tile_kernel<false, false>, blocks, kThreads, 0, s, a);
    }
  } else {
    int64_t blocks = (batch * heads * seq * (head_dim / 2) + 255) / 256;
    if (blocks > sms * 8) blocks = sms * 8;
    err = launch_kernel(split_rope_scalar_kernel, blocks, 256, 0, s,
        static_cast<const uint16_t*>(gqkv), static_cast<uint16_t*>(gate), static_cast<uint16_t*>(q),
        static_cast<uint16_t*>(k), static_cast<uint16_t*>(v), static_cast<uint16_t*>(kc), static_cast<uint16_t*>(vc),
        batch, seq, (int)heads, (int)head_dim, (int)offset, theta, table, cache_len, cache_offset);
  }
  return err;
}

}  // namespace hrm
