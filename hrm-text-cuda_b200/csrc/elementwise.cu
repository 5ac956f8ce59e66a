// Elementwise bf16 streams: the SwiGLU gate, the residual add, the sigmoid
// attention gate and the row broadcast.
//
// Both are pure HBM streams (2 reads + 1 write per element, ~0.5 flop/B), so
// the kernel is shaped for bytes in flight, not arithmetic:
//   * one 16-byte vector (8 bf16) per access, every warp-wide access a fully
//     used, contiguous 512-byte span;
//   * U independent vectors per operand per thread issued before any use
//     (U = 2 -> 4 x 16 B loads in flight per thread);
//   * a grid that covers the tensor once (one U-vector group per thread) with
//     8 resident 256-thread CTAs per SM (<= 32 registers, all 64 warp slots):
//     the hardware refills SMs as CTAs retire.  Measured on B200: 6.74 TB/s
//     for SwiGLU, against 6.50 with 4 resident CTAs and 6.06 for a persistent
//     one-wave grid with 4 vectors in flight per thread.  (Pairing the fp32
//     multiplies into f32x2 instructions measured slower at every occupancy.)
//   * loads with the default L2 priority (1.3-1.6% faster than evict-first
//     ones on B200) and evict-first stores, so the output stream does not
//     flush reused L2 lines;
//   * a launch too small to give every SM a CTA that way (decode sizes) takes
//     one vector per thread instead, doubling its CTAs.
// The arithmetic per element is the reference's, operation for operation:
//   swiglu: g * (1.0f / (1.0f + __expf(-g))) * u    (src/kernels/swiglu_ffn.cu:31-35)
//   add   : a + b                                   (src/kernels/additive_inject.cu:29-31)
//   gate  : (1.0f / (1.0f + __expf(-g))) * a        (src/kernels/apply_attn_gate.cu:28-29)
// each rounded once to bf16 (RNE), so results match the reference bit for bit.
#include "common.cuh"
#include "launch.h"

namespace hrm {
namespace {

// Launch shape (compile-time; the defaults are the tuned values):
//   HRM_EW_UNROLL     vectors per operand per thread per iteration
//   HRM_EW_WAVES      grid cap in waves of resident CTAs (0: no cap, one
//                     iteration per thread)
//   HRM_EW_MINBLOCKS  __launch_bounds__ minimum resident CTAs per SM
#ifndef HRM_EW_UNROLL
#define HRM_EW_UNROLL 2
#endif
#ifndef HRM_EW_WAVES
#define HRM_EW_WAVES 0
#endif
#ifndef HRM_EW_MINBLOCKS
#define HRM_EW_MINBLOCKS 8
#endif
constexpr int kThreads = 256;
constexpr int kUnroll = HRM_EW_UNROLL;

struct SwigluOp {
  __device__ __forceinline__ float f(float g, float u) const {
    float sig = 1.0f / (1.0f + __expf(-g));
    return g * sig * u;
  }
};
struct AddOp {
  __device__ __forceinline__ float f(float a, float b) const { return a + b; }
};
struct GateOp {  // first operand: gate, second: attention output
  __device__ __forceinline__ float f(float g, float a) const { return (1.0f / (1.0f + __expf(-g))) * a; }
};

// dst[r, :] = src[:]: one 16-byte chunk per thread per step, the source row
// read through L1 (every CTA reads the same few KB), stores streamed.
__global__ void __launch_bounds__(kThreads) broadcast_vec_kernel(uint4* dst, const uint4* src, int64_t n_copies,
                                                                  int64_t chunks) {
  grid_dependency_begin();
  const int64_t total = n_copies * chunks;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < total; i += stride)
    st_stream(dst + i, ld_keep(src + i % chunks));
}

__global__ void __launch_bounds__(kThreads) broadcast_scalar_kernel(uint16_t* dst, const uint16_t* src,
                                                                    int64_t n_copies, int64_t vec_len) {
  grid_dependency_begin();
  const int64_t total = n_copies * vec_len;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < total; i += stride) dst[i] = src[i % vec_len];
}

template <class Op>
__device__ __forceinline__ uint4 apply8(const Op& op, const uint4& a, const uint4& b) {
  uint4 o;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uint32_t wa = vget(a, w), wb = vget(b, w);
    vset(o, w, pack_bf16x2(op.f(bf16_lo(wa), bf16_lo(wb)), op.f(bf16_hi(wa), bf16_hi(wb))));
  }
  return o;
}

// a, b, out: 16-byte aligned; nvec = n / 8 full vectors; the n % 8 trailing
// elements (starting at element nvec * 8) are done by global thread 0.  U
// vectors per operand per thread: kUnroll, or 1 for a launch too small to
// give every SM a CTA otherwise (decode sizes).
template <class Op, int U>
__global__ void __launch_bounds__(kThreads, HRM_EW_MINBLOCKS) ew_vec_kernel(const uint4* a, const uint4* b, uint4* out,
                                                          int64_t nvec, int tail) {
  grid_dependency_begin();
  const Op op;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  for (; i + (U - 1) * stride < nvec; i += U * stride) {
    uint4 va[U], vb[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      va[j] = ld_l2(a + i + j * stride);
      vb[j] = ld_l2(b + i + j * stride);
    }
#pragma unroll
    for (int j = 0; j < U; ++j) st_stream(out + i + j * stride, apply8(op, va[j], vb[j]));
  }
  for (; i < nvec; i += stride) st_stream(out + i, apply8(op, ld_l2(a + i), ld_l2(b + i)));

  if (tail > 0 && blockIdx.x == 0 && threadIdx.x == 0) {
    const uint16_t* as = reinterpret_cast<const uint16_t*>(a + nvec);
    const uint16_t* bs = reinterpret_cast<const uint16_t*>(b + nvec);
    uint16_t* os = reinterpret_cast<uint16_t*>(out + nvec);
    for (int t = 0; t < tail; ++t) os[t] = f32_to_bf16(op.f(bf16_to_f32(as[t]), bf16_to_f32(bs[t])));
  }
}

// Any alignment: one element per thread per step.
template <class Op>
__global__ void __launch_bounds__(kThreads) ew_scalar_kernel(const uint16_t* a, const uint16_t* b, uint16_t* out,
                                                             int64_t n) {
  grid_dependency_begin();
  const Op op;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride)
    out[i] = f32_to_bf16(op.f(bf16_to_f32(a[i]), bf16_to_f32(b[i])));
}

template <class Op>
cudaError_t launch_ew(const void* a, const void* b, void* out, int64_t n, cudaStream_t s) {
  cudaError_t err = cudaSuccess;
  const int64_t max_blocks = (int64_t)device_sm_count() * (2048 / kThreads);
  if (aligned16(a) && aligned16(b) && aligned16(out)) {
    const int64_t nvec = n / 8;
    int64_t blocks = (nvec + (int64_t)kThreads * kUnroll - 1) / ((int64_t)kThreads * kUnroll);
    if (blocks < device_sm_count()) {  // small launch: one vector per thread, more CTAs
      blocks = (nvec + kThreads - 1) / kThreads;
      if (blocks < 1) blocks = 1;
      return launch_kernel(ew_vec_kernel<Op, 1>, blocks, kThreads, 0, s, static_cast<const uint4*>(a),
          static_cast<const uint4*>(b), static_cast<uint4*>(out), nvec, (int)(n % 8));
    }
    if (HRM_EW_WAVES > 0 && blocks > max_blocks * HRM_EW_WAVES) blocks = max_blocks * HRM_EW_WAVES;
    if (blocks > INT32_MAX) blocks = INT32_MAX;
    err = launch_kernel(ew_vec_kernel<Op, kUnroll>, blocks, kThreads, 0, s, static_cast<const uint4*>(a),
        static_cast<const uint4*>(b), static_cast<uint4*>(out), nvec, (int)(n % 8));
  } else {
    int64_t blocks = (n + kThreads - 1) / kThreads;
    if (blocks > max_blocks) blocks = max_blocks;
    err = launch_kernel(ew_scalar_kernel<Op>, blocks, kThreads, 0, s, static_cast<const uint16_t*>(a),
        static_cast<const uint16_t*>(b), static_cast<uint16_t*>(out), n);
  }
  return err;
}

}  // namespace

cudaError_t launch_swiglu(const void* gate, const void* up, void* out, int64_t n, cudaStream_t s) {
  return launch_ew<SwigluOp>(gate, up, out, n, s);
}

cudaError_t launch_additive_inject(const void* a, const void* b, void* out, int64_t n, cudaStream_t s) {
  return launch_ew<AddOp>(a, b, out, n, s);
}

cudaError_t launch_attn_gate(const void* gate, const void* attn, void* out, int64_t n, cudaStream_t s) {
  return launch_ew<GateOp>(gate, attn, out, n, s);
}

cudaError_t launch_broadcast(void* dst, const void* src, int64_t n_copies, int64_t vec_len, cudaStream_t s) {
  cudaError_t err = cudaSuccess;
  const int64_t cap = (int64_t)device_sm_count() * (2048 / kThreads) * 4;
  if (vec_len % 8 == 0 && aligned16(dst) && aligned16(src)) {
    const int64_t chunks = vec_len / 8;
    int64_t blocks = (n_copies * chunks + kThreads - 1) / kThreads;
    if (blocks > cap) blocks = cap;
    err = launch_kernel(broadcast_vec_kernel, blocks, kThreads, 0, s, static_cast<uint4*>(dst),
        static_cast<const uint4*>(src), n_copies, chunks);
  } else {
    int64_t blocks = (n_copies * vec_len + kThreads - 1) / kThreads;
    if (blocks > cap) blocks = cap;
    err = launch_kernel(broadcast_scalar_kernel, blocks, kThreads, 0, s, static_cast<uint16_t*>(dst),
        static_cast<const uint16_t*>(src), n_copies,
        vec_len);
  }
  return err;
}

}  // namespace hrm
