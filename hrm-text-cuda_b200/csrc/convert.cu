// Checkpoint element conversion to bf16 on the GPU (the reference's weight
// loader converts on the host, one element at a time: src/lib.rs:1981-2008).
//
// Semantics are those of the `half` crate (2.7.1, pinned in the reference's
// Cargo.lock) that the loader calls:
//   f32 -> bf16: round to nearest, ties to even; a NaN keeps its sign and its
//                top 16 bits and gets the quiet bit (0x0040) set -- unlike
//                the CUDA intrinsic, which returns one canonical NaN;
//   f16 -> f32:  exact widening (subnormals normalised; a NaN keeps its
//                payload, shifted, with the quiet bit set), then as above.
// Both are done with integer operations so every bit pattern, NaNs included,
// converts exactly as on the host.
//
// Fast path (16-byte aligned src and dst): 8 values per thread per step --
// two 16-byte loads of f32 or one of f16, one 16-byte store.  Any other
// alignment reads the source byte by byte (checkpoint tensors sit at
// arbitrary byte offsets in a safetensors file).
#include "../../include/hrm_ops.h"
#include "common.cuh"
#include "launch.h"

namespace hrm {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint16_t loader_f32_to_bf16(uint32_t x) {
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x0040u);
  return (uint16_t)((x + 0x7fffu + ((x >> 16) & 1u)) >> 16);
}

__device__ __forceinline__ uint32_t f16_to_f32_bits(uint32_t h) {
  const uint32_t sign = (h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  if (exp == 0x1fu) return sign | 0x7f800000u | (man ? (0x00400000u | (man << 13)) : 0u);
  if (exp == 0) {
    if (man == 0) return sign;
    // subnormal: value = man * 2^-24; normalise so the leading one is bit 10
    const int shift = __clz(man) - 21;  // leading zeros within the 11-bit field
    man = (man << shift) & 0x3ffu;
    return sign | ((uint32_t)(127 - 15 - shift + 1) << 23) | (man << 13);
  }
  return sign | ((exp + 112u) << 23) | (man << 13);
}

template <int DTYPE>
__device__ __forceinline__ uint16_t convert_one(uint32_t bits) {
  return DTYPE == HRM_DTYPE_F32 ? loader_f32_to_bf16(bits) : loader_f32_to_bf16(f16_to_f32_bits(bits));
}

// Source loads with the default L2 priority (ld_l2): 2^28 f32 values 6.25 ->
// 6.63 TB/s on B200 against evict-first loads; the store policy made no
// difference, so the outputs stay evict-first.
template <int DTYPE>
__global__ void __launch_bounds__(kThreads) convert_vec_kernel(const uint4* src, uint4* dst, int64_t nvec) {
  grid_dependency_begin();
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < nvec; i += stride) {
    uint32_t in[8];
    if (DTYPE == HRM_DTYPE_F32) {
      const uint4 a = ld_l2(src + 2 * i), b = ld_l2(src + 2 * i + 1);
      in[0] = a.x; in[1] = a.y; in[2] = a.z; in[3] = a.w; in[4] = b.x; in[5] = b.y; in[6] = b.z; in[7] = b.w;
    } else {
      const uint4 a = ld_l2(src + i);
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        in[2 * w] = vget(a, w) & 0xffffu;
        in[2 * w + 1] = vget(a, w) >> 16;
      }
    }
    uint4 o;
#pragma unroll
    for (int w = 0; w < 4; ++w)
      vset(o, w, (uint32_t)convert_one<DTYPE>(in[2 * w]) | ((uint32_t)convert_one<DTYPE>(in[2 * w + 1]) << 16));
    st_stream(dst + i, o);
  }
}

// Any alignment: element i's bytes assembled little-endian from src + i * size.
template <int DTYPE>
__global__ void __launch_bounds__(kThreads) convert_scalar_kernel(const uint8_t* src, uint16_t* dst, int64_t n) {
  grid_dependency_begin();
  constexpr int kSize = DTYPE == HRM_DTYPE_F32 ? 4 : 2;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride) {
    uint32_t bits = 0;
#pragma unroll
    for (int b = 0; b < kSize; ++b) bits |= (uint32_t)src[i * kSize + b] << (8 * b);
    dst[i] = convert_one<DTYPE>(bits);
  }
}

template <int DTYPE>
cudaError_t launch_dtype(const void* src, void* dst, int64_t n, cudaStream_t s) {
  cudaError_t err = cudaSuccess;
  const int64_t cap = (int64_t)device_sm_count() * (2048 / kThreads) * 4;
  int64_t done = 0;
  if (aligned16(src) && aligned16(dst)) {
    const int64_t nvec = n / 8;
    if (nvec > 0) {
      int64_t blocks = (nvec + kThreads - 1) / kThreads;
      if (blocks > cap) blocks = cap;
      err = launch_kernel(convert_vec_kernel<DTYPE>, blocks, kThreads, 0, s, static_cast<const uint4*>(src),
          static_cast<uint4*>(dst), nvec);
      done = nvec * 8;
    }
  }
  const int64_t rest = n - done;
  if (rest > 0 && err == cudaSuccess) {
    constexpr int kSize = DTYPE == HRM_DTYPE_F32 ? 4 : 2;
    int64_t blocks = (rest + kThreads - 1) / kThreads;
    if (blocks > cap) blocks = cap;
    err = launch_kernel(convert_scalar_kernel<DTYPE>, blocks, kThreads, 0, s,
        static_cast<const uint8_t*>(src) + done * kSize, static_cast<uint16_t*>(dst) + done, rest);
  }
  return err;
}

}  // namespace

cudaError_t launch_convert_to_bf16(const void* src, int dtype, void* dst, int64_t n, cudaStream_t s) {
  if (dtype == HRM_DTYPE_F32) return launch_dtype<HRM_DTYPE_F32>(src, dst, n, s);
  if (dtype == HRM_DTYPE_F16) return launch_dtype<HRM_DTYPE_F16>(src, dst, n, s);
  return cudaMemcpyAsync(dst, src, (size_t)n * 2, cudaMemcpyDeviceToDevice, s);
}

}  // namespace hrm
