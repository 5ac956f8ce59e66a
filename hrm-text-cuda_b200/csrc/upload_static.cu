// hrm_upload_to_bf16_static: the checkpoint upload + bf16 conversion of
// hrm_upload_to_bf16 for callers that must not allocate device memory, with
// its staging buffer in a fixed array of this library instead of one the
// caller passes.
//
// Who needs it: a caller whose GPU memory is reserved in full by another
// allocator (a serving engine's memory pool, a framework's caching allocator
// that owns the budget) and that therefore has no staging buffer to give and
// may not call cudaMalloc for one; and a caller that reloads weights while
// other streams keep running, where cudaMalloc / cudaFree would synchronise
// the device.
//
// The array lives in device memory for as long as the library is loaded: every
// GPU on which the library's code is loaded holds HRM_UPLOAD_STATIC_BYTES
// (16 MiB) for it until the process exits.  Host code must not pass the
// array's name to a kernel or a copy: on the host that name is a stand-in
// object, not the device address.  The address is queried per device with
// cudaGetSymbolAddress, with that device current, by the first call on the
// device, and cached; make that first call before any stream capture.
#include <atomic>
#include <climits>

#include "../../include/hrm_ops.h"
#include "launch.h"

namespace {

// 16 MiB of raw checkpoint bytes per call: 4 Mi f32 or 8 Mi f16 values.
constexpr int64_t kStaticBytes = HRM_UPLOAD_STATIC_BYTES;

static __device__ __align__(256) unsigned char g_upload_scratch[HRM_UPLOAD_STATIC_BYTES];

// Device address of g_upload_scratch on the current device (queried once per
// device).  Returns the CUDA error of the query, or cudaSuccess.
cudaError_t scratch_address(void** out) {
  static std::atomic<void*> cache[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64) {
    void* p = cache[dev].load(std::memory_order_acquire);
    if (p != nullptr) {
      *out = p;
      return cudaSuccess;
    }
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_upload_scratch);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64) cache[dev].store(p, std::memory_order_release);
  *out = p;
  return cudaSuccess;
}

bool overlaps(const void* a, int64_t abytes, const void* b, int64_t bbytes) {
  if (a == nullptr || b == nullptr || abytes <= 0 || bbytes <= 0) return false;
  const uintptr_t pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b);
  return pa < pb + (uintptr_t)bbytes && pb < pa + (uintptr_t)abytes;
}

}  // namespace

extern "C" int hrm_upload_to_bf16_static(const void* src, int src_dtype, void* dst, int64_t n,
                                         hrm_stream_t stream) {
  if (src_dtype != HRM_DTYPE_BF16 && src_dtype != HRM_DTYPE_F32 && src_dtype != HRM_DTYPE_F16) return HRM_ERR_DTYPE;
  if (n < 0) return HRM_ERR_INVALID_SHAPE;
  if (n == 0) return HRM_OK;
  if (!src || !dst) return HRM_ERR_NULL_POINTER;
  const int64_t size = src_dtype == HRM_DTYPE_F32 ? 4 : 2;
  if (n > INT64_MAX / 8) return HRM_ERR_SIZE_OVERFLOW;
  const int64_t in_bytes = n * size, out_bytes = n * 2;
  if (overlaps(src, in_bytes, dst, out_bytes)) return HRM_ERR_ALIASING;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // bf16 needs no conversion, hence no scratch: one copy straight into dst.
  if (src_dtype == HRM_DTYPE_BF16) {
    const cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)in_bytes, cudaMemcpyDefault, s);
    return e == cudaSuccess ? HRM_OK : HRM_ERR_CUDA + (int)e;
  }
  if (in_bytes > kStaticBytes) return HRM_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  cudaError_t e = scratch_address(&scratch);
  if (e != cudaSuccess) return HRM_ERR_CUDA + (int)e;
  if (overlaps(scratch, in_bytes, dst, out_bytes) || overlaps(scratch, in_bytes, src, in_bytes))
    return HRM_ERR_ALIASING;
  // Every scratch byte the conversion reads is written by this copy first, so
  // nothing has to start at zero.
  e = cudaMemcpyAsync(scratch, src, (size_t)in_bytes, cudaMemcpyDefault, s);
  if (e == cudaSuccess) e = hrm::launch_convert_to_bf16(scratch, src_dtype, dst, n, s);
  return e == cudaSuccess ? HRM_OK : HRM_ERR_CUDA + (int)e;
}
