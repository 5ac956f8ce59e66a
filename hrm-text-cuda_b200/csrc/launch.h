// Host-side launchers of the sm_100a layer-op kernels (called by abi.cu after
// argument validation; they assume valid, non-empty arguments).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace hrm {

// SM count of the current device, queried once per device and cached.
int device_sm_count();

// True when p is 16-byte aligned (a uint4 access is legal).
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Warps per CTA of a one-warp-per-row launch over `rows` rows: max_warps, or
// fewer when there are fewer than max_warps rows per SM, so that a small
// (decode-size) launch spreads over as many SMs as it has rows instead of
// rows / max_warps of them.
inline int warps_per_cta(int64_t rows, int max_warps) {
  const int64_t per_sm = rows / device_sm_count();
  if (per_sm >= max_warps) return max_warps;
  return per_sm < 1 ? 1 : (int)per_sm;
}

// Programmatic dependent launches (1) or plain stream-ordered ones (0).
#ifndef HRM_PDL
#define HRM_PDL 1
#endif

// Launches kernel k as grid x block threads with smem dynamic shared bytes on
// stream s.  The launch is programmatic (cudaLaunchAttributeProgrammatic-
// StreamSerialization): it may start before the previous kernel in s has
// finished, which is safe because every kernel of this library waits for that
// kernel at its entry (grid_dependency_begin).  Returns the launch's own
// status, so an error left pending by an earlier, unrelated call is neither
// reported as this launch's nor cleared.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*k)(KArgs...), int64_t grid, int block, size_t smem, cudaStream_t s,
                                 Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = HRM_PDL ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, static_cast<Args&&>(args)...);
}

cudaError_t launch_additive_inject(const void* a, const void* b, void* out, int64_t n, cudaStream_t s);
cudaError_t launch_attn_gate(const void* gate, const void* attn, void* out, int64_t n, cudaStream_t s);
cudaError_t launch_broadcast(void* dst, const void* src, int64_t n_copies, int64_t vec_len, cudaStream_t s);
cudaError_t launch_swiglu(const void* gate, const void* up, void* out, int64_t n, cudaStream_t s);

cudaError_t launch_rms_norm_bf16(const void* x, void* y, const void* w, int64_t rows, int64_t hidden,
                                 float eps, cudaStream_t s);
cudaError_t launch_rms_norm_f32(const float* x, float* y, const float* w, int64_t rows, int64_t hidden,
                                float eps, cudaStream_t s);
cudaError_t launch_add_rms_norm(const void* x, const void* b, void* r, void* y, const void* w, int64_t rows,
                                int64_t hidden, float eps, cudaStream_t s);
cudaError_t launch_embed_rms_norm(const uint32_t* ids, const void* table, void* h, void* y, const void* w,
                                  int64_t rows, int64_t hidden, int64_t vocab, float scale, float eps,
                                  cudaStream_t s);
cudaError_t launch_embedding(const uint32_t* ids, const void* table, void* out, int64_t tokens, int64_t hidden,
                             int64_t vocab, float scale, cudaStream_t s);

cudaError_t launch_rope(void* q, void* k, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                        int64_t offset, float theta, const float* table, bool token_major, cudaStream_t s);
cudaError_t launch_split_rope(const void* gqkv, void* gate, void* q, void* k, void* v, void* kc, void* vc,
                              int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, int64_t offset,
                              float theta, const float* table, int64_t cache_len, int64_t cache_offset,
                              cudaStream_t s);
cudaError_t launch_rope_table(float* table, int64_t max_pos, int64_t head_dim, float theta, cudaStream_t s);

cudaError_t launch_convert_to_bf16(const void* src, int dtype, void* dst, int64_t n, cudaStream_t s);

// Bounded waits that ran out in the row kernels (device counter); reset sets it to 0.
cudaError_t rownorm_wait_timeouts(unsigned int* count, bool reset);

}  // namespace hrm
