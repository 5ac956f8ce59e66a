// Test-only harness around the reference's own kernels, compiled from the
// reference sources where they lie (oracle/Makefile passes -I to
// src/kernels of the reference checkout) into oracle/_ref/libref_kernels.so.
// Each ref_* function launches one reference kernel with the launch
// configuration its wrapper in src/lib.rs computes, so the GPU tests can pin
// the CPU oracle -- and this project's kernels -- against the reference
// itself, and time it on the same GPU.  Returns the cudaError_t of the launch.
#include <cuda_runtime.h>
#include <stdint.h>

#include "additive_inject.cu"
#include "apply_attn_gate.cu"
#include "broadcast_vec.cu"
#include "embedding_lookup.cu"
#include "gated_attn_output.cu"
#include "kv_cache_update.cu"
#include "rms_norm.cu"
#include "rope_embed.cu"
#include "split_gqkv.cu"
#include "swiglu_ffn.cu"

namespace {
unsigned blocks_for(int64_t work, int64_t threads) { return (unsigned)((work + threads - 1) / threads); }
}  // namespace

extern "C" {

// src/lib.rs:384-396
int ref_additive_inject(const void* a, const void* b, void* out, int64_t n, cudaStream_t s) {
  const unsigned blocks = blocks_for((n + 7) / 8, 256);
  additive_inject_kernel_vec8<<<blocks, 256, 0, s>>>((const __nv_bfloat16*)a, (const __nv_bfloat16*)b,
                                                     (__nv_bfloat16*)out, (int)n);
  return (int)cudaGetLastError();
}

// src/lib.rs:408-419
int ref_rms_norm(const void* x, void* y, int64_t rows, int64_t hidden, float eps, cudaStream_t s) {
  rms_norm_kernel<<<(unsigned)rows, 256, 8 * sizeof(float), s>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)y,
                                                                 (int)hidden, eps);
  return (int)cudaGetLastError();
}

// src/lib.rs:433-455
int ref_rope_embed(void* q, void* k, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, int64_t offset,
                   float theta, cudaStream_t s) {
  const unsigned blocks = blocks_for(batch * heads * seq * (head_dim / 2), 256);
  rope_embed_kernel<<<blocks, 256, 0, s>>>((__nv_bfloat16*)q, (__nv_bfloat16*)k, (int)batch, (int)heads, (int)seq,
                                           (int)head_dim, (int)offset, theta);
  return (int)cudaGetLastError();
}

// src/lib.rs:489-501
int ref_swiglu_ffn(const void* g, const void* u, void* out, int64_t n, cudaStream_t s) {
  const unsigned blocks = blocks_for((n + 7) / 8, 256);
  swiglu_ffn_kernel<<<blocks, 256, 0, s>>>((const __nv_bfloat16*)g, (const __nv_bfloat16*)u, (__nv_bfloat16*)out,
                                           (int)n);
  return (int)cudaGetLastError();
}

// src/lib.rs:540-562
int ref_embedding_lookup(const uint32_t* ids, const void* table, void* out, int64_t batch, int64_t seq,
                         int64_t hidden, int64_t vocab, float scale, cudaStream_t s) {
  const unsigned blocks = blocks_for(batch * seq * (hidden / 8), 256);
  embedding_lookup_kernel<<<blocks, 256, 0, s>>>(ids, (const __nv_bfloat16*)table, (__nv_bfloat16*)out, (int)batch,
                                                 (int)seq, (int)hidden, (int)vocab, scale);
  return (int)cudaGetLastError();
}

// src/lib.rs:579-602
int ref_split_gqkv(const void* gqkv, void* gate, void* q, void* k, void* v, int64_t batch, int64_t seq,
                   int64_t heads, int64_t head_dim, cudaStream_t s) {
  const unsigned blocks = blocks_for(batch * seq * heads * (head_dim / 8), 256);
  split_gqkv_kernel<<<blocks, 256, 0, s>>>((const __nv_bfloat16*)gqkv, (__nv_bfloat16*)gate, (__nv_bfloat16*)q,
                                           (__nv_bfloat16*)k, (__nv_bfloat16*)v, (int)batch, (int)seq, (int)heads,
                                           (int)head_dim);
  return (int)cudaGetLastError();
}

// src/lib.rs:719-744
int ref_kv_cache_update(const void* k, const void* v, void* kc, void* vc, int64_t batch, int64_t heads, int64_t seq,
                        int64_t head_dim, int64_t max_len, int64_t cached_len, int is_decode, cudaStream_t s) {
  int64_t blocks = (batch * heads * seq * head_dim + 255) / 256;
  if (blocks > 65535) blocks = 65535;
  if (blocks < 1) blocks = 1;
  kv_cache_update_kernel<<<(unsigned)blocks, 256, 0, s>>>((const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
                                                          (__nv_bfloat16*)kc, (__nv_bfloat16*)vc, (int)batch,
                                                          (int)heads, (int)seq, (int)head_dim, (int)max_len,
                                                          (int)cached_len, is_decode);
  return (int)cudaGetLastError();
}

// src/lib.rs:613-627 (in place)
int ref_apply_attn_gate(const void* gate, void* attn, int64_t n, cudaStream_t s) {
  apply_attn_gate_kernel<<<blocks_for((n + 7) / 8, 256), 256, 0, s>>>((const __nv_bfloat16*)gate,
                                                                      (__nv_bfloat16*)attn, (int)n);
  return (int)cudaGetLastError();
}

// src/lib.rs:512-524
int ref_gated_attn_output(const void* gate, const void* attn, void* out, int64_t n, cudaStream_t s) {
  gated_attn_output_kernel<<<blocks_for((n + 7) / 8, 256), 256, 0, s>>>(
      (const __nv_bfloat16*)gate, (const __nv_bfloat16*)attn, (__nv_bfloat16*)out, (int)n);
  return (int)cudaGetLastError();
}

// src/lib.rs:755-764
int ref_broadcast_vec(void* dst, const void* src, int64_t n_copies, int64_t vec_len, cudaStream_t s) {
  int64_t blocks = (n_copies * vec_len + 255) / 256;
  if (blocks > 65535) blocks = 65535;
  if (blocks < 1) blocks = 1;
  broadcast_vec_kernel<<<(unsigned)blocks, 256, 0, s>>>((__nv_bfloat16*)dst, (const __nv_bfloat16*)src,
                                                        (int)n_copies, (int)vec_len);
  return (int)cudaGetLastError();
}

}  // extern "C"
