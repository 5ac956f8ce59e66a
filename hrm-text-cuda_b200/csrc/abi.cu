// extern "C" entry points declared in include/hrm_ops.h: argument checks, then
// the launcher.  Every check runs before anything is queued, so an error
// status never leaves partial work on the stream.
#include <atomic>
#include <climits>

#include "../../include/hrm_ops.h"
#include "launch.h"

namespace hrm {

int device_sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  int v = (dev >= 0 && dev < 64) ? cache[dev].load(std::memory_order_relaxed) : 0;
  if (v > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) {
    cudaGetLastError();  // clear, and size grids for a B200
    v = 148;
  }
  if (dev >= 0 && dev < 64) cache[dev].store(v, std::memory_order_relaxed);
  return v;
}

}  // namespace hrm

namespace {

constexpr int kAbiVersion = 10000;  // 1.0.0

int cuda_status(cudaError_t e) { return e == cudaSuccess ? HRM_OK : HRM_ERR_CUDA + (int)e; }

// n * m for non-negative operands, or -1 when it would exceed limit.
int64_t mul_checked(int64_t n, int64_t m, int64_t limit = INT64_MAX / 8) {
  if (n < 0 || m < 0) return -1;
  if (n != 0 && m > limit / n) return -1;
  return n * m;
}

// True when [a, a + abytes) and [b, b + bbytes) share a byte.
bool overlap(const void* a, int64_t abytes, const void* b, int64_t bbytes) {
  if (a == nullptr || b == nullptr || abytes <= 0 || bbytes <= 0) return false;
  const uintptr_t pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b);
  return pa < pb + (uintptr_t)bbytes && pb < pa + (uintptr_t)abytes;
}

// Partial overlap (anything but identical ranges) of two equal-sized buffers.
bool partial_overlap(const void* a, const void* b, int64_t bytes) { return a != b && overlap(a, bytes, b, bytes); }

cudaStream_t as_cuda(hrm_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

}  // namespace

extern "C" {

const char* hrm_status_string(int status) {
  switch (status) {
    case HRM_OK: return "ok";
    case HRM_ERR_NULL_POINTER: return "a required pointer is NULL";
    case HRM_ERR_INVALID_SHAPE: return "invalid shape argument";
    case HRM_ERR_SIZE_OVERFLOW: return "size arithmetic overflows";
    case HRM_ERR_ALIASING: return "buffers that must be distinct overlap";
    case HRM_ERR_TABLE_RANGE: return "position_offset + seq_len exceeds the rope table";
    case HRM_ERR_DTYPE: return "unsupported dtype";
    case HRM_ERR_SCRATCH_LIMIT: return "request exceeds the fixed device scratch of an allocation-free entry point";
    default: break;
  }
  if (status > HRM_ERR_CUDA) return cudaGetErrorString(static_cast<cudaError_t>(status - HRM_ERR_CUDA));
  return "unknown status";
}

int hrm_abi_version(void) { return kAbiVersion; }

int hrm_additive_inject(const void* z_a, const void* z_b, void* z_out, int64_t total_elements,
                        hrm_stream_t stream) {
  if (total_elements < 0) return HRM_ERR_INVALID_SHAPE;
  if (total_elements == 0) return HRM_OK;
  if (!z_a || !z_b || !z_out) return HRM_ERR_NULL_POINTER;
  const int64_t bytes = mul_checked(total_elements, 2);
  if (bytes < 0) return HRM_ERR_SIZE_OVERFLOW;
  if (partial_overlap(z_out, z_a, bytes) || partial_overlap(z_out, z_b, bytes)) return HRM_ERR_ALIASING;
  return cuda_status(hrm::launch_additive_inject(z_a, z_b, z_out, total_elements, as_cuda(stream)));
}

int hrm_swiglu_ffn(const void* gate, const void* up, void* output, int64_t total_elements, hrm_stream_t stream) {
  if (total_elements < 0) return HRM_ERR_INVALID_SHAPE;
  if (total_elements == 0) return HRM_OK;
  if (!gate || !up || !output) return HRM_ERR_NULL_POINTER;
  const int64_t bytes = mul_checked(total_elements, 2);
  if (bytes < 0) return HRM_ERR_SIZE_OVERFLOW;
  if (partial_overlap(output, gate, bytes) || partial_overlap(output, up, bytes)) return HRM_ERR_ALIASING;
  return cuda_status(hrm::launch_swiglu(gate, up, output, total_elements, as_cuda(stream)));
}

int hrm_gated_attn_output(const void* gate, const void* attn_out, void* output, int64_t total_elements,
                          hrm_stream_t stream) {
  if (total_elements < 0) return HRM_ERR_INVALID_SHAPE;
  if (total_elements == 0) return HRM_OK;
  if (!gate || !attn_out || !output) return HRM_ERR_NULL_POINTER;
  const int64_t bytes = mul_checked(total_elements, 2);
  if (bytes < 0) return HRM_ERR_SIZE_OVERFLOW;
  if (partial_overlap(output, attn_out, bytes) || overlap(output, bytes, gate, bytes)) return HRM_ERR_ALIASING;
  return cuda_status(hrm::launch_attn_gate(gate, attn_out, output, total_elements, as_cuda(stream)));
}

int hrm_apply_attn_gate(const void* gate, void* attn_out, int64_t total_elements, hrm_stream_t stream) {
  return hrm_gated_attn_output(gate, attn_out, attn_out, total_elements, stream);
}

int hrm_broadcast_vec(void* dst, const void* src, int64_t n_copies, int64_t vec_len, hrm_stream_t stream) {
  if (n_copies < 0 || vec_len < 0) return HRM_ERR_INVALID_SHAPE;
  if (n_copies == 0 || vec_len == 0) return HRM_OK;
  if (!dst || !src) return HRM_ERR_NULL_POINTER;
  const int64_t bytes = mul_checked(mul_checked(n_copies, vec_len), 2);
  if (bytes < 0) return HRM_ERR_SIZE_OVERFLOW;
  if (overlap(dst, bytes, src, vec_len * 2)) return HRM_ERR_ALIASING;
  return cuda_status(hrm::launch_broadcast(dst, src, n_copies, vec_len, as_cuda(stream)));
}

int hrm_rms_norm(const void* input, void* output, const void* weight, int64_t rows, int64_t hidden_size,
                 float eps, hrm_stream_t stream) {
  if (rows < 0 || hidden_size <= 0 || hidden_size > INT32_MAX) return HRM_ERR_INVALID_SHAPE;
  if (rows == 0) return HRM_OK;
  if (!input || !output) return HRM_ERR_NULL_POINTER;
  const int64_t bytes = mul_checked(mul_checked(rows, hidden_size), 2);
  if (bytes < 0) return HRM_ERR_SIZE_OVERFLOW;
  if (overlap(input, bytes, output, bytes) || overlap(weight, hidden_size * 2, output, bytes))
    return HRM_ERR_ALIASING;
  return cuda_status(hrm::launch_rms_norm_bf16(input, output, weight, rows, hidden_size, eps, as_cuda(stream)));
}

int hrm_rms_norm_f32(const float* input, float* output, const float* weight, int64_t rows, int64_t hidden_size,
                     float eps, hrm_stream_t stream) {
  if (rows < 0 || hidden_size <= 0 || hidden_size > INT32_MAX) return HRM_ERR_INVALID_SHAPE;
  if (rows == 0) return HRM_OK;
  if (!input || !output) return HRM_ERR_NULL_POINTER;
  const int64_t bytes = mul_checked(mul_checked(rows, hidden_size), 4);
  if (bytes < 0) return HRM_ERR_SIZE_OVERFLOW;
  if (overlap(input, bytes, output, bytes) || overlap(weight, hidden_size * 4, output, bytes))
    return HRM_ERR_ALIASING;
  return cuda_status(hrm::launch_rms_norm_f32(input, output, weight, rows, hidden_size, eps, as_cuda(stream)));
}

int hrm_add_rms_norm(const void* x, const void* branch, void* residual_out, void* normed_out, const void* weight,
                     int64_t rows, int64_t hidden_size, float eps, hrm_stream_t stream) {
  if (rows < 0 || hidden_size <= 0 || hidden_size > INT32_MAX) return HRM_ERR_INVALID_SHAPE;
  if (rows == 0) return HRM_OK;
  if (!x || !branch || !residual_out || !normed_out) return HRM_ERR_NULL_POINTER;
  const int64_t bytes = mul_checked(mul_checked(rows, hidden_size), 2);
  if (bytes < 0) return HRM_ERR_SIZE_OVERFLOW;
  if (partial_overlap(residual_out, x, bytes) || partial_overlap(residual_out, branch, bytes) ||
      overlap(normed_out, bytes, x, bytes) || overlap(normed_out, bytes, branch, bytes) ||
      overlap(normed_out, bytes, residual_out, bytes) || overlap(weight, hidden_size * 2, normed_out, bytes) ||
      overlap(weight, hidden_size * 2, residual_out, bytes))
    return HRM_ERR_ALIASING;
  return cuda_status(
      hrm::launch_add_rms_norm(x, branch, residual_out, normed_out, weight, rows, hidden_size, eps, as_cuda(stream)));
}

}  // extern "C"

namespace {

int rope_common(void* q, void* k, int64_t batch_size, int64_t num_heads, int64_t seq_len, int64_t head_dim,
                int64_t position_offset, float theta, const float* rope_table, int64_t table_positions,
                bool token_major, hrm_stream_t stream) {
  if (batch_size < 0 || num_heads < 0 || seq_len < 0 || head_dim <= 0 || head_dim % 2 != 0 ||
      position_offset < 0 || num_heads > INT32_MAX || head_dim > INT32_MAX)
    return HRM_ERR_INVALID_SHAPE;
  // offset + seq <= INT32_MAX, checked without forming a sum that could overflow
  if (seq_len > INT32_MAX || position_offset > INT32_MAX - seq_len) return HRM_ERR_SIZE_OVERFLOW;
  if (batch_size == 0 || num_heads == 0 || seq_len == 0) return HRM_OK;
  if (!q || !k) return HRM_ERR_NULL_POINTER;
  const int64_t bytes = mul_checked(mul_checked(mul_checked(mul_checked(batch_size, num_heads), seq_len), head_dim), 2);
  if (bytes < 0) return HRM_ERR_SIZE_OVERFLOW;
  if (overlap(q, bytes, k, bytes)) return HRM_ERR_ALIASING;
  if (rope_table != nullptr) {
    if (table_positions < position_offset + seq_len) return HRM_ERR_TABLE_RANGE;
    const int64_t tbytes = mul_checked(mul_checked(table_positions, head_dim), 4);
    if (tbytes < 0) return HRM_ERR_SIZE_OVERFLOW;
    if (overlap(rope_table, tbytes, q, bytes) || overlap(rope_table, tbytes, k, bytes)) return HRM_ERR_ALIASING;
  }
  return cuda_status(hrm::launch_rope(q, k, batch_size, num_heads, seq_len, head_dim, position_offset, theta,
                                      rope_table, token_major, as_cuda(stream)));
}

}  // namespace

extern "C" {

int hrm_rope_embed(void* q, void* k, int64_t batch_size, int64_t num_heads, int64_t seq_len, int64_t head_dim,
                   int64_t position_offset, float theta, const float* rope_table, int64_t table_positions,
                   hrm_stream_t stream) {
  return rope_common(q, k, batch_size, num_heads, seq_len, head_dim, position_offset, theta, rope_table,
                     table_positions, false, stream);
}

int hrm_rope_embed_token_major(void* q, void* k, int64_t batch_size, int64_t seq_len, int64_t num_heads,
                               int64_t head_dim, int64_t position_offset, float theta, const float* rope_table,
                               int64_t table_positions, hrm_stream_t stream) {
  return rope_common(q, k, batch_size, num_heads, seq_len, head_dim, position_offset, theta, rope_table,
                     table_positions, true, stream);
}

int hrm_rope_table_build(float* table, int64_t max_positions, int64_t head_dim, float theta, hrm_stream_t stream) {
  if (max_positions < 0 || head_dim <= 0 || head_dim % 2 != 0 || head_dim > INT32_MAX) return HRM_ERR_INVALID_SHAPE;
  if (max_positions > INT32_MAX) return HRM_ERR_SIZE_OVERFLOW;
  if (max_positions == 0) return HRM_OK;
  if (!table) return HRM_ERR_NULL_POINTER;
  if (mul_checked(mul_checked(max_positions, head_dim), 4) < 0) return HRM_ERR_SIZE_OVERFLOW;
  return cuda_status(hrm::launch_rope_table(table, max_positions, head_dim, theta, as_cuda(stream)));
}

int hrm_embedding_lookup(const uint32_t* input_ids, const void* embedding_table, void* output, int64_t batch_size,
                         int64_t seq_len, int64_t hidden_size, int64_t vocab_size, float embedding_scale,
                         hrm_stream_t stream) {
  if (batch_size < 0 || seq_len < 0 || hidden_size <= 0 || vocab_size <= 0 || vocab_size > UINT32_MAX)
    return HRM_ERR_INVALID_SHAPE;
  const int64_t tokens = mul_checked(batch_size, seq_len);
  if (tokens < 0) return HRM_ERR_SIZE_OVERFLOW;
  if (tokens == 0) return HRM_OK;
  if (!input_ids || !embedding_table || !output) return HRM_ERR_NULL_POINTER;
  const int64_t obytes = mul_checked(mul_checked(tokens, hidden_size), 2);
  const int64_t tbytes = mul_checked(mul_checked(vocab_size, hidden_size), 2);
  if (obytes < 0 || tbytes < 0) return HRM_ERR_SIZE_OVERFLOW;
  if (overlap(output, obytes, embedding_table, tbytes) || overlap(output, obytes, input_ids, tokens * 4))
    return HRM_ERR_ALIASING;
  return cuda_status(hrm::launch_embedding(input_ids, embedding_table, output, tokens, hidden_size, vocab_size,
                                           embedding_scale, as_cuda(stream)));
}

int hrm_embed_rms_norm(const uint32_t* input_ids, const void* embedding_table, void* hidden_out, void* normed_out,
                       const void* weight, int64_t rows, int64_t hidden_size, int64_t vocab_size,
                       float embedding_scale, float eps, hrm_stream_t stream) {
  if (rows < 0 || hidden_size <= 0 || hidden_size > INT32_MAX || vocab_size <= 0 || vocab_size > UINT32_MAX)
    return HRM_ERR_INVALID_SHAPE;
  if (rows == 0) return HRM_OK;
  if (!input_ids || !embedding_table || !normed_out) return HRM_ERR_NULL_POINTER;
  const int64_t obytes = mul_checked(mul_checked(rows, hidden_size), 2);
  const int64_t tbytes = mul_checked(mul_checked(vocab_size, hidden_size), 2);
  if (obytes < 0 || tbytes < 0) return HRM_ERR_SIZE_OVERFLOW;
  if (overlap(normed_out, obytes, embedding_table, tbytes) || overlap(hidden_out, obytes, embedding_table, tbytes) ||
      overlap(normed_out, obytes, hidden_out, obytes) || overlap(normed_out, obytes, input_ids, rows * 4) ||
      overlap(hidden_out, obytes, input_ids, rows * 4) || overlap(weight, hidden_size * 2, normed_out, obytes) ||
      overlap(weight, hidden_size * 2, hidden_out, obytes))
    return HRM_ERR_ALIASING;
  return cuda_status(hrm::launch_embed_rms_norm(input_ids, embedding_table, hidden_out, normed_out, weight, rows,
                                                hidden_size, vocab_size, embedding_scale, eps, as_cuda(stream)));
}

int hrm_split_gqkv_rope(const void* gqkv, void* gate_out, void* q_out, void* k_out, void* v_out, void* k_cache,
                        void* v_cache, int64_t batch_size, int64_t seq_len, int64_t num_heads, int64_t head_dim,
                        int64_t position_offset, float theta, const float* rope_table, int64_t table_positions,
                        int64_t cache_len, int64_t cache_offset, hrm_stream_t stream) {
  if (batch_size < 0 || num_heads < 0 || seq_len < 0 || head_dim <= 0 || head_dim % 2 != 0 ||
      position_offset < 0 || cache_offset < 0 || num_heads > INT32_MAX || head_dim > INT32_MAX)
    return HRM_ERR_INVALID_SHAPE;
  // offset + seq <= INT32_MAX, checked without forming a sum that could overflow
  if (seq_len > INT32_MAX || position_offset > INT32_MAX - seq_len) return HRM_ERR_SIZE_OVERFLOW;
  if ((k_cache == nullptr) != (v_cache == nullptr)) return HRM_ERR_NULL_POINTER;
  const bool cache = k_cache != nullptr;
  if (cache && (cache_len < 0 || seq_len > cache_len || cache_offset > cache_len - seq_len))
    return HRM_ERR_INVALID_SHAPE;
  if (batch_size == 0 || num_heads == 0 || seq_len == 0) return HRM_OK;
  if (!gqkv || !gate_out || !q_out || !k_out || !v_out) return HRM_ERR_NULL_POINTER;
  const int64_t bytes = mul_checked(mul_checked(mul_checked(mul_checked(batch_size, num_heads), seq_len), head_dim), 2);
  const int64_t in_bytes = mul_checked(bytes, 4);
  const int64_t cbytes =
      cache ? mul_checked(mul_checked(mul_checked(mul_checked(batch_size, num_heads), cache_len), head_dim), 2) : 0;
  if (bytes < 0 || in_bytes < 0 || cbytes < 0) return HRM_ERR_SIZE_OVERFLOW;
  const void* bufs[7] = {gqkv, gate_out, q_out, k_out, v_out, k_cache, v_cache};
  const int64_t sizes[7] = {in_bytes, bytes, bytes, bytes, bytes, cbytes, cbytes};
  for (int x = 0; x < 7; ++x)
    for (int y = x + 1; y < 7; ++y)
      if (overlap(bufs[x], sizes[x], bufs[y], sizes[y])) return HRM_ERR_ALIASING;
  if (rope_table != nullptr) {
    if (table_positions < position_offset + seq_len) return HRM_ERR_TABLE_RANGE;
    const int64_t tbytes = mul_checked(mul_checked(table_positions, head_dim), 4);
    if (tbytes < 0) return HRM_ERR_SIZE_OVERFLOW;
    for (int x = 1; x < 7; ++x)
      if (overlap(rope_table, tbytes, bufs[x], sizes[x])) return HRM_ERR_ALIASING;
  }
  return cuda_status(hrm::launch_split_rope(gqkv, gate_out, q_out, k_out, v_out, k_cache, v_cache, batch_size,
                                            num_heads, seq_len, head_dim, position_offset, theta, rope_table,
                                            cache ? cache_len : 0, cache ? cache_offset : 0, as_cuda(stream)));
}

int hrm_convert_to_bf16(const void* src, int src_dtype, void* dst, int64_t n, hrm_stream_t stream) {
  if (src_dtype != HRM_DTYPE_BF16 && src_dtype != HRM_DTYPE_F32 && src_dtype != HRM_DTYPE_F16) return HRM_ERR_DTYPE;
  if (n < 0) return HRM_ERR_INVALID_SHAPE;
  if (n == 0) return HRM_OK;
  if (!src || !dst) return HRM_ERR_NULL_POINTER;
  const int64_t in_bytes = mul_checked(n, src_dtype == HRM_DTYPE_F32 ? 4 : 2), out_bytes = mul_checked(n, 2);
  if (in_bytes < 0 || out_bytes < 0) return HRM_ERR_SIZE_OVERFLOW;
  if (overlap(src, in_bytes, dst, out_bytes)) return HRM_ERR_ALIASING;
  return cuda_status(hrm::launch_convert_to_bf16(src, src_dtype, dst, n, as_cuda(stream)));
}

int hrm_upload_to_bf16(const void* src, int src_dtype, void* dst, int64_t n, void* staging,
                       int64_t staging_bytes, hrm_stream_t stream) {
  if (src_dtype != HRM_DTYPE_BF16 && src_dtype != HRM_DTYPE_F32 && src_dtype != HRM_DTYPE_F16) return HRM_ERR_DTYPE;
  if (n < 0 || staging_bytes < 0) return HRM_ERR_INVALID_SHAPE;
  if (n == 0) return HRM_OK;
  if (!src || !dst || !staging) return HRM_ERR_NULL_POINTER;
  if (staging_bytes < 16) return HRM_ERR_INVALID_SHAPE;
  const int64_t size = src_dtype == HRM_DTYPE_F32 ? 4 : 2;
  const int64_t in_bytes = mul_checked(n, size), out_bytes = mul_checked(n, 2);
  if (in_bytes < 0 || out_bytes < 0) return HRM_ERR_SIZE_OVERFLOW;
  if (overlap(staging, staging_bytes, dst, out_bytes) || overlap(src, in_bytes, dst, out_bytes) ||
      overlap(src, in_bytes, staging, staging_bytes))
    return HRM_ERR_ALIASING;
  const cudaStream_t s = as_cuda(stream);
  // bf16 needs no conversion: one copy straight into dst.
  if (src_dtype == HRM_DTYPE_BF16) return cuda_status(cudaMemcpyAsync(dst, src, (size_t)in_bytes, cudaMemcpyDefault, s));
  // Pieces of a whole number of 16-byte groups, so that every piece starts the
  // staging buffer with a whole element and its output at a whole element.
  const int64_t piece = staging_bytes / 16 * 16;
  for (int64_t off = 0; off < in_bytes; off += piece) {
    const int64_t len = in_bytes - off < piece ? in_bytes - off : piece;
    cudaError_t e = cudaMemcpyAsync(staging, static_cast<const char*>(src) + off, (size_t)len, cudaMemcpyDefault, s);
    if (e != cudaSuccess) return cuda_status(e);
    e = hrm::launch_convert_to_bf16(staging, src_dtype, static_cast<char*>(dst) + off / size * 2, len / size, s);
    if (e != cudaSuccess) return cuda_status(e);
  }
  return HRM_OK;
}

int hrm_wait_timeouts(unsigned int* count, int reset) {
  if (!count) return HRM_ERR_NULL_POINTER;
  return cuda_status(hrm::rownorm_wait_timeouts(count, reset != 0));
}

}  // extern "C"
