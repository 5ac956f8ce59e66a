/*
 * hrm_ops.h -- C ABI of the sm_100a per-token layer operators for the
 * HRM-Text forward/decode loop (ArjavDesa912/hrm-text-cuda).
 *
 * Every entry point replaces one launch wrapper of `HrmForwardPass` in the
 * reference's src/lib.rs (cited per function) together with the PTX kernel
 * that wrapper loaded (src/kernels/<name>.cu).  The functions are:
 *   - stateless: no allocation, no free, no host synchronisation;
 *   - stream ordered: work is queued on `stream` (NULL = the legacy default
 *     stream of the current device) in the caller's current CUDA context,
 *     which is the device primary context that cudarc binds;
 *   - reentrant: the only globals are per-device launch tuning values that
 *     are written once (SM count), so calls from several host threads on
 *     different streams are safe.
 * Device pointers are plain addresses (cudarc: `*slice.device_ptr()`).
 * bf16 tensors are passed as `void*` holding IEEE bfloat16 (the top 16 bits
 * of a binary32), row-major.  Sizes are int64_t element counts.
 *
 * Return value: HRM_OK (0) or one of the hrm_status codes below; a CUDA
 * launch failure is reported as HRM_ERR_CUDA + cudaError_t.  Nothing here
 * traps or aborts, and no call leaves work half-queued on an argument error
 * (arguments are checked before anything is launched).
 */
#ifndef HRM_OPS_H
#define HRM_OPS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t and CUstream (cudarc: `*dev.cu_stream()`). */
typedef struct CUstream_st* hrm_stream_t;

enum hrm_status {
  HRM_OK = 0,
  HRM_ERR_NULL_POINTER = 1,   /* a required pointer is NULL                     */
  HRM_ERR_INVALID_SHAPE = 2,  /* negative size, odd head_dim, hidden == 0, ...   */
  HRM_ERR_SIZE_OVERFLOW = 3,  /* a product of sizes overflows int64 / grid limits */
  HRM_ERR_ALIASING = 4,       /* buffers that must be distinct overlap           */
  HRM_ERR_TABLE_RANGE = 5,    /* position_offset + seq_len exceeds the rope table */
  HRM_ERR_DTYPE = 6,          /* unsupported element type                        */
  HRM_ERR_SCRATCH_LIMIT = 7,  /* request larger than a fixed in-library scratch  */
  HRM_ERR_CUDA = 1000         /* HRM_ERR_CUDA + cudaError_t of the failed launch  */
};

/* Human-readable text for a status code (static storage, never NULL). */
const char* hrm_status_string(int status);

/* ABI version: major * 10000 + minor * 100 + patch. */
int hrm_abi_version(void);

/* ------------------------------------------------------------------------ */
/* Residual add.  z_out[i] = bf16_rn(f32(z_a[i]) + f32(z_b[i])), i < n.
 * Replaces HrmForwardPass::additive_inject (src/lib.rs:378-399) and
 * additive_inject_kernel_vec8 (src/kernels/additive_inject.cu:6-44).
 * z_out may alias z_a or z_b exactly (elementwise, in place is fine).      */
int hrm_additive_inject(const void* z_a, const void* z_b, void* z_out,
                        int64_t total_elements, hrm_stream_t stream);

/* Sigmoid-gated attention output:
 *   out[i] = bf16_rn((1 / (1 + exp(-g))) * a),  g = f32(gate[i]), a = f32(attn[i])
 * (exp by the __expf intrinsic, as in the reference).  hrm_apply_attn_gate
 * writes in place over attn_out and replaces HrmForwardPass::apply_attn_gate
 * (src/lib.rs:607-630, src/kernels/apply_attn_gate.cu:8-42);
 * hrm_gated_attn_output writes to `output` (which may alias attn_out exactly)
 * and replaces HrmForwardPass::gated_attn_output (src/lib.rs:505-527,
 * src/kernels/gated_attn_output.cu:8-43).                                   */
int hrm_apply_attn_gate(const void* gate, void* attn_out, int64_t total_elements, hrm_stream_t stream);
int hrm_gated_attn_output(const void* gate, const void* attn_out, void* output, int64_t total_elements,
                          hrm_stream_t stream);

/* dst[r, j] = src[j] for r < n_copies, j < vec_len (bf16).  Replaces
 * HrmForwardPass::broadcast_vec (src/lib.rs:748-767,
 * src/kernels/broadcast_vec.cu:7-21), used to initialise z_L from z_l_init
 * (src/lib.rs:1203).  dst must not overlap src.                             */
int hrm_broadcast_vec(void* dst, const void* src, int64_t n_copies, int64_t vec_len, hrm_stream_t stream);

/* RMSNorm over the last dim of a row-major [rows, hidden_size] bf16 tensor:
 *   ss  = sum_j f32(x_j)^2   (fp32, the reference's 256-thread order)
 *   inv = 1 / sqrtf(ss / hidden_size + eps)
 *   y_j = bf16_rn(f32(x_j) * inv)            weight == NULL (reference form)
 *   y_j = bf16_rn((f32(x_j) * inv) * f32(w_j))   weight = bf16 [hidden_size]
 * Replaces HrmForwardPass::rms_norm (src/lib.rs:401-422; eps was read from
 * config.norm_eps there and is explicit here) and rms_norm_kernel
 * (src/kernels/rms_norm.cu:8-66).  output must not overlap input.          */
int hrm_rms_norm(const void* input, void* output, const void* weight,
                 int64_t rows, int64_t hidden_size, float eps,
                 hrm_stream_t stream);

/* fp32-I/O RMSNorm (same formula, fp32 x / w / y).  No reference
 * counterpart: it serves fp32 activations with the same reduction order as
 * rms_norm_kernel (src/kernels/rms_norm.cu:25-59).                         */
int hrm_rms_norm_f32(const float* input, float* output, const float* weight,
                     int64_t rows, int64_t hidden_size, float eps,
                     hrm_stream_t stream);

/* Fused residual add + RMSNorm (one HBM pass):
 *   r = bf16_rn(f32(x) + f32(branch))  -> residual_out
 *   y = rms_norm(r) [* weight]         -> normed_out  (statistics from the
 *                                         bf16-rounded r, as when the
 *                                         reference reads r back from HBM)
 * Replaces the pair additive_inject -> rms_norm of src/lib.rs:976-979 and
 * src/lib.rs:1015-1028 + 969.  residual_out may alias x or branch exactly;
 * normed_out must not overlap any other buffer.                             */
int hrm_add_rms_norm(const void* x, const void* branch, void* residual_out,
                     void* normed_out, const void* weight, int64_t rows,
                     int64_t hidden_size, float eps, hrm_stream_t stream);

/* Rotary embedding, in place on q and k, layout [batch, heads, seq, head_dim]
 * bf16, rotate-half (NeoX) pairing (x[i], x[i + head_dim/2]):
 *   a  = (float)(s + position_offset) * expf((-2.0f*i*logf(theta))/head_dim)
 *   x0' = x0*cos(a) - x1*sin(a);  x1' = x1*cos(a) + x0*sin(a)
 * rope_table == NULL: angles are evaluated in-kernel with exactly that fp32
 * formula (as src/kernels/rope_embed.cu:41-43 does).  Otherwise rope_table
 * is an fp32 table written by hrm_rope_table_build for the same head_dim and
 * theta, with table_positions rows; position_offset + seq_len must not
 * exceed table_positions.  Replaces HrmForwardPass::rope_embed
 * (src/lib.rs:424-458; theta was config.rope_theta there) and
 * rope_embed_kernel (src/kernels/rope_embed.cu:12-54).  q and k must not
 * overlap.  head_dim must be even.                                          */
int hrm_rope_embed(void* q, void* k, int64_t batch_size, int64_t num_heads,
                   int64_t seq_len, int64_t head_dim, int64_t position_offset,
                   float theta, const float* rope_table,
                   int64_t table_positions, hrm_stream_t stream);

/* The same rotation for token-major q and k, [batch, seq, heads, head_dim]
 * (each token's heads contiguous, as a projection GEMM writes them); position
 * of token s is s + position_offset.  No reference counterpart (the reference
 * splits into [batch, heads, seq, head_dim] first); same arguments and rules
 * as hrm_rope_embed, note the (batch, seq, heads) order.                    */
int hrm_rope_embed_token_major(void* q, void* k, int64_t batch_size, int64_t seq_len,
                               int64_t num_heads, int64_t head_dim, int64_t position_offset,
                               float theta, const float* rope_table,
                               int64_t table_positions, hrm_stream_t stream);

/* Writes the fp32 cos/sin table used by hrm_rope_embed:
 *   table[p * head_dim + i]            = cos(a(p, i)),
 *   table[p * head_dim + head_dim/2 + i] = sin(a(p, i)),  p < max_positions,
 * with a(p, i) the angle formula above at s + position_offset = p.  The
 * table has max_positions * head_dim floats.  No reference counterpart
 * (the reference evaluates the angle per element); build it once per
 * (head_dim, theta, max_positions), e.g. next to ScratchBuffers.            */
int hrm_rope_table_build(float* table, int64_t max_positions,
                         int64_t head_dim, float theta, hrm_stream_t stream);

/* SwiGLU gate: out[i] = bf16_rn((g * (1 / (1 + exp(-g)))) * u), g = f32(gate[i]),
 * u = f32(up[i]), exp evaluated by the __expf intrinsic as in the reference.
 * Replaces HrmForwardPass::swiglu_ffn (src/lib.rs:483-504) and
 * swiglu_ffn_kernel (src/kernels/swiglu_ffn.cu:9-47).  output may alias
 * gate or up exactly.                                                       */
int hrm_swiglu_ffn(const void* gate, const void* up, void* output,
                   int64_t total_elements, hrm_stream_t stream);

/* Token-embedding gather:
 *   id' = id >= vocab_size ? vocab_size - 1 : id
 *   out[t, j] = bf16_rn(f32(table[id', j]) * embedding_scale)
 * for t < batch_size * seq_len (ids row-major [batch, seq]).  Bit-exact with
 * the reference.  Replaces HrmForwardPass::embedding_lookup
 * (src/lib.rs:529-565) and embedding_lookup_kernel
 * (src/kernels/embedding_lookup.cu:10-51).  Any hidden_size is accepted (the
 * reference kernel needs hidden_size % 8 == 0).                            */
int hrm_embedding_lookup(const uint32_t* input_ids, const void* embedding_table,
                         void* output, int64_t batch_size, int64_t seq_len,
                         int64_t hidden_size, int64_t vocab_size,
                         float embedding_scale, hrm_stream_t stream);

/* Fused embedding gather + RMSNorm (one pass over the gathered rows):
 *   h = embedding_lookup(...)          -> hidden_out (may be NULL: not stored)
 *   y = rms_norm(h) [* weight]         -> normed_out
 * Replaces embedding_lookup (src/lib.rs:1191-1200) followed by the first
 * rms_norm on the same rows (src/lib.rs:969).                               */
int hrm_embed_rms_norm(const uint32_t* input_ids, const void* embedding_table,
                       void* hidden_out, void* normed_out, const void* weight,
                       int64_t rows, int64_t hidden_size, int64_t vocab_size,
                       float embedding_scale, float eps, hrm_stream_t stream);

/* Fused attention-input preparation: split + RoPE + KV-cache write, reading
 * the projection output once.
 *   gqkv      [batch, seq, 4*heads*head_dim] bf16; per token the heads are laid
 *             out [gate heads | q heads | k heads | v heads]
 *   gate_out  [batch, seq, heads, head_dim]        copy of the gate heads
 *   q_out, k_out, v_out [batch, heads, seq, head_dim]; q and k rotated exactly
 *             as hrm_rope_embed does at position_offset (rope_table optional,
 *             same rules), v copied
 *   k_cache, v_cache: both NULL (no cache write) or both [batch, heads,
 *             cache_len, head_dim]; the rotated k and the v of token s are
 *             also written at cache position cache_offset + s
 *             (cache_offset + seq_len <= cache_len)
 * Replaces split_gqkv (src/lib.rs:567-605, src/kernels/split_gqkv.cu:10-49)
 * -> rope_embed (src/lib.rs:821-836) -> kv_cache_update (src/lib.rs:706-747,
 * src/kernels/kv_cache_update.cu:12-48) as the attention prologue runs them
 * (src/lib.rs:798-857 and 900-916; prefill writes the cache at 0, decode at
 * cached_len, which is also its position_offset).  Outputs are bit-identical
 * to that three-kernel sequence.  head_dim must be even; no two buffers may
 * overlap.                                                                  */
int hrm_split_gqkv_rope(const void* gqkv, void* gate_out, void* q_out, void* k_out, void* v_out,
                        void* k_cache, void* v_cache, int64_t batch_size, int64_t seq_len,
                        int64_t num_heads, int64_t head_dim, int64_t position_offset, float theta,
                        const float* rope_table, int64_t table_positions, int64_t cache_len,
                        int64_t cache_offset, hrm_stream_t stream);

/* Element types of checkpoint tensors (safetensors dtypes). */
enum hrm_dtype { HRM_DTYPE_BF16 = 0, HRM_DTYPE_F32 = 1, HRM_DTYPE_F16 = 2 };

/* Converts n little-endian values of src_dtype at `src` (raw checkpoint
 * bytes copied to the device, any byte alignment) to bf16 at `dst`, with the
 * conversions of the reference's weight loader raw_to_bf16
 * (src/lib.rs:1981-2008), i.e. half 2.7.1's bf16::from_f32 (round to nearest
 * even; a NaN keeps its sign and top payload bits and gets the quiet bit) and
 * f16::to_f32 (exact widening) before it.  BF16 is copied as is.  Replaces
 * that host loop so a checkpoint can be uploaded raw and converted on the
 * GPU.  dst must not overlap src.                                           */
int hrm_convert_to_bf16(const void* src, int src_dtype, void* dst, int64_t n, hrm_stream_t stream);

/* Upload + conversion of one checkpoint tensor: n little-endian values of
 * src_dtype at `src` -- host memory (pinned for full PCIe speed; pageable
 * works, the copy then returns once the driver has staged the bytes) or
 * device memory -- are copied, in pieces of at most staging_bytes, into the
 * caller's device buffer `staging` and converted from there into the bf16
 * device tensor `dst` with the rules of hrm_convert_to_bf16, all on
 * `stream` (bf16 values need no conversion and are copied straight into
 * dst).  Replaces the reference loader's raw_to_bf16 host loop followed
 * by htod_copy (src/lib.rs:1981-2008, 2055-2112); its gate_up split
 * (src/lib.rs:2072-2078) is two calls on the two halves of the tensor's
 * bytes.  `staging` is scratch: the pieces reuse it in stream order, so no
 * work on another stream may use it until `stream` has passed this call.
 * staging_bytes >= 16 (a 16-byte aligned staging buffer takes the vectorised
 * conversion); dst must not overlap staging or src.                         */
int hrm_upload_to_bf16(const void* src, int src_dtype, void* dst, int64_t n, void* staging,
                       int64_t staging_bytes, hrm_stream_t stream);

/* Bytes of device scratch compiled into the library for
 * hrm_upload_to_bf16_static (held on every GPU the library is loaded on). */
#define HRM_UPLOAD_STATIC_BYTES (16 * 1024 * 1024)

/* hrm_upload_to_bf16 without the caller's staging buffer, for callers that
 * must not allocate device memory: a process whose GPU memory is reserved in
 * full by another allocator (a serving engine's pool, a framework's caching
 * allocator), or one that reloads weights while other streams run and cannot
 * afford cudaMalloc's device synchronisation.  No counterpart in the
 * reference.  The raw bytes go through a fixed device array of
 * HRM_UPLOAD_STATIC_BYTES inside the library, which every GPU that loads the
 * library holds until the process exits.  Limit: an f32 or f16 request of more
 * than HRM_UPLOAD_STATIC_BYTES raw bytes returns HRM_ERR_SCRATCH_LIMIT (upload
 * a larger tensor in several calls on consecutive element ranges; the
 * conversion is elementwise); bf16 is copied straight into dst and has no
 * limit.  The call allocates nothing (no cudaMalloc, no cudaFree).  The first
 * call on a device looks up the array's address there (cudaGetSymbolAddress,
 * with that device current); make that first call before any stream capture.
 * All calls share the array: calls that overlap on the GPU (on different
 * streams, or from several host threads) race on it, so order them on one
 * stream.  Results equal hrm_upload_to_bf16's bit for bit.                  */
int hrm_upload_to_bf16_static(const void* src, int src_dtype, void* dst, int64_t n, hrm_stream_t stream);

/* Number of bounded device-side waits that ran out on the current device
 * since the library was loaded there (or since the last reset).  The
 * bulk-copy kernels of the opt-in build wait on mbarriers with a deadline of
 * about one second; a wait that runs out counts itself here and the kernel
 * returns instead of hanging, leaving the affected rows unwritten.  It reads
 * device memory: call it after synchronizing the streams that ran the
 * library's kernels.  0 in correct operation (and always 0 in the default
 * build, which has no waits).  reset != 0 sets the count back to 0 after
 * reading it.  No reference counterpart (the reference's kernels have no
 * waits).                                                                   */
int hrm_wait_timeouts(unsigned int* count, int reset);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* HRM_OPS_H */
