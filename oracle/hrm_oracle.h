/*
 * hrm_oracle.h -- CPU restatement of the reference's per-token layer kernels
 * (ArjavDesa912/hrm-text-cuda, src/kernels/<op>.cu), used ONLY as the checker
 * by the tests and as the timed CPU baseline.  It is never linked into, or
 * called by, the sm_100a library.
 *
 * Parity pins: the reference's own known answers (src/lib.rs:2227-2279) are
 * fixtures in tests/golden/, and the reference kernels compiled from source
 * (oracle/_ref, built by oracle/Makefile) are run on the GPU against this
 * restatement by the GPU tests.
 *
 * bf16 values are uint16_t bit patterns.  Arithmetic is IEEE fp32 with no
 * contraction (built with -ffp-contract=off); where the reference's nvcc
 * build contracts a multiply-add into an FMA (the RMSNorm sum of squares, the
 * RoPE rotation) the oracle calls fmaf in the same place.  Transcendentals
 * come from the C library (expf, logf, sinf, cosf), not CUDA's; the tests
 * allow for that difference (2 bf16 ulp) where it can show.
 */
#ifndef HRM_ORACLE_H
#define HRM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

uint16_t ora_f32_to_bf16(float x); /* round to nearest even; NaN -> 0x7fff */
float ora_bf16_to_f32(uint16_t h);
int ora_max_threads(void);
void ora_set_threads(int n);

/* additive_inject.cu:26-31 / :38-42 */
void ora_additive_inject(const uint16_t* a, const uint16_t* b, uint16_t* out, int64_t n);

/* swiglu_ffn.cu:27-35 / :40-45 (expf in place of the __expf intrinsic) */
void ora_swiglu_ffn(const uint16_t* gate, const uint16_t* up, uint16_t* out, int64_t n);

/* rms_norm.cu:25-65 with the optional weight: y = (x * inv) * w. */
void ora_rms_norm(const uint16_t* x, uint16_t* y, const uint16_t* w, int64_t rows, int64_t hidden, float eps);
void ora_rms_norm_f32(const float* x, float* y, const float* w, int64_t rows, int64_t hidden, float eps);

/* additive_inject then rms_norm on the bf16-rounded sum. */
void ora_add_rms_norm(const uint16_t* x, const uint16_t* branch, uint16_t* residual, uint16_t* normed,
                      const uint16_t* w, int64_t rows, int64_t hidden, float eps);

/* embedding_lookup.cu:27-50 */
void ora_embedding_lookup(const uint32_t* ids, const uint16_t* table, uint16_t* out, int64_t tokens, int64_t hidden,
                          int64_t vocab, float scale);

/* embedding_lookup then rms_norm on the gathered rows (hidden_out may be NULL). */
void ora_embed_rms_norm(const uint32_t* ids, const uint16_t* table, uint16_t* hidden_out, uint16_t* normed,
                        const uint16_t* w, int64_t rows, int64_t hidden, int64_t vocab, float scale, float eps);

/* rope_embed.cu:22-53; table == NULL evaluates the angle per element, else
 * reads cos/sin from a table laid out as hrm_rope_table_build writes it. */
void ora_rope_table(float* table, int64_t positions, int64_t head_dim, float theta);
void ora_rope_embed(uint16_t* q, uint16_t* k, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                    int64_t offset, float theta, const float* table);
/* The same rotation over token-major [batch, seq, heads, head_dim] rows. */
void ora_rope_embed_token_major(uint16_t* q, uint16_t* k, int64_t batch, int64_t seq, int64_t heads,
                                int64_t head_dim, int64_t offset, float theta, const float* table);

/* apply_attn_gate.cu:28-29 / gated_attn_output.cu:71-72:
 * out = (1 / (1 + exp(-g))) * a (expf in place of the __expf intrinsic). */
void ora_gated_attn_output(const uint16_t* gate, const uint16_t* attn, uint16_t* out, int64_t n);

/* broadcast_vec.cu:102-105: dst[r, j] = src[j]. */
void ora_broadcast_vec(uint16_t* dst, const uint16_t* src, int64_t n_copies, int64_t vec_len);

/* The reference's weight loader raw_to_bf16 (src/lib.rs:1981-2008) with the
 * half 2.7.1 conversions it calls (Cargo.lock: half 2.7.1, not vendored;
 * restated from its documented behaviour): dtype 0 bf16 copy, 1 f32, 2 f16;
 * src is little-endian bytes. */
void ora_convert_to_bf16(const void* src, int dtype, uint16_t* dst, int64_t n);

/* split_gqkv.cu:27-48: per token [gate | q | k | v] heads -> gate [b, s, h, :],
 * q, k, v [b, h, s, :] (plain copies). */
void ora_split_gqkv(const uint16_t* gqkv, uint16_t* gate, uint16_t* q, uint16_t* k, uint16_t* v, int64_t batch,
                    int64_t seq, int64_t heads, int64_t head_dim);

/* kv_cache_update.cu:78-95: [b, h, s, :] -> cache [b, h, max_len, :] at row
 * s (prefill) or cached_len + s (decode). */
void ora_kv_cache_update(const uint16_t* k, const uint16_t* v, uint16_t* k_cache, uint16_t* v_cache, int64_t batch,
                         int64_t heads, int64_t seq, int64_t head_dim, int64_t max_len, int64_t cached_len,
                         int is_decode);

/* Counter-based synthetic inputs (SplitMix64 + Box-Muller keyed by seed,
 * tensor tag and global element index): normal bf16 values and token ids of
 * elements [start, start + n) of the (seed, tag) stream. */
void ora_fill_normal_bf16(uint16_t* out, int64_t n, uint64_t seed, uint64_t tag, int64_t start, double std_,
                          double mean);
void ora_fill_ids(uint32_t* out, int64_t n, uint64_t seed, uint64_t tag, int64_t start, uint32_t vocab);

#ifdef __cplusplus
}
#endif

#endif
