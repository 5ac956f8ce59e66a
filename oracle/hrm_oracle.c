/*
 * hrm_oracle.c -- test-only CPU restatement of the reference kernels (see
 * hrm_oracle.h).  Each function cites the reference lines it restates.
 * OpenMP parallelises over rows / elements only; the arithmetic of each
 * element is sequential and independent of the thread count.
 */
#include "hrm_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

#define REF_THREADS 256 /* rms_norm launch: block = 256 (src/lib.rs:408-417) */

uint16_t ora_f32_to_bf16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fffu; /* canonical NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

float ora_bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

int ora_max_threads(void) { return omp_get_max_threads(); }
void ora_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}

/* additive_inject.cu:26-31: fa + fb in fp32, then RNE. */
void ora_additive_inject(const uint16_t* a, const uint16_t* b, uint16_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = ora_f32_to_bf16(ora_bf16_to_f32(a[i]) + ora_bf16_to_f32(b[i]));
}

/* swiglu_ffn.cu:31-35: sig = 1/(1+exp(-g)); out = (g*sig)*u. */
void ora_swiglu_ffn(const uint16_t* gate, const uint16_t* up, uint16_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float g = ora_bf16_to_f32(gate[i]), u = ora_bf16_to_f32(up[i]);
    const float sig = 1.0f / (1.0f + expf(-g));
    out[i] = ora_f32_to_bf16(g * sig * u);
  }
}

/*
 * Sum of squares of one row in the order rms_norm_kernel produces it
 * (rms_norm.cu:25-56): thread t of 256 accumulates v[t], v[t+256], ... with a
 * fused multiply-add (nvcc contracts `local_sum += v * v`); a shuffle-down
 * tree with offsets 16..1 in each warp; the 8 warp sums reduced by a
 * shuffle-down tree with offsets 4, 2, 1.  Only lane 0's value survives in
 * each tree, so each level is "x[m] += x[m + off] for m < off".
 */
static float ref_sum_squares(const float* v, int64_t hidden) {
  float part[REF_THREADS];
  for (int t = 0; t < REF_THREADS; ++t) {
    float s = 0.0f;
    for (int64_t i = t; i < hidden; i += REF_THREADS) s = fmaf(v[i], v[i], s);
    part[t] = s;
  }
  float warp_sum[REF_THREADS / 32];
  for (int w = 0; w < REF_THREADS / 32; ++w) {
    float* x = part + 32 * w;
    for (int off = 16; off > 0; off >>= 1)
      for (int m = 0; m < off; ++m) x[m] = x[m] + x[m + off];
    warp_sum[w] = x[0];
  }
  for (int off = (REF_THREADS / 32) / 2; off > 0; off >>= 1)
    for (int m = 0; m < off; ++m) warp_sum[m] = warp_sum[m] + warp_sum[m + off];
  return warp_sum[0];
}

/* rms_norm.cu:58-59 */
static float ref_inv_rms(float ss, int64_t hidden, float eps) {
  const float rms = sqrtf(ss / (float)hidden + eps);
  return 1.0f / rms;
}

/* Normalises one row already converted to fp32 (v) into bf16 y. */
static void norm_row_bf16(const float* v, uint16_t* y, const uint16_t* w, int64_t hidden, float eps) {
  const float inv = ref_inv_rms(ref_sum_squares(v, hidden), hidden, eps);
  for (int64_t i = 0; i < hidden; ++i) {
    float o = v[i] * inv; /* rms_norm.cu:64 */
    if (w) o = o * ora_bf16_to_f32(w[i]);
    y[i] = ora_f32_to_bf16(o);
  }
}

void ora_rms_norm(const uint16_t* x, uint16_t* y, const uint16_t* w, int64_t rows, int64_t hidden, float eps) {
#pragma omp parallel
  {
    float* v = (float*)malloc((size_t)hidden * sizeof(float));
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      for (int64_t i = 0; i < hidden; ++i) v[i] = ora_bf16_to_f32(x[r * hidden + i]);
      norm_row_bf16(v, y + r * hidden, w, hidden, eps);
    }
    free(v);
  }
}

void ora_rms_norm_f32(const float* x, float* y, const float* w, int64_t rows, int64_t hidden, float eps) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float* v = x + r * hidden;
    const float inv = ref_inv_rms(ref_sum_squares(v, hidden), hidden, eps);
    for (int64_t i = 0; i < hidden; ++i) {
      float o = v[i] * inv;
      if (w) o = o * w[i];
      y[r * hidden + i] = o;
    }
  }
}

/* additive_inject (additive_inject.cu:29-31) then rms_norm of the rounded sum. */
void ora_add_rms_norm(const uint16_t* x, const uint16_t* branch, uint16_t* residual, uint16_t* normed,
                      const uint16_t* w, int64_t rows, int64_t hidden, float eps) {
#pragma omp parallel
  {
    float* v = (float*)malloc((size_t)hidden * sizeof(float));
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      for (int64_t i = 0; i < hidden; ++i) {
        const int64_t e = r * hidden + i;
        const uint16_t s = ora_f32_to_bf16(ora_bf16_to_f32(x[e]) + ora_bf16_to_f32(branch[e]));
        residual[e] = s;
        v[i] = ora_bf16_to_f32(s);
      }
      norm_row_bf16(v, normed + r * hidden, w, hidden, eps);
    }
    free(v);
  }
}

/* embedding_lookup.cu:33-35 */
static int64_t clamp_id(uint32_t id, int64_t vocab) { return id >= (uint32_t)vocab ? vocab - 1 : (int64_t)id; }

/* embedding_lookup.cu:37-50: one fp32 multiply, RNE. */
void ora_embedding_lookup(const uint32_t* ids, const uint16_t* table, uint16_t* out, int64_t tokens, int64_t hidden,
                          int64_t vocab, float scale) {
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < tokens; ++t) {
    const uint16_t* row = table + clamp_id(ids[t], vocab) * hidden;
    for (int64_t j = 0; j < hidden; ++j) out[t * hidden + j] = ora_f32_to_bf16(ora_bf16_to_f32(row[j]) * scale);
  }
}

void ora_embed_rms_norm(const uint32_t* ids, const uint16_t* table, uint16_t* hidden_out, uint16_t* normed,
                        const uint16_t* w, int64_t rows, int64_t hidden, int64_t vocab, float scale, float eps) {
#pragma omp parallel
  {
    float* v = (float*)malloc((size_t)hidden * sizeof(float));
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      const uint16_t* row = table + clamp_id(ids[r], vocab) * hidden;
      for (int64_t j = 0; j < hidden; ++j) {
        const uint16_t h = ora_f32_to_bf16(ora_bf16_to_f32(row[j]) * scale);
        if (hidden_out) hidden_out[r * hidden + j] = h;
        v[j] = ora_bf16_to_f32(h);
      }
      norm_row_bf16(v, normed + r * hidden, w, hidden, eps);
    }
    free(v);
  }
}

/* rope_embed.cu:41: angle = (pos + offset) * exp(((-2*i) * log(theta)) / head_dim). */
static float rope_angle(int pos, int i, int head_dim, float theta) {
  return (float)pos * expf(-2.0f * i * logf(theta) / (float)head_dim);
}

void ora_rope_table(float* table, int64_t positions, int64_t head_dim, float theta) {
  const int64_t half = head_dim / 2;
#pragma omp parallel for schedule(static)
  for (int64_t p = 0; p < positions; ++p)
    for (int64_t i = 0; i < half; ++i) {
      const float a = rope_angle((int)p, (int)i, (int)head_dim, theta);
      table[p * head_dim + i] = cosf(a);
      table[p * head_dim + half + i] = sinf(a);
    }
}

/* rope_embed.cu:45-53 as nvcc contracts it (established by running the
 * reference kernel against every candidate rounding): x0' = fma(x0, c, -(x1*s))
 * for q and k; x1' = fma(x1, c, x0*s) for q but fma(x0, s, x1*c) for k. */
static float rot_lo(float x0, float x1, float c, float s) { return fmaf(x0, c, -(x1 * s)); }
static float rot_hi_q(float x0, float x1, float c, float s) { return fmaf(x1, c, x0 * s); }
static float rot_hi_k(float x0, float x1, float c, float s) { return fmaf(x0, s, x1 * c); }

/* rope_embed.cu:27-53: the pairs (i, i + D/2) of one head row of q and of k
 * at position pos, Q then K. */
static void rope_rows(uint16_t* qr, uint16_t* kr, int pos, int64_t head_dim, float theta, const float* table) {
  const int64_t half = head_dim / 2;
  for (int64_t i = 0; i < half; ++i) {
    float c, s;
    if (table) {
      c = table[(int64_t)pos * head_dim + i];
      s = table[(int64_t)pos * head_dim + half + i];
    } else {
      const float a = rope_angle(pos, (int)i, (int)head_dim, theta);
      c = cosf(a);
      s = sinf(a);
    }
    const float x0 = ora_bf16_to_f32(qr[i]), x1 = ora_bf16_to_f32(qr[i + half]);
    qr[i] = ora_f32_to_bf16(rot_lo(x0, x1, c, s));
    qr[i + half] = ora_f32_to_bf16(rot_hi_q(x0, x1, c, s));
    const float k0 = ora_bf16_to_f32(kr[i]), k1 = ora_bf16_to_f32(kr[i + half]);
    kr[i] = ora_f32_to_bf16(rot_lo(k0, k1, c, s));
    kr[i + half] = ora_f32_to_bf16(rot_hi_k(k0, k1, c, s));
  }
}

/* [B, H, S, D] (rope_embed.cu:35): row (b, h, s) is at position s + offset. */
void ora_rope_embed(uint16_t* q, uint16_t* k, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                    int64_t offset, float theta, const float* table) {
  const int64_t rows = batch * heads * seq;
#pragma omp parallel for schedule(static)
  for (int64_t row = 0; row < rows; ++row)
    rope_rows(q + row * head_dim, k + row * head_dim, (int)(row % seq) + (int)offset, head_dim, theta, table);
}

/* The same rotation over [B, S, H, D]: row (b, s, h) is at position s + offset. */
void ora_rope_embed_token_major(uint16_t* q, uint16_t* k, int64_t batch, int64_t seq, int64_t heads,
                                int64_t head_dim, int64_t offset, float theta, const float* table) {
  const int64_t rows = batch * seq * heads;
#pragma omp parallel for schedule(static)
  for (int64_t row = 0; row < rows; ++row)
    rope_rows(q + row * head_dim, k + row * head_dim, (int)((row / heads) % seq) + (int)offset, head_dim, theta,
              table);
}

/* split_gqkv.cu:27-48 */
void ora_split_gqkv(const uint16_t* gqkv, uint16_t* gate, uint16_t* q, uint16_t* k, uint16_t* v, int64_t batch,
                    int64_t seq, int64_t heads, int64_t head_dim) {
#pragma omp parallel for schedule(static)
  for (int64_t tok = 0; tok < batch * seq; ++tok) {
    const int64_t b = tok / seq, s = tok % seq;
    const uint16_t* in = gqkv + tok * 4 * heads * head_dim;
    for (int64_t h = 0; h < heads; ++h) {
      const int64_t o = ((b * heads + h) * seq + s) * head_dim;
      memcpy(gate + (tok * heads + h) * head_dim, in + h * head_dim, (size_t)head_dim * 2);
      memcpy(q + o, in + (heads + h) * head_dim, (size_t)head_dim * 2);
      memcpy(k + o, in + (2 * heads + h) * head_dim, (size_t)head_dim * 2);
      memcpy(v + o, in + (3 * heads + h) * head_dim, (size_t)head_dim * 2);
    }
  }
}

/* kv_cache_update.cu:78-95 */
void ora_kv_cache_update(const uint16_t* k, const uint16_t* v, uint16_t* k_cache, uint16_t* v_cache, int64_t batch,
                         int64_t heads, int64_t seq, int64_t head_dim, int64_t max_len, int64_t cached_len,
                         int is_decode) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < batch * heads * seq; ++r) {
    const int64_t bh = r / seq, s = r % seq;
    const int64_t pos = is_decode ? cached_len + s : s;
    memcpy(k_cache + (bh * max_len + pos) * head_dim, k + r * head_dim, (size_t)head_dim * 2);
    memcpy(v_cache + (bh * max_len + pos) * head_dim, v + r * head_dim, (size_t)head_dim * 2);
  }
}

/* apply_attn_gate.cu:28-29: sigmoid first, then times a, one rounding. */
void ora_gated_attn_output(const uint16_t* gate, const uint16_t* attn, uint16_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float g = ora_bf16_to_f32(gate[i]), a = ora_bf16_to_f32(attn[i]);
    out[i] = ora_f32_to_bf16((1.0f / (1.0f + expf(-g))) * a);
  }
}

/* broadcast_vec.cu:102-105 */
void ora_broadcast_vec(uint16_t* dst, const uint16_t* src, int64_t n_copies, int64_t vec_len) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < n_copies; ++r) memcpy(dst + r * vec_len, src, (size_t)vec_len * 2);
}

/* half 2.7.1 bf16::from_f32: a NaN keeps sign and high bits and is made
 * quiet; otherwise round half to even on bit 15 (round bit) with the low 15
 * bits and bit 16 (the kept LSB) deciding ties. */
static uint16_t half_f32_to_bf16(uint32_t x) {
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x0040u);
  if ((x & 0x8000u) && (x & 0x17fffu)) return (uint16_t)((x >> 16) + 1u);
  return (uint16_t)(x >> 16);
}

/* half 2.7.1 f16::to_f32: exact; NaN payload shifted up with the quiet bit. */
static uint32_t half_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const int exp = (h >> 10) & 0x1f;
  const uint32_t man = h & 0x3ffu;
  if (exp == 0x1f) return sign | (man ? 0x7fc00000u | (man << 13) : 0x7f800000u);
  /* finite: the value is man * 2^(exp - 25) (+ implicit one), exact in fp32 */
  const float mag = exp == 0 ? ldexpf((float)man, -24) : ldexpf((float)(man | 0x400u), exp - 25);
  uint32_t bits;
  memcpy(&bits, &mag, 4);
  return sign | bits;
}

void ora_convert_to_bf16(const void* src, int dtype, uint16_t* dst, int64_t n) {
  const uint8_t* b = (const uint8_t*)src;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    if (dtype == 1) {
      const uint32_t x = (uint32_t)b[4 * i] | (uint32_t)b[4 * i + 1] << 8 | (uint32_t)b[4 * i + 2] << 16 |
                         (uint32_t)b[4 * i + 3] << 24;
      dst[i] = half_f32_to_bf16(x);
    } else {
      const uint16_t h = (uint16_t)(b[2 * i] | b[2 * i + 1] << 8);
      dst[i] = dtype == 2 ? half_f32_to_bf16(half_f16_to_f32(h)) : h;
    }
  }
}

/* ------------------------------------------------ counter-based inputs
 * The benchmark's synthetic inputs (the library's synth module restates the
 * same scheme for numpy and torch): every element is a function of (seed,
 * tensor tag, global index) alone, through the SplitMix64 finaliser:
 *   key    = mix(seed * 0x9E3779B97F4A7C15 + tag)
 *   bits_i = mix(key ^ mix(i))
 *   normal : u = ((bits >> 11) + 1) * 2^-53 from i = 2j and 2j + 1;
 *            z = sqrt(-2 ln u1) cos(2 pi u2) in double (Box-Muller);
 *            value = bf16_rne(f32_rne(mean + std * z))
 *   ids    : bits_i mod vocab */
static uint64_t sm64_mix(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static const double kPi = 3.14159265358979323846; /* the double nearest pi */

static double sm64_unit(uint64_t b) { return ((double)(b >> 11) + 1.0) * 0x1p-53; }

void ora_fill_normal_bf16(uint16_t* out, int64_t n, uint64_t seed, uint64_t tag, int64_t start, double std_,
                          double mean) {
  const uint64_t key = sm64_mix(seed * 0x9E3779B97F4A7C15ull + tag);
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < n; ++j) {
    const uint64_t i = 2 * (uint64_t)(start + j);
    const double u1 = sm64_unit(sm64_mix(key ^ sm64_mix(i)));
    const double u2 = sm64_unit(sm64_mix(key ^ sm64_mix(i + 1)));
    const double z = sqrt(-2.0 * log(u1)) * cos(2.0 * kPi * u2);
    out[j] = ora_f32_to_bf16((float)(mean + std_ * z));
  }
}

void ora_fill_ids(uint32_t* out, int64_t n, uint64_t seed, uint64_t tag, int64_t start, uint32_t vocab) {
  const uint64_t key = sm64_mix(seed * 0x9E3779B97F4A7C15ull + tag);
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < n; ++j) out[j] = (uint32_t)(sm64_mix(key ^ sm64_mix((uint64_t)(start + j))) % vocab);
}
