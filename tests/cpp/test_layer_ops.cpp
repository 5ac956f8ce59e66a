// Known-answer tests of the C++ host layer, restating the reference's GPU
// tests (src/lib.rs:2225-2279: test_additive_inject, test_rms_norm,
// test_swiglu_ffn) through HrmLayerOps, plus known answers for the two ops
// the reference never tested (embedding_lookup, rope_embed) and the fused
// entry points.  Needs a GPU, except with --host-only, which runs only the
// tests of host code; prints one line per test and exits non-zero on the
// first failure.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iterator>
#include <functional>
#include <string>
#include <vector>

#include "hrm_layer_ops.hpp"
#include "safetensors.hpp"

using hrm::bf16;
using hrm::CudaSlice;
using hrm::HrmError;
using hrm::HrmLayerOps;

namespace {

std::vector<bf16> to_bf16(const std::vector<float>& v) {
  std::vector<bf16> o;
  for (float x : v) o.push_back(bf16::from_f32(x));
  return o;
}

struct Failure {
  std::string what;
};

void expect(bool ok, const std::string& what) {
  if (!ok) throw Failure{what};
}

// Host-side f32 -> bf16 (half 2.7.1's bf16::from_f32): RNE, and a NaN keeps its
// sign and payload's high bits with the quiet bit set -- the same bits as the
// GPU loader conversion.
void test_bf16_from_f32() {
  const uint32_t in[] = {0x3f800000u, 0x3f808000u, 0x3f818000u, 0x3f808001u, 0x7f800000u, 0xff800000u,
                         0x7fc00000u, 0xffc00001u, 0x7f800001u, 0xff812345u, 0x00000001u, 0x7f7fffffu};
  const uint16_t want[] = {0x3f80, 0x3f80, 0x3f82, 0x3f81, 0x7f80, 0xff80,
                           0x7fc0, 0xffc0, 0x7fc0, 0xffc1, 0x0000, 0x7f80};
  for (int i = 0; i < 12; ++i) {
    float f;
    std::memcpy(&f, &in[i], 4);
    expect(bf16::from_f32(f).bits == want[i], "from_f32 case " + std::to_string(i));
  }
}

std::string g_golden = "tests/golden";  // --golden DIR

std::vector<uint8_t> file_bytes(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  expect((bool)f, "cannot open " + path);
  return std::vector<uint8_t>(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
}

// The fixture checkpoints (tests/golden/make_checkpoint.py): header parsed in
// data order, metadata read, the first tensor at the start of the data.
void test_safetensors_header() {
  const std::string path = g_golden + "/ckpt_tiny_attn.safetensors";
  const auto h = hrm::SafetensorsHeader::read(path);
  const auto bytes = file_bytes(path);
  expect(h.tensors.size() == 21, "21 tensors");
  expect(h.metadata.size() == 2 && h.metadata.at("format") == "pt", "metadata");
  expect(h.tensors[0].name == "model.extra.odd_bias" && h.tensors[0].dtype == hrm::StDtype::BF16 &&
             h.tensors[0].begin == 0 && h.tensors[0].end == 6,
         "first tensor");
  for (size_t i = 1; i < h.tensors.size(); ++i) expect(h.tensors[i].begin == h.tensors[i - 1].end, "data order");
  expect(h.data_offset() % 8 == 0 && h.data_offset() + h.data_len() == bytes.size(), "data section");
  const auto* g = h.find("model.L_module.layers.1.mlp.gate_up_proj.weight");
  expect(g && g->shape.size() == 2 && g->shape[0] == 96 && g->shape[1] == 32, "gate_up shape");
  // the same bytes through parse()
  const auto h2 = hrm::SafetensorsHeader::parse(bytes.data(), bytes.size(), bytes.size());
  expect(h2.tensors.size() == 21 && h2.header_len == h.header_len, "parse == read");
  const auto f = hrm::SafetensorsHeader::read(g_golden + "/ckpt_tiny_flat.safetensors");
  expect(f.tensors.size() == 19 && f.metadata.empty(), "flat file");
}

// exact f16 -> f32 widening (half's f16::to_f32), for the expected values
float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const int e = (h >> 10) & 0x1f;
  const uint32_t m = h & 0x3ffu;
  uint32_t bits;
  if (e == 0x1f) {
    bits = sign | (m ? 0x7fc00000u | (m << 13) : 0x7f800000u);
  } else {
    const float mag = e == 0 ? std::ldexp((float)m, -24) : std::ldexp((float)(m | 0x400u), e - 25);
    std::memcpy(&bits, &mag, 4);
    bits |= sign;
  }
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

// The expected bf16 bits of elements [first, first + n) of tensor t: the
// reference's raw_to_bf16 on the host (bf16 copied, f32 and f16 through
// half's from_f32).
std::vector<uint16_t> expected_bf16(const std::vector<uint8_t>& file, const hrm::SafetensorsHeader& h,
                                    const hrm::StTensor& t, uint64_t first, uint64_t n) {
  std::vector<uint16_t> out;
  const size_t es = hrm::st_dtype_size(t.dtype);
  const uint8_t* p = file.data() + h.data_offset() + t.begin + first * es;
  for (uint64_t i = 0; i < n; ++i, p += es) {
    if (t.dtype == hrm::StDtype::BF16) {
      out.push_back((uint16_t)(p[0] | p[1] << 8));
    } else if (t.dtype == hrm::StDtype::F16) {
      out.push_back(bf16::from_f32(f16_to_f32((uint16_t)(p[0] | p[1] << 8))).bits);
    } else {
      const uint32_t u = (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
      float f;
      std::memcpy(&f, &u, 4);
      out.push_back(bf16::from_f32(f).bits);
    }
  }
  return out;
}

// load_safetensors (src/lib.rs:2023-2125) on both fixture checkpoints, with
// chunks small enough that tensors straddle chunk ends: every slice equals
// the host conversion of its bytes, gate_up split at intermediate x hidden.
void test_load_safetensors(HrmLayerOps& hrm) {
  const hrm::HrmConfig saved = hrm.config;
  hrm.config.n_layers = 2;
  hrm.config.hidden_size = 32;
  hrm.config.intermediate_size = 48;
  for (const char* file : {"ckpt_tiny_attn.safetensors", "ckpt_tiny_flat.safetensors"}) {
    for (size_t chunk : {(size_t)4096, (size_t)(64u << 20)}) {
      const std::string path = g_golden + "/" + file;
      const auto bytes = file_bytes(path);
      const auto h = hrm::SafetensorsHeader::read(path);
      auto w = hrm.load_safetensors(path, chunk, 3);
      const bool attn = std::string(file).find("attn") != std::string::npos;
      auto check_slice = [&](CudaSlice<bf16>&& s, const std::string& name, uint64_t first, uint64_t n) {
        const hrm::StTensor* t = h.find(name);
        expect(t != nullptr, "fixture has " + name);
        expect(s.len() == n, name + ": length");
        const auto got = hrm.sync_reclaim(std::move(s));
        const auto want = expected_bf16(bytes, h, *t, first, n);
        for (uint64_t i = 0; i < n; ++i)
          expect(got[i].bits == want[i], name + ": element " + std::to_string(first + i));
      };
      const uint64_t split = 48 * 32;
      for (int mod = 0; mod < 2; ++mod) {
        auto& m = mod == 0 ? w.h_module : w.l_module;
        expect(m.layers.size() == 2, "two layers");
        for (size_t i = 0; i < 2; ++i) {
          const std::string p = std::string(mod == 0 ? "model.H_module.layers." : "model.L_module.layers.") +
                                std::to_string(i);
          const std::string a = attn ? ".attn" : "", mm = attn ? ".mlp" : "";
          check_slice(std::move(m.layers[i].gqkv_proj), p + a + ".gqkv_proj.weight", 0, 128 * 32);
          check_slice(std::move(m.layers[i].o_proj), p + a + ".o_proj.weight", 0, 32 * 32);
          check_slice(std::move(m.layers[i].gate_proj), p + mm + ".gate_up_proj.weight", 0, split);
          check_slice(std::move(m.layers[i].up_proj), p + mm + ".gate_up_proj.weight", split, 96 * 32 - split);
          check_slice(std::move(m.layers[i].down_proj), p + mm + ".down_proj.weight", 0, 32 * 48);
        }
      }
      check_slice(std::move(w.embed_tokens), "model.embed_tokens.weight", 0, 20 * 32);
      check_slice(std::move(w.lm_head), attn ? "lm_head.weight" : "model.lm_head.weight", 0, 20 * 32);
      check_slice(std::move(w.z_l_init), "model.z_L_init", 0, 32);
    }
  }
  // a missing tensor is InvalidInput, an unreadable file Io
  hrm.config.n_layers = 3;
  bool missing = false, io = false;
  try {
    hrm.load_safetensors(g_golden + "/ckpt_tiny_flat.safetensors");
  } catch (const HrmError& e) {
    missing = e.kind() == HrmError::Kind::InvalidInput &&
              std::string(e.what()).find("missing tensor: model.H_module.layers.2.gqkv_proj.weight") == 0;
  }
  try {
    hrm.load_safetensors(g_golden + "/no_such_file.safetensors");
  } catch (const HrmError& e) {
    io = e.kind() == HrmError::Kind::Io;
  }
  hrm.config = saved;
  expect(missing, "missing tensor reported");
  expect(io, "unreadable file reported");
}

// src/lib.rs:2227-2243
void test_additive_inject(HrmLayerOps& hrm) {
  auto a = hrm.htod_copy_bf16(to_bf16({1.0f, 2.0f, 3.0f, 4.0f}));
  auto b = hrm.htod_copy_bf16(to_bf16({0.5f, 1.5f, 2.5f, 3.5f}));
  auto out = hrm.alloc_zero_bf16(4);
  hrm.additive_inject(a, b, out, 4);
  auto host = hrm.sync_reclaim(std::move(out));
  const float expected[4] = {1.5f, 3.5f, 5.5f, 7.5f};
  for (int i = 0; i < 4; ++i) expect(std::fabs(host[i].to_f32() - expected[i]) < 0.01f, "additive_inject value");
}

// src/lib.rs:2247-2261
void test_rms_norm(HrmLayerOps& hrm) {
  auto inp = hrm.htod_copy_bf16(to_bf16({1.0f, 2.0f, 3.0f, 4.0f}));
  auto out = hrm.alloc_zero_bf16(4);
  hrm.rms_norm(inp, out, 1, 4);
  auto host = hrm.sync_reclaim(std::move(out));
  const float rms = std::sqrt(1.0f + 4.0f + 9.0f + 16.0f) / 2.0f;
  for (int i = 0; i < 4; ++i) expect(std::fabs(host[i].to_f32() - (i + 1) / rms) < 0.01f, "rms_norm value");
}

// src/lib.rs:2265-2279
void test_swiglu_ffn(HrmLayerOps& hrm) {
  auto g = hrm.htod_copy_bf16(to_bf16({0.0f, 0.0f, 0.0f, 0.0f}));
  auto u = hrm.htod_copy_bf16(to_bf16({2.0f, 2.0f, 2.0f, 2.0f}));
  auto out = hrm.alloc_zero_bf16(4);
  hrm.swiglu_ffn(g, u, out, 4);
  auto host = hrm.sync_reclaim(std::move(out));
  for (int i = 0; i < 4; ++i) expect(std::fabs(host[i].to_f32()) < 0.01f, "swiglu_ffn value");
}

// Embedding with scale 1 returns table rows exactly; an id >= vocab reads
// row vocab-1 (src/kernels/embedding_lookup.cu:35).
void test_embedding_lookup(HrmLayerOps& hrm) {
  const size_t vocab = 3, hidden = 8;
  std::vector<float> t(vocab * hidden);
  for (size_t i = 0; i < t.size(); ++i) t[i] = 0.25f * (float)i - 1.0f;
  auto table = hrm.htod_copy_bf16(to_bf16(t));
  auto ids = hrm.htod_copy_u32({2, 0, 7});
  auto out = hrm.alloc_zero_bf16(3 * hidden);
  hrm.embedding_lookup(ids, table, out, 1, 3, hidden, vocab, 1.0f);
  auto host = hrm.sync_reclaim(std::move(out));
  const size_t rows[3] = {2, 0, 2};
  for (size_t r = 0; r < 3; ++r)
    for (size_t j = 0; j < hidden; ++j)
      expect(host[r * hidden + j].to_f32() == t[rows[r] * hidden + j], "embedding_lookup row");
}

// RoPE at position 0 is the identity; at position 1 pair 0 rotates by 1 rad.
void test_rope_embed(HrmLayerOps& hrm) {
  const size_t hd = 128, n = 2 * hd;  // batch 1, heads 1, seq 2
  std::vector<float> v(n);
  for (size_t i = 0; i < n; ++i) v[i] = (float)((i % 7) + 1) * 0.125f;
  auto host_in = to_bf16(v);
  auto q = hrm.htod_copy_bf16(host_in);
  auto k = hrm.htod_copy_bf16(host_in);
  hrm.rope_embed(q, k, 1, 1, 2, hd, 0);
  auto qh = hrm.sync_reclaim(std::move(q));
  for (size_t i = 0; i < hd; ++i) expect(qh[i].bits == host_in[i].bits, "rope position 0 identity");
  const float x0 = host_in[hd].to_f32(), x1 = host_in[hd + hd / 2].to_f32();
  const float e0 = x0 * std::cos(1.0f) - x1 * std::sin(1.0f);
  expect(std::fabs(qh[hd].to_f32() - e0) < 0.01f, "rope position 1 pair 0");
}

// Fused add + norm equals additive_inject followed by rms_norm, bit for bit.
void test_add_rms_norm(HrmLayerOps& hrm) {
  const size_t rows = 3, hidden = 2048;
  std::vector<float> a(rows * hidden), b(rows * hidden);
  for (size_t i = 0; i < a.size(); ++i) {
    a[i] = std::sin(0.37f * (float)i);
    b[i] = std::cos(0.11f * (float)i) * 0.5f;
  }
  auto da = hrm.htod_copy_bf16(to_bf16(a));
  auto db = hrm.htod_copy_bf16(to_bf16(b));
  auto r1 = hrm.alloc_zero_bf16(a.size());
  auto y1 = hrm.alloc_zero_bf16(a.size());
  auto r2 = hrm.alloc_zero_bf16(a.size());
  auto y2 = hrm.alloc_zero_bf16(a.size());
  hrm.additive_inject(da, db, r1, a.size());
  hrm.rms_norm(r1, y1, rows, hidden);
  hrm.add_rms_norm(da, db, r2, y2, nullptr, rows, hidden);
  auto hr1 = hrm.sync_reclaim(std::move(r1)), hy1 = hrm.sync_reclaim(std::move(y1));
  auto hr2 = hrm.sync_reclaim(std::move(r2)), hy2 = hrm.sync_reclaim(std::move(y2));
  for (size_t i = 0; i < a.size(); ++i) {
    expect(hr1[i].bits == hr2[i].bits, "add_rms_norm residual");
    expect(hy1[i].bits == hy2[i].bits, "add_rms_norm normed");
  }
}

// split_gqkv_rope == rope_embed applied to the q / k segments of gqkv, and the
// cache rows at the offset hold the rotated k and the v.
void test_split_gqkv_rope(HrmLayerOps& hrm) {
  const size_t b = 1, s = 3, h = 2, d = 128, off = 5, cache_len = 9, n = b * s * h * d;
  std::vector<float> g(4 * n);
  for (size_t i = 0; i < g.size(); ++i) g[i] = std::sin(0.01f * (float)i);
  auto hg = to_bf16(g);
  auto dg = hrm.htod_copy_bf16(hg);
  auto gate = hrm.alloc_zero_bf16(n), q = hrm.alloc_zero_bf16(n), k = hrm.alloc_zero_bf16(n);
  auto v = hrm.alloc_zero_bf16(n);
  auto kc = hrm.alloc_zero_bf16(b * h * cache_len * d), vc = hrm.alloc_zero_bf16(b * h * cache_len * d);
  hrm.split_gqkv_rope(dg, gate, q, k, v, &kc, &vc, b, s, h, d, off, cache_len, off);
  // reference path: the q / k segments copied into [b, h, s, d] and rotated by rope_embed
  std::vector<bf16> hq(n), hk(n);
  for (size_t t = 0; t < s; ++t)
    for (size_t hh = 0; hh < h; ++hh)
      for (size_t i = 0; i < d; ++i) {
        hq[(hh * s + t) * d + i] = hg[t * 4 * h * d + (h + hh) * d + i];
        hk[(hh * s + t) * d + i] = hg[t * 4 * h * d + (2 * h + hh) * d + i];
      }
  auto rq = hrm.htod_copy_bf16(hq), rk = hrm.htod_copy_bf16(hk);
  hrm.rope_embed(rq, rk, b, h, s, d, off);
  auto q1 = hrm.sync_reclaim(std::move(q)), q2 = hrm.sync_reclaim(std::move(rq));
  auto k1 = hrm.sync_reclaim(std::move(k)), k2 = hrm.sync_reclaim(std::move(rk));
  auto v1 = hrm.sync_reclaim(std::move(v)), kc1 = hrm.sync_reclaim(std::move(kc)), vc1 = hrm.sync_reclaim(std::move(vc));
  for (size_t i = 0; i < n; ++i) {
    expect(q1[i].bits == q2[i].bits, "split_gqkv_rope q");
    expect(k1[i].bits == k2[i].bits, "split_gqkv_rope k");
  }
  for (size_t hh = 0; hh < h; ++hh)
    for (size_t t = 0; t < s; ++t)
      for (size_t i = 0; i < d; ++i) {
        expect(kc1[(hh * cache_len + off + t) * d + i].bits == k1[(hh * s + t) * d + i].bits, "k cache row");
        expect(vc1[(hh * cache_len + off + t) * d + i].bits == v1[(hh * s + t) * d + i].bits, "v cache row");
      }
}

// Argument errors come back as HrmError::InvalidInput, not as a launch.
void test_invalid_input(HrmLayerOps& hrm) {
  auto a = hrm.alloc_zero_bf16(4);
  auto out = hrm.alloc_zero_bf16(4);
  bool thrown = false;
  try {
    hrm.additive_inject(a, a, out, 8);  // slices hold 4 elements
  } catch (const HrmError& e) {
    thrown = e.kind() == HrmError::Kind::InvalidInput;
  }
  expect(thrown, "short slice rejected");
  thrown = false;
  try {
    hrm.rope_embed(a, out, 1, 1, 1, 3, 0);  // odd head_dim (slices hold 4 >= 3)
  } catch (const HrmError& e) {
    thrown = e.kind() == HrmError::Kind::InvalidInput && e.status() == HRM_ERR_INVALID_SHAPE;
  }
  expect(thrown, "odd head_dim rejected");
}

// gated_attn_output / apply_attn_gate with gate = 0 (sigmoid 0.5: exact halves)
// and broadcast_vec (src/lib.rs:505-527, 607-630, 748-767).
void test_gates_and_broadcast(HrmLayerOps& hrm) {
  const size_t n = 1003;  // a vector body and a scalar tail
  std::vector<float> a(n);
  for (size_t i = 0; i < n; ++i) a[i] = (float)((int)(i % 37) - 18) * 0.25f;
  auto gate = hrm.htod_copy_bf16(to_bf16(std::vector<float>(n, 0.0f)));
  auto attn = hrm.htod_copy_bf16(to_bf16(a));
  auto out = hrm.alloc_zero_bf16(n);
  hrm.gated_attn_output(gate, attn, out, n);
  auto got = hrm.sync_reclaim(std::move(out));
  for (size_t i = 0; i < n; ++i) expect(got[i].to_f32() == 0.5f * a[i], "gated_attn_output value");
  hrm.apply_attn_gate(gate, attn, n);
  auto inplace = hrm.sync_reclaim(std::move(attn));
  for (size_t i = 0; i < n; ++i) expect(inplace[i].to_f32() == 0.5f * a[i], "apply_attn_gate value");

  const size_t copies = 37, len = 2050;
  std::vector<float> v(len);
  for (size_t i = 0; i < len; ++i) v[i] = (float)i - 1000.0f;
  auto src = hrm.htod_copy_bf16(to_bf16(v));
  auto dst = hrm.alloc_zero_bf16(copies * len);
  hrm.broadcast_vec(dst, src, copies, len);
  auto rows = hrm.sync_reclaim(std::move(dst));
  const auto want = to_bf16(v);
  for (size_t r = 0; r < copies; ++r)
    for (size_t i = 0; i < len; ++i) expect(rows[r * len + i].bits == want[i].bits, "broadcast_vec row");
}

// raw_to_bf16 (src/lib.rs:1981-2008): f32 rounds to nearest even; a NaN keeps
// its sign and top payload bits and becomes quiet (half 2.7.1); f16 widens
// exactly first; bf16 is copied.
void test_raw_to_bf16(HrmLayerOps& hrm) {
  auto le = [](std::vector<uint8_t>& out, uint32_t v, int bytes) {
    for (int b = 0; b < bytes; ++b) out.push_back((uint8_t)(v >> (8 * b)));
  };
  std::vector<uint8_t> f32;
  const uint32_t in32[] = {0x3f800000u, 0xc0200000u, 0x3f808000u, 0x3f818000u, 0x7f800001u, 0xffa00000u, 0x00000001u};
  const uint16_t out32[] = {0x3f80, 0xc020, 0x3f80, 0x3f82, 0x7fc0, 0xffe0, 0x0000};
  for (uint32_t v : in32) le(f32, v, 4);
  auto got = hrm.raw_to_bf16(HRM_DTYPE_F32, f32);
  expect(got.size() == 7, "f32 count");
  for (int i = 0; i < 7; ++i) expect(got[i].bits == out32[i], "f32 -> bf16 bits " + std::to_string(i));

  std::vector<uint8_t> f16;
  const uint16_t in16[] = {0x3c00, 0xc000, 0x0001, 0x7c00, 0x7e01};
  const uint16_t out16[] = {0x3f80, 0xc000, 0x3380, 0x7f80, 0x7fc0};
  for (uint16_t v : in16) le(f16, v, 2);
  got = hrm.raw_to_bf16(HRM_DTYPE_F16, f16);
  for (int i = 0; i < 5; ++i) expect(got[i].bits == out16[i], "f16 -> bf16 bits " + std::to_string(i));

  std::vector<uint8_t> b16;
  for (uint16_t v : out32) le(b16, v, 2);
  got = hrm.raw_to_bf16(HRM_DTYPE_BF16, b16);
  for (int i = 0; i < 7; ++i) expect(got[i].bits == out32[i], "bf16 copy");

  bool thrown = false;
  try {
    hrm.raw_to_bf16(HRM_DTYPE_F32, std::vector<uint8_t>(6));
  } catch (const HrmError& e) {
    thrown = e.kind() == HrmError::Kind::InvalidInput;
  }
  expect(thrown, "partial element rejected");
}

// An error the caller left pending (a failed allocation) is neither reported
// as a layer-op failure nor cleared: each launch returns its own status.
void test_pending_error_not_claimed(HrmLayerOps& hrm) {
  auto a = hrm.htod_copy_bf16(to_bf16({1.0f, 2.0f, 3.0f, 4.0f}));
  auto out = hrm.alloc_zero_bf16(4);
  void* huge = nullptr;
  expect(cudaMalloc(&huge, (size_t)1 << 62) != cudaSuccess, "the oversized allocation fails");
  hrm.additive_inject(a, a, out, 4);  // must not throw
  expect(cudaGetLastError() == cudaErrorMemoryAllocation, "the caller's error is still pending");
  auto host = hrm.sync_reclaim(std::move(out));
  expect(host[3].to_f32() == 8.0f, "additive_inject value");
}

// transformer_module (the fused schedule) == the reference's order of wrapper
// calls and device copies (src/lib.rs:955-1030 per layer, 1036-1105 per module,
// 1215-1256 per cycle), bit for bit, over 2 H-cycles x 2 L-cycles of 3-layer
// modules.  Stand-ins for attention and the FFN GEMMs are exact device copies:
// a = n; gate = up = [n | n]; down = act[:, :hidden].
void test_transformer_module(HrmLayerOps&) {
  hrm::HrmConfig cfg;
  cfg.hidden_size = 256;
  cfg.intermediate_size = 512;
  cfg.norm_eps = 1e-5f;
  HrmLayerOps m(0, cfg);
  const size_t rows = 64, H = 256, I = 512, L = 3, n = rows * H;
  cudaStream_t st = m.cu_stream();
  auto copy2d = [&](bf16* dst, size_t dpitch, const bf16* src, size_t spitch, size_t width) {
    expect(cudaMemcpy2DAsync(dst, dpitch * sizeof(bf16), src, spitch * sizeof(bf16), width * sizeof(bf16), rows,
                             cudaMemcpyDeviceToDevice, st) == cudaSuccess,
           "cudaMemcpy2DAsync");
  };
  auto copy = [&](CudaSlice<bf16>& dst, const CudaSlice<bf16>& src) {
    expect(cudaMemcpyAsync(dst.device_ptr(), src.device_ptr(), n * sizeof(bf16), cudaMemcpyDeviceToDevice, st) ==
               cudaSuccess,
           "cudaMemcpyAsync");
  };
  HrmLayerOps::LayerCallbacks cb;
  cb.attention = [&](size_t, const CudaSlice<bf16>& nn, CudaSlice<bf16>& a) {
    copy2d(a.device_ptr(), H, nn.device_ptr(), H, H);
  };
  cb.gate_up = [&](size_t, const CudaSlice<bf16>& nn, CudaSlice<bf16>& g, CudaSlice<bf16>& u) {
    for (CudaSlice<bf16>* t : {&g, &u}) {
      copy2d(t->device_ptr(), I, nn.device_ptr(), H, H);
      copy2d(t->device_ptr() + H, I, nn.device_ptr(), H, H);
    }
  };
  cb.down = [&](size_t, const CudaSlice<bf16>& act, CudaSlice<bf16>& d) {
    copy2d(d.device_ptr(), H, act.device_ptr(), I, H);
  };

  // The reference's buffers and order.
  auto tmp1 = m.alloc_zero_bf16(n), tmp2 = m.alloc_zero_bf16(n), norm_buf = m.alloc_zero_bf16(n);
  auto attn_out = m.alloc_zero_bf16(n), norm2 = m.alloc_zero_bf16(n), down = m.alloc_zero_bf16(n);
  auto res = m.alloc_zero_bf16(n), g = m.alloc_zero_bf16(rows * I), u = m.alloc_zero_bf16(rows * I);
  auto act = m.alloc_zero_bf16(rows * I);
  auto reference_module = [&](CudaSlice<bf16>& out, const CudaSlice<bf16>& z_b) {  // out = module(out + z_b)
    m.additive_inject(out, z_b, tmp1, n);
    copy(tmp2, tmp1);
    for (size_t i = 0; i < L; ++i) {
      CudaSlice<bf16>* x = &tmp2;
      if (i > 0) {
        copy(tmp1, out);
        x = &tmp1;
      }
      m.rms_norm(*x, norm_buf, rows, H);
      cb.attention(i, norm_buf, attn_out);
      m.additive_inject(*x, attn_out, out, n);
      m.rms_norm(out, norm2, rows, H);
      cb.gate_up(i, norm2, g, u);
      m.swiglu_ffn(g, u, act, rows * I);
      cb.down(i, act, down);
      m.additive_inject(out, down, res, n);
      copy(out, res);
    }
    m.rms_norm(out, tmp1, rows, H);
    copy(out, tmp1);
  };

  std::vector<bf16> h0(n), l0(n);
  uint32_t state = 12345u;
  for (size_t i = 0; i < n; ++i) {
    state = state * 1664525u + 1013904223u;
    h0[i] = bf16::from_f32(((state >> 8) * (1.0f / 16777216.0f)) * 4.0f - 2.0f);
    state = state * 1664525u + 1013904223u;
    l0[i] = bf16::from_f32(((state >> 8) * (1.0f / 16777216.0f)) * 4.0f - 2.0f);
  }
  auto rh = m.htod_copy_bf16(h0), rl = m.htod_copy_bf16(l0);
  auto fh = m.htod_copy_bf16(h0), fl = m.htod_copy_bf16(l0);
  HrmLayerOps::ModuleScratch scratch(m, rows);
  for (int hc = 0; hc < 2; ++hc) {
    for (int lc = 0; lc < 2; ++lc) {
      reference_module(rl, rh);
      m.transformer_module(fl, fh, fl, L, cb, scratch);
    }
    reference_module(rh, rl);
    m.transformer_module(fh, fl, fh, L, cb, scratch);
  }
  const auto want_h = m.sync_reclaim(std::move(rh)), want_l = m.sync_reclaim(std::move(rl));
  const auto got_h = m.sync_reclaim(std::move(fh)), got_l = m.sync_reclaim(std::move(fl));
  size_t bad = 0;
  for (size_t i = 0; i < n; ++i) bad += (got_h[i].bits != want_h[i].bits) + (got_l[i].bits != want_l[i].bits);
  expect(bad == 0, std::to_string(bad) + " elements of z_H / z_L differ from the reference order");
  bool finite = true;
  for (size_t i = 0; i < n; ++i) finite = finite && std::isfinite(got_h[i].to_f32());
  expect(finite, "z_H finite");

  bool thrown = false;
  try {
    m.transformer_module(scratch.n, scratch.x, scratch.x, L, cb, scratch);
  } catch (const HrmError& e) {
    thrown = e.kind() == HrmError::Kind::InvalidInput && e.status() == HRM_ERR_ALIASING;
  }
  expect(thrown, "output aliasing z_b rejected");
}

// recurrent_forward == the reference's loop (src/lib.rs:1189-1270) built from
// the unfused wrappers and device copies: embedding, broadcast, then 2 H-cycles
// x 3 L-cycles of 2-layer modules; the attention sees the reference's KV slots.
void test_recurrent_forward(HrmLayerOps&) {
  hrm::HrmConfig cfg;
  cfg.hidden_size = 256;
  cfg.intermediate_size = 512;
  cfg.norm_eps = 1e-5f;
  cfg.embedding_scale = 16.0f;
  HrmLayerOps m(0, cfg);
  const size_t rows = 40, H = 256, I = 512, L = 2, V = 50, n = rows * H;
  cudaStream_t st = m.cu_stream();
  auto copy2d = [&](bf16* dst, size_t dpitch, const bf16* src, size_t spitch, size_t width) {
    expect(cudaMemcpy2DAsync(dst, dpitch * sizeof(bf16), src, spitch * sizeof(bf16), width * sizeof(bf16), rows,
                             cudaMemcpyDeviceToDevice, st) == cudaSuccess,
           "cudaMemcpy2DAsync");
  };
  auto copy = [&](CudaSlice<bf16>& dst, const CudaSlice<bf16>& src) {
    expect(cudaMemcpyAsync(dst.device_ptr(), src.device_ptr(), n * sizeof(bf16), cudaMemcpyDeviceToDevice, st) ==
               cudaSuccess,
           "cudaMemcpyAsync");
  };
  std::vector<size_t> slots;
  HrmLayerOps::ModuleCallbacks mod;
  mod.n_layers = L;
  mod.attention = [&](size_t, size_t slot, const CudaSlice<bf16>& nn, CudaSlice<bf16>& a) {
    slots.push_back(slot);
    copy2d(a.device_ptr(), H, nn.device_ptr(), H, H);
  };
  mod.gate_up = [&](size_t, const CudaSlice<bf16>& nn, CudaSlice<bf16>& g, CudaSlice<bf16>& u) {
    for (CudaSlice<bf16>* t : {&g, &u}) {
      copy2d(t->device_ptr(), I, nn.device_ptr(), H, H);
      copy2d(t->device_ptr() + H, I, nn.device_ptr(), H, H);
    }
  };
  mod.down = [&](size_t, const CudaSlice<bf16>& act, CudaSlice<bf16>& d) {
    copy2d(d.device_ptr(), H, act.device_ptr(), I, H);
  };

  std::vector<uint32_t> ids(rows);
  std::vector<float> table(V * H), init(H);
  uint32_t state = 777u;
  auto next = [&]() {
    state = state * 1664525u + 1013904223u;
    return ((state >> 8) * (1.0f / 16777216.0f)) * 2.0f - 1.0f;
  };
  for (size_t i = 0; i < rows; ++i) ids[i] = (uint32_t)((i * 7919u) % (V + 3));  // a few out of range
  for (float& t : table) t = next() * 0.1f;
  for (float& t : init) t = next();
  auto d_ids = m.htod_copy_u32(ids);
  auto d_table = m.htod_copy_bf16(to_bf16(table));
  auto d_init = m.htod_copy_bf16(to_bf16(init));

  // the fused loop
  auto fh = m.alloc_zero_bf16(n), fl = m.alloc_zero_bf16(n);
  HrmLayerOps::ModuleScratch scratch(m, rows);
  m.recurrent_forward(d_ids, d_table, V, d_init, 2, 3, mod, mod, scratch, fh, fl);
  const std::vector<size_t> fused_slots = slots;
  slots.clear();

  // the reference's order
  auto rh = m.alloc_zero_bf16(n), rl = m.alloc_zero_bf16(n);
  m.embedding_lookup(d_ids, d_table, rh, 1, rows, H, V, cfg.embedding_scale);
  m.broadcast_vec(rl, d_init, rows, H);
  auto tmp1 = m.alloc_zero_bf16(n), tmp2 = m.alloc_zero_bf16(n), norm_buf = m.alloc_zero_bf16(n);
  auto attn_out = m.alloc_zero_bf16(n), norm2 = m.alloc_zero_bf16(n), down = m.alloc_zero_bf16(n);
  auto res = m.alloc_zero_bf16(n), g = m.alloc_zero_bf16(rows * I), u = m.alloc_zero_bf16(rows * I);
  auto act = m.alloc_zero_bf16(rows * I);
  size_t slot = 0;
  auto reference_module = [&](CudaSlice<bf16>& out, const CudaSlice<bf16>& z_b) {
    m.additive_inject(out, z_b, tmp1, n);
    copy(tmp2, tmp1);
    for (size_t i = 0; i < L; ++i) {
      CudaSlice<bf16>* x = &tmp2;
      if (i > 0) {
        copy(tmp1, out);
        x = &tmp1;
      }
      m.rms_norm(*x, norm_buf, rows, H);
      mod.attention(i, slot + i, norm_buf, attn_out);
      m.additive_inject(*x, attn_out, out, n);
      m.rms_norm(out, norm2, rows, H);
      mod.gate_up(i, norm2, g, u);
      m.swiglu_ffn(g, u, act, rows * I);
      mod.down(i, act, down);
      m.additive_inject(out, down, res, n);
      copy(out, res);
    }
    m.rms_norm(out, tmp1, rows, H);
    copy(out, tmp1);
    slot += L;
  };
  for (int h = 0; h < 2; ++h) {
    for (int l = 0; l < 3; ++l) reference_module(rl, rh);
    reference_module(rh, rl);
  }
  expect(fused_slots == slots, "KV slot numbering");
  expect(fused_slots.size() == 2 * 4 * L && fused_slots.back() == 2 * 4 * L - 1, "slots 0 .. 15 in order");
  const auto want_h = m.sync_reclaim(std::move(rh)), want_l = m.sync_reclaim(std::move(rl));
  const auto got_h = m.sync_reclaim(std::move(fh)), got_l = m.sync_reclaim(std::move(fl));
  size_t bad = 0;
  for (size_t i = 0; i < n; ++i) bad += (got_h[i].bits != want_h[i].bits) + (got_l[i].bits != want_l[i].bits);
  expect(bad == 0, std::to_string(bad) + " elements of z_H / z_L differ from the reference's loop");
}

}  // namespace

// --parse FILE: prints "ok <tensors> <data offset>" or "error <kind>" for the
// header of FILE (the CPU tests compare it with the Python parser).
int parse_only(const char* path) {
  static const char* kinds[] = {"HeaderTooSmall",   "HeaderTooLarge",    "InvalidHeaderLength",
                                "InvalidHeader",    "InvalidHeaderStart", "InvalidHeaderDeserialization",
                                "InvalidOffset",    "TensorInvalidInfo", "ValidationOverflow",
                                "MetadataIncompleteBuffer", "Io"};
  try {
    const auto h = hrm::SafetensorsHeader::read(path);
    std::printf("ok %zu %llu\n", h.tensors.size(), (unsigned long long)h.data_offset());
  } catch (const hrm::SafetensorsError& e) {
    std::printf("error %s\n", kinds[(int)e.kind()]);
  }
  return 0;
}

int main(int argc, char** argv) {
  bool host_only = false;
  for (int i = 1; i < argc; ++i) {
    if (std::strcmp(argv[i], "--host-only") == 0) host_only = true;
    else if (std::strcmp(argv[i], "--golden") == 0 && i + 1 < argc) g_golden = argv[++i];
    else if (std::strcmp(argv[i], "--parse") == 0 && i + 1 < argc) return parse_only(argv[++i]);
  }
  const std::vector<std::pair<const char*, std::function<void()>>> host_tests = {
      {"test_bf16_from_f32", test_bf16_from_f32},
      {"test_safetensors_header", test_safetensors_header},
  };
  for (const auto& t : host_tests) {
    try {
      t.second();
    } catch (const Failure& f) {
      std::printf("FAIL %s: %s\n", t.first, f.what.c_str());
      return 1;
    } catch (const std::exception& e) {
      std::printf("FAIL %s: %s\n", t.first, e.what());
      return 1;
    }
    std::printf("ok   %s\n", t.first);
  }
  if (host_only) {
    std::printf("all %zu host tests passed\n", host_tests.size());
    return 0;
  }
  const std::vector<std::pair<const char*, std::function<void(HrmLayerOps&)>>> tests = {
      {"test_additive_inject", test_additive_inject}, {"test_rms_norm", test_rms_norm},
      {"test_swiglu_ffn", test_swiglu_ffn},           {"test_embedding_lookup", test_embedding_lookup},
      {"test_rope_embed", test_rope_embed},           {"test_add_rms_norm", test_add_rms_norm},
      {"test_split_gqkv_rope", test_split_gqkv_rope},
      {"test_invalid_input", test_invalid_input},
      {"test_gates_and_broadcast", test_gates_and_broadcast},
      {"test_pending_error_not_claimed", test_pending_error_not_claimed},
      {"test_raw_to_bf16", test_raw_to_bf16},
      {"test_transformer_module", test_transformer_module},
      {"test_recurrent_forward", test_recurrent_forward},
      {"test_load_safetensors", test_load_safetensors},
  };
  try {
    HrmLayerOps hrm(0);
    for (const auto& t : tests) {
      try {
        t.second(hrm);
      } catch (const Failure& f) {
        std::printf("FAIL %s: %s\n", t.first, f.what.c_str());
        return 1;
      }
      std::printf("ok   %s\n", t.first);
    }
  } catch (const HrmError& e) {
    std::printf("FAIL HrmError: %s\n", e.what());
    return 1;
  }
  std::printf("all %zu tests passed\n", tests.size());
  return 0;
}
