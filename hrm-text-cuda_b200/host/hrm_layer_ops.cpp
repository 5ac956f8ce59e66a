// Implementation of the C++ host layer (see hrm_layer_ops.hpp).
#include "hrm_layer_ops.hpp"

#include <cstring>
#include <string>

namespace hrm {

namespace {

[[noreturn]] void fail(HrmError::Kind kind, int status, const std::string& what) { throw HrmError(kind, status, what); }

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    fail(HrmError::Kind::Driver, HRM_ERR_CUDA + (int)e, std::string(what) + ": " + cudaGetErrorString(e));
}

template <class T>
void need(const CudaSlice<T>& s, size_t elems, const char* op, const char* name) {
  if (s.len() < elems)
    fail(HrmError::Kind::InvalidInput, HRM_ERR_INVALID_SHAPE,
         std::string(op) + ": " + name + " holds " + std::to_string(s.len()) + " elements, " +
             std::to_string(elems) + " required");
}

}  // namespace

// half 2.7.1's bf16::from_f32, the conversion the reference's host code uses:
// round to nearest even; a NaN keeps its sign and high payload bits and is
// made quiet (0x0040), as the GPU loader conversion (hrm_convert_to_bf16) does.
bf16 bf16::from_f32(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  bf16 r;
  if ((u & 0x7fffffffu) > 0x7f800000u) {
    r.bits = (uint16_t)((u >> 16) | 0x0040u);
  } else {
    u += 0x7fffu + ((u >> 16) & 1u);
    r.bits = (uint16_t)(u >> 16);
  }
  return r;
}

float bf16::to_f32() const {
  const uint32_t u = (uint32_t)bits << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

HrmLayerOps::HrmLayerOps(int dev_ordinal, HrmConfig cfg) : config(cfg), dev_(dev_ordinal) {
  if (hrm_abi_version() / 10000 != 1)
    fail(HrmError::Kind::KernelNotFound, 0, "libhrm_ops ABI major version mismatch");
  cuda_check(cudaSetDevice(dev_ordinal), "cudaSetDevice");
  cuda_check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
}

HrmLayerOps::~HrmLayerOps() {
  if (stream_) cudaStreamDestroy(stream_);
}

void HrmLayerOps::check(int status, const char* op) const {
  if (status == HRM_OK) return;
  const HrmError::Kind kind = status >= HRM_ERR_CUDA ? HrmError::Kind::Driver : HrmError::Kind::InvalidInput;
  fail(kind, status, std::string(op) + ": " + hrm_status_string(status));
}

CudaSlice<bf16> HrmLayerOps::alloc_zero_bf16(size_t len) const {
  void* p = nullptr;
  cuda_check(cudaMalloc(&p, len * sizeof(bf16) + (len == 0)), "cudaMalloc");
  CudaSlice<bf16> s(static_cast<bf16*>(p), len);
  cuda_check(cudaMemsetAsync(p, 0, len * sizeof(bf16), stream_), "cudaMemsetAsync");
  return s;
}

CudaSlice<bf16> HrmLayerOps::htod_copy_bf16(const std::vector<bf16>& host) const {
  CudaSlice<bf16> s = alloc_zero_bf16(host.size());
  cuda_check(cudaMemcpyAsync(s.device_ptr(), host.data(), host.size() * sizeof(bf16), cudaMemcpyHostToDevice, stream_),
             "cudaMemcpyAsync");
  cuda_check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");  // host vector may die after return
  return s;
}

CudaSlice<uint32_t> HrmLayerOps::htod_copy_u32(const std::vector<uint32_t>& host) const {
  void* p = nullptr;
  cuda_check(cudaMalloc(&p, host.size() * sizeof(uint32_t) + host.empty()), "cudaMalloc");
  CudaSlice<uint32_t> s(static_cast<uint32_t*>(p), host.size());
  cuda_check(cudaMemcpyAsync(p, host.data(), host.size() * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_),
             "cudaMemcpyAsync");
  cuda_check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
  return s;
}

std::vector<bf16> HrmLayerOps::sync_reclaim(CudaSlice<bf16>&& slice) const {
  std::vector<bf16> host(slice.len());
  cuda_check(cudaMemcpyAsync(host.data(), slice.device_ptr(), slice.len() * sizeof(bf16), cudaMemcpyDeviceToHost,
                             stream_),
             "cudaMemcpyAsync");
  cuda_check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
  CudaSlice<bf16> drop(std::move(slice));
  return host;
}

void HrmLayerOps::additive_inject(const CudaSlice<bf16>& z_a, const CudaSlice<bf16>& z_b, CudaSlice<bf16>& z_out,
                                  size_t total_elements) const {
  need(z_a, total_elements, "additive_inject", "z_a");
  need(z_b, total_elements, "additive_inject", "z_b");
  need(z_out, total_elements, "additive_inject", "z_out");
  check(hrm_additive_inject(z_a.device_ptr(), z_b.device_ptr(), z_out.device_ptr(), (int64_t)total_elements,
                            stream_),
        "additive_inject");
}

void HrmLayerOps::rms_norm(const CudaSlice<bf16>& input, CudaSlice<bf16>& output, size_t rows,
                           size_t hidden_size) const {
  need(input, rows * hidden_size, "rms_norm", "input");
  need(output, rows * hidden_size, "rms_norm", "output");
  check(hrm_rms_norm(input.device_ptr(), output.device_ptr(), nullptr, (int64_t)rows, (int64_t)hidden_size,
                     config.norm_eps, stream_),
        "rms_norm");
}

void HrmLayerOps::rope_embed(CudaSlice<bf16>& q, CudaSlice<bf16>& k, size_t batch_size, size_t num_heads,
                             size_t seq_len, size_t head_dim, size_t position_offset) const {
  const size_t n = batch_size * num_heads * seq_len * head_dim;
  need(q, n, "rope_embed", "q");
  need(k, n, "rope_embed", "k");
  const bool use_table = rope_table_.device_ptr() != nullptr && head_dim == config.head_dim &&
                         position_offset + seq_len <= rope_positions_;
  check(hrm_rope_embed(q.device_ptr(), k.device_ptr(), (int64_t)batch_size, (int64_t)num_heads, (int64_t)seq_len,
                       (int64_t)head_dim, (int64_t)position_offset, config.rope_theta,
                       use_table ? rope_table_.device_ptr() : nullptr, use_table ? (int64_t)rope_positions_ : 0,
                       stream_),
        "rope_embed");
}

void HrmLayerOps::swiglu_ffn(const CudaSlice<bf16>& gate, const CudaSlice<bf16>& up, CudaSlice<bf16>& output,
                             size_t total_elements) const {
  need(gate, total_elements, "swiglu_ffn", "gate");
  need(up, total_elements, "swiglu_ffn", "up");
  need(output, total_elements, "swiglu_ffn", "output");
  check(hrm_swiglu_ffn(gate.device_ptr(), up.device_ptr(), output.device_ptr(), (int64_t)total_elements, stream_),
        "swiglu_ffn");
}

void HrmLayerOps::embedding_lookup(const CudaSlice<uint32_t>& input_ids, const CudaSlice<bf16>& embedding_table,
                                   CudaSlice<bf16>& output, size_t batch_size, size_t seq_len, size_t hidden_size,
                                   size_t vocab_size, float embedding_scale) const {
  need(input_ids, batch_size * seq_len, "embedding_lookup", "input_ids");
  need(embedding_table, vocab_size * hidden_size, "embedding_lookup", "embedding_table");
  need(output, batch_size * seq_len * hidden_size, "embedding_lookup", "output");
  check(hrm_embedding_lookup(input_ids.device_ptr(), embedding_table.device_ptr(), output.device_ptr(),
                             (int64_t)batch_size, (int64_t)seq_len, (int64_t)hidden_size, (int64_t)vocab_size,
                             embedding_scale, stream_),
        "embedding_lookup");
}

void HrmLayerOps::add_rms_norm(const CudaSlice<bf16>& x, const CudaSlice<bf16>& branch, CudaSlice<bf16>& residual_out,
                               CudaSlice<bf16>& normed_out, const CudaSlice<bf16>* weight, size_t rows,
                               size_t hidden_size) const {
  const size_t n = rows * hidden_size;
  need(x, n, "add_rms_norm", "x");
  need(branch, n, "add_rms_norm", "branch");
  need(residual_out, n, "add_rms_norm", "residual_out");
  need(normed_out, n, "add_rms_norm", "normed_out");
  if (weight) need(*weight, hidden_size, "add_rms_norm", "weight");
  check(hrm_add_rms_norm(x.device_ptr(), branch.device_ptr(), residual_out.device_ptr(), normed_out.device_ptr(),
                         weight ? weight->device_ptr() : nullptr, (int64_t)rows, (int64_t)hidden_size,
                         config.norm_eps, stream_),
        "add_rms_norm");
}

void HrmLayerOps::embed_rms_norm(const CudaSlice<uint32_t>& input_ids, const CudaSlice<bf16>& embedding_table,
                                 CudaSlice<bf16>* hidden_out, CudaSlice<bf16>& normed_out,
                                 const CudaSlice<bf16>* weight, size_t rows, size_t hidden_size, size_t vocab_size,
                                 float embedding_scale) const {
  need(input_ids, rows, "embed_rms_norm", "input_ids");
  need(embedding_table, vocab_size * hidden_size, "embed_rms_norm", "embedding_table");
  need(normed_out, rows * hidden_size, "embed_rms_norm", "normed_out");
  if (hidden_out) need(*hidden_out, rows * hidden_size, "embed_rms_norm", "hidden_out");
  if (weight) need(*weight, hidden_size, "embed_rms_norm", "weight");
  check(hrm_embed_rms_norm(input_ids.device_ptr(), embedding_table.device_ptr(),
                           hidden_out ? hidden_out->device_ptr() : nullptr, normed_out.device_ptr(),
                           weight ? weight->device_ptr() : nullptr, (int64_t)rows, (int64_t)hidden_size,
                           (int64_t)vocab_size, embedding_scale, config.norm_eps, stream_),
        "embed_rms_norm");
}

void HrmLayerOps::split_gqkv_rope(const CudaSlice<bf16>& gqkv, CudaSlice<bf16>& gate, CudaSlice<bf16>& q,
                                  CudaSlice<bf16>& k, CudaSlice<bf16>& v, CudaSlice<bf16>* k_cache,
                                  CudaSlice<bf16>* v_cache, size_t batch_size, size_t seq_len, size_t num_heads,
                                  size_t head_dim, size_t position_offset, size_t cache_len,
                                  size_t cache_offset) const {
  const size_t n = batch_size * seq_len * num_heads * head_dim;
  need(gqkv, 4 * n, "split_gqkv_rope", "gqkv");
  need(gate, n, "split_gqkv_rope", "gate");
  need(q, n, "split_gqkv_rope", "q");
  need(k, n, "split_gqkv_rope", "k");
  need(v, n, "split_gqkv_rope", "v");
  if ((k_cache == nullptr) != (v_cache == nullptr))
    fail(HrmError::Kind::InvalidInput, HRM_ERR_NULL_POINTER, "split_gqkv_rope: pass both caches or neither");
  if (k_cache) {
    need(*k_cache, batch_size * num_heads * cache_len * head_dim, "split_gqkv_rope", "k_cache");
    need(*v_cache, batch_size * num_heads * cache_len * head_dim, "split_gqkv_rope", "v_cache");
  }
  const bool use_table = rope_table_.device_ptr() != nullptr && head_dim == config.head_dim &&
                         position_offset + seq_len <= rope_positions_;
  check(hrm_split_gqkv_rope(gqkv.device_ptr(), gate.device_ptr(), q.device_ptr(), k.device_ptr(), v.device_ptr(),
                            k_cache ? k_cache->device_ptr() : nullptr, v_cache ? v_cache->device_ptr() : nullptr,
                            (int64_t)batch_size, (int64_t)seq_len, (int64_t)num_heads, (int64_t)head_dim,
                            (int64_t)position_offset, config.rope_theta,
                            use_table ? rope_table_.device_ptr() : nullptr, use_table ? (int64_t)rope_positions_ : 0,
                            (int64_t)cache_len, (int64_t)cache_offset, stream_),
        "split_gqkv_rope");
}

void HrmLayerOps::build_rope_table(size_t max_positions) {
  void* p = nullptr;
  const size_t n = max_positions * config.head_dim;
  cuda_check(cudaMalloc(&p, n * sizeof(float) + (n == 0)), "cudaMalloc");
  CudaSlice<float> table(static_cast<float*>(p), n);
  check(hrm_rope_table_build(table.device_ptr(), (int64_t)max_positions, (int64_t)config.head_dim,
                             config.rope_theta, stream_),
        "rope_table_build");
  rope_table_ = std::move(table);
  rope_positions_ = max_positions;
}

void HrmLayerOps::gated_attn_output(const CudaSlice<bf16>& gate, const CudaSlice<bf16>& attn_out,
                                    CudaSlice<bf16>& output, size_t total_elements) const {
  need(gate, total_elements, "gated_attn_output", "gate");
  need(attn_out, total_elements, "gated_attn_output", "attn_out");
  need(output, total_elements, "gated_attn_output", "output");
  check(hrm_gated_attn_output(gate.device_ptr(), attn_out.device_ptr(), output.device_ptr(), (int64_t)total_elements,
                              stream_),
        "gated_attn_output");
}

void HrmLayerOps::apply_attn_gate(const CudaSlice<bf16>& gate, CudaSlice<bf16>& attn_out,
                                  size_t total_elements) const {
  need(gate, total_elements, "apply_attn_gate", "gate");
  need(attn_out, total_elements, "apply_attn_gate", "attn_out");
  check(hrm_apply_attn_gate(gate.device_ptr(), attn_out.device_ptr(), (int64_t)total_elements, stream_),
        "apply_attn_gate");
}

void HrmLayerOps::broadcast_vec(CudaSlice<bf16>& dst, const CudaSlice<bf16>& src, size_t n_copies,
                                size_t vec_len) const {
  need(src, vec_len, "broadcast_vec", "src");
  need(dst, n_copies * vec_len, "broadcast_vec", "dst");
  check(hrm_broadcast_vec(dst.device_ptr(), src.device_ptr(), (int64_t)n_copies, (int64_t)vec_len, stream_),
        "broadcast_vec");
}

CudaSlice<bf16> HrmLayerOps::htod_raw_as_bf16(int dtype, const uint8_t* raw, size_t nbytes) const {
  const size_t size = dtype == HRM_DTYPE_F32 ? 4 : 2;
  if (dtype != HRM_DTYPE_BF16 && dtype != HRM_DTYPE_F32 && dtype != HRM_DTYPE_F16)
    fail(HrmError::Kind::InvalidInput, HRM_ERR_DTYPE, "raw_to_bf16: unsupported dtype");
  if (nbytes % size)
    fail(HrmError::Kind::InvalidInput, HRM_ERR_INVALID_SHAPE,
         "raw_to_bf16: " + std::to_string(nbytes) + " bytes is not a whole number of elements");
  const size_t n = nbytes / size;
  void* d_raw = nullptr;
  cuda_check(cudaMalloc(&d_raw, nbytes + (nbytes == 0)), "cudaMalloc");
  struct Free {
    void* p;
    ~Free() { cudaFree(p); }
  } free_raw{d_raw};
  cuda_check(cudaMemcpyAsync(d_raw, raw, nbytes, cudaMemcpyHostToDevice, stream_), "cudaMemcpyAsync");
  CudaSlice<bf16> out = alloc_zero_bf16(n);
  check(hrm_convert_to_bf16(d_raw, dtype, out.device_ptr(), (int64_t)n, stream_), "raw_to_bf16");
  cuda_check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");  // before d_raw is freed
  return out;
}

std::vector<bf16> HrmLayerOps::raw_to_bf16(int dtype, const std::vector<uint8_t>& raw) const {
  return sync_reclaim(htod_raw_as_bf16(dtype, raw.data(), raw.size()));
}

HrmLayerOps::ModuleScratch::ModuleScratch(const HrmLayerOps& ops, size_t rows_)
    : rows(rows_),
      x(ops.alloc_zero_bf16(rows_ * ops.config.hidden_size)),
      n(ops.alloc_zero_bf16(rows_ * ops.config.hidden_size)),
      n2(ops.alloc_zero_bf16(rows_ * ops.config.hidden_size)),
      a(ops.alloc_zero_bf16(rows_ * ops.config.hidden_size)),
      d(ops.alloc_zero_bf16(rows_ * ops.config.hidden_size)),
      g(ops.alloc_zero_bf16(rows_ * ops.config.intermediate_size)),
      u(ops.alloc_zero_bf16(rows_ * ops.config.intermediate_size)),
      act(ops.alloc_zero_bf16(rows_ * ops.config.intermediate_size)) {}

void HrmLayerOps::transformer_module(const CudaSlice<bf16>& z_a, const CudaSlice<bf16>& z_b, CudaSlice<bf16>& output,
                                     size_t n_layers, const LayerCallbacks& layer, ModuleScratch& s) const {
  const size_t rows = s.rows, hidden = config.hidden_size;
  if (n_layers == 0) fail(HrmError::Kind::InvalidInput, HRM_ERR_INVALID_SHAPE, "transformer_module: no layers");
  if (!layer.attention || !layer.gate_up || !layer.down)
    fail(HrmError::Kind::InvalidInput, HRM_ERR_NULL_POINTER, "transformer_module: a layer callback is empty");
  if (s.x.len() < rows * hidden || s.g.len() < rows * config.intermediate_size)
    fail(HrmError::Kind::InvalidInput, HRM_ERR_INVALID_SHAPE,
         "transformer_module: scratch was built for another hidden / intermediate size");
  need(z_a, rows * hidden, "transformer_module", "z_a");
  need(z_b, rows * hidden, "transformer_module", "z_b");
  need(output, rows * hidden, "transformer_module", "output");
  if (output.device_ptr() == z_b.device_ptr())
    fail(HrmError::Kind::InvalidInput, HRM_ERR_ALIASING, "transformer_module: output aliases z_b");
  add_rms_norm(z_a, z_b, s.x, s.n, nullptr, rows, hidden);
  for (size_t i = 0; i < n_layers; ++i) {
    layer.attention(i, s.n, s.a);
    add_rms_norm(s.x, s.a, s.x, s.n2, nullptr, rows, hidden);
    layer.gate_up(i, s.n2, s.g, s.u);
    swiglu_ffn(s.g, s.u, s.act, rows * config.intermediate_size);
    layer.down(i, s.act, s.d);
    add_rms_norm(s.x, s.d, s.x, i + 1 == n_layers ? output : s.n, nullptr, rows, hidden);
  }
}

void HrmLayerOps::recurrent_forward(const CudaSlice<uint32_t>& input_ids, const CudaSlice<bf16>& embed_table,
                                    size_t vocab_size, const CudaSlice<bf16>& z_l_init, size_t h_cycles,
                                    size_t l_cycles, const ModuleCallbacks& l_module,
                                    const ModuleCallbacks& h_module, ModuleScratch& scratch, CudaSlice<bf16>& z_h,
                                    CudaSlice<bf16>& z_l) const {
  const size_t rows = scratch.rows, hidden = config.hidden_size;
  embedding_lookup(input_ids, embed_table, z_h, 1, rows, hidden, vocab_size, config.embedding_scale);
  broadcast_vec(z_l, z_l_init, rows, hidden);
  size_t slot = 0;
  auto run = [&](const ModuleCallbacks& m, CudaSlice<bf16>& z_a, const CudaSlice<bf16>& z_b) {
    LayerCallbacks cb;
    const size_t base = slot;
    cb.attention = [&m, base](size_t i, const CudaSlice<bf16>& n, CudaSlice<bf16>& out) {
      m.attention(i, base + i, n, out);
    };
    cb.gate_up = m.gate_up;
    cb.down = m.down;
    transformer_module(z_a, z_b, z_a, m.n_layers, cb, scratch);
    slot += m.n_layers;
  };
  for (size_t h = 0; h < h_cycles; ++h) {
    for (size_t l = 0; l < l_cycles; ++l) run(l_module, z_l, z_h);
    run(h_module, z_h, z_l);
  }
}

}  // namespace hrm
