// C++ host layer over the C ABI (include/hrm_ops.h), mirroring the kernel
// wrapper methods of the reference's `HrmForwardPass` (src/lib.rs:154-565):
// same method names, argument order and meaning, hyper-parameters read from
// an HrmConfig, and failures reported as an HrmError of the same kinds as the
// reference's error enum (src/lib.rs:5-19).  Rust's `CudaResult<()>` maps to
// a void method that throws HrmError.
//
// Device memory follows cudarc's CudaSlice<T> (an owned, typed allocation on
// one device); the layer owns one CUDA stream, the analogue of
// `CudaDevice::cu_stream()`, and every launch is queued on it.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

#include "hrm_ops.h"

namespace hrm {

// IEEE bfloat16 storage, as half::bf16 (round-to-nearest-even from f32).
struct bf16 {
  uint16_t bits = 0;
  static bf16 from_f32(float f);
  float to_f32() const;
};

// Mirrors HrmError (src/lib.rs:5-19): Driver = a CUDA error, InvalidInput =
// a rejected argument, KernelNotFound = the kernel library is not usable,
// Io = a checkpoint that cannot be read or deserialised.
class HrmError : public std::runtime_error {
 public:
  enum class Kind { Driver, InvalidInput, KernelNotFound, Io };
  HrmError(Kind kind, int status, const std::string& what)
      : std::runtime_error(what), kind_(kind), status_(status) {}
  Kind kind() const { return kind_; }
  int status() const { return status_; }

 private:
  Kind kind_;
  int status_;
};

// Mirrors HrmConfig and its defaults (src/lib.rs:24-60).
struct HrmConfig {
  size_t hidden_size = 1536;
  size_t num_heads = 12;
  size_t head_dim = 128;
  size_t intermediate_size = 4096;
  size_t h_cycles = 2;
  size_t l_cycles = 3;
  size_t n_layers = 16;
  size_t max_seq_len = 4096;
  size_t vocab_size = 65536;
  float rope_theta = 10000.0f;
  float norm_eps = 1e-6f;
  float init_std = 0.025515518153991442f;  // 1 / sqrt(1536)
  float embedding_scale = 39.191835884530846f;
};

// Owned device allocation of `len` elements of T (cudarc CudaSlice<T>).
template <class T>
class CudaSlice {
 public:
  CudaSlice() = default;
  CudaSlice(T* ptr, size_t len) : ptr_(ptr), len_(len) {}
  CudaSlice(const CudaSlice&) = delete;
  CudaSlice& operator=(const CudaSlice&) = delete;
  CudaSlice(CudaSlice&& o) noexcept : ptr_(o.ptr_), len_(o.len_) { o.ptr_ = nullptr; o.len_ = 0; }
  CudaSlice& operator=(CudaSlice&& o) noexcept {
    if (this != &o) { reset(); ptr_ = o.ptr_; len_ = o.len_; o.ptr_ = nullptr; o.len_ = 0; }
    return *this;
  }
  ~CudaSlice() { reset(); }
  T* device_ptr() const { return ptr_; }
  size_t len() const { return len_; }

 private:
  void reset() { if (ptr_) cudaFree(ptr_); ptr_ = nullptr; len_ = 0; }
  T* ptr_ = nullptr;
  size_t len_ = 0;
};

class HrmLayerOps {
 public:
  // CudaDevice::new(dev_ordinal) + a stream (src/lib.rs:185-186).
  explicit HrmLayerOps(int dev_ordinal, HrmConfig config = HrmConfig());
  ~HrmLayerOps();
  HrmLayerOps(const HrmLayerOps&) = delete;
  HrmLayerOps& operator=(const HrmLayerOps&) = delete;

  HrmConfig config;

  // ---- buffers (src/lib.rs:258-267 and cudarc's htod_copy / sync_reclaim)
  CudaSlice<bf16> alloc_zero_bf16(size_t len) const;
  CudaSlice<bf16> htod_copy_bf16(const std::vector<bf16>& host) const;
  CudaSlice<uint32_t> htod_copy_u32(const std::vector<uint32_t>& host) const;
  std::vector<bf16> sync_reclaim(CudaSlice<bf16>&& slice) const;  // waits for the stream
  cudaStream_t cu_stream() const { return stream_; }

  // ---- the kernel wrappers (same signatures as src/lib.rs:378-565)
  void additive_inject(const CudaSlice<bf16>& z_a, const CudaSlice<bf16>& z_b, CudaSlice<bf16>& z_out,
                       size_t total_elements) const;
  void rms_norm(const CudaSlice<bf16>& input, CudaSlice<bf16>& output, size_t rows, size_t hidden_size) const;
  void rope_embed(CudaSlice<bf16>& q, CudaSlice<bf16>& k, size_t batch_size, size_t num_heads, size_t seq_len,
                  size_t head_dim, size_t position_offset) const;
  void swiglu_ffn(const CudaSlice<bf16>& gate, const CudaSlice<bf16>& up, CudaSlice<bf16>& output,
                  size_t total_elements) const;
  void embedding_lookup(const CudaSlice<uint32_t>& input_ids, const CudaSlice<bf16>& embedding_table,
                        CudaSlice<bf16>& output, size_t batch_size, size_t seq_len, size_t hidden_size,
                        size_t vocab_size, float embedding_scale) const;

  // src/lib.rs:505-527: output = sigmoid(gate) * attn_out.
  void gated_attn_output(const CudaSlice<bf16>& gate, const CudaSlice<bf16>& attn_out, CudaSlice<bf16>& output,
                         size_t total_elements) const;
  // src/lib.rs:607-630: attn_out *= sigmoid(gate), in place.
  void apply_attn_gate(const CudaSlice<bf16>& gate, CudaSlice<bf16>& attn_out, size_t total_elements) const;
  // src/lib.rs:748-767: dst[r, :] = src for r < n_copies.
  void broadcast_vec(CudaSlice<bf16>& dst, const CudaSlice<bf16>& src, size_t n_copies, size_t vec_len) const;

  // ---- weight loading (src/lib.rs:1981-2008)
  // raw_to_bf16: little-endian checkpoint bytes of `dtype` (HRM_DTYPE_BF16 /
  // F32 / F16) -> bf16 values on the host, as the reference's loader returns
  // them, converted on the GPU with the same bits (half 2.7.1 rules).  A byte
  // count that is not a whole number of elements, or another dtype, throws
  // InvalidInput (the reference asserts or panics).
  std::vector<bf16> raw_to_bf16(int dtype, const std::vector<uint8_t>& raw) const;
  // The same conversion into a new device slice, for a loader that keeps the
  // weights on the GPU (the reference converts on the host, then htod_copy).
  CudaSlice<bf16> htod_raw_as_bf16(int dtype, const uint8_t* raw, size_t nbytes) const;

  // ---- checkpoint loading (src/lib.rs:2023-2125)
  struct LayerWeights {  // src/lib.rs:62-69
    CudaSlice<bf16> gqkv_proj, o_proj, gate_proj, up_proj, down_proj;
  };
  struct ModuleWeights {  // src/lib.rs:72-74
    std::vector<LayerWeights> layers;
  };
  struct ModelWeights {  // src/lib.rs:77-83
    ModuleWeights h_module, l_module;
    CudaSlice<bf16> embed_tokens, lm_head, z_l_init;
  };
  // load_safetensors: the model's tensors from one safetensors file, as bf16
  // device slices, with the reference's names and rules: per module
  // ("model.H_module.layers", "model.L_module.layers") and layer, gqkv_proj,
  // o_proj, gate_up_proj split at intermediate x hidden elements into
  // gate_proj and up_proj, and down_proj, under ".attn." / ".mlp." when
  // "model.H_module.layers.0.attn.gqkv_proj.weight" exists; then
  // model.embed_tokens.weight, lm_head.weight (else model.lm_head.weight) and
  // model.z_L_init.  The header is parsed and validated as safetensors 0.4.5
  // does (safetensors.hpp); the bytes of the tensors used are read from the
  // file in chunks into pinned host buffers (several reader threads), copied
  // to the GPU and converted there (hrm_upload_to_bf16), reading chunk i + 1
  // while chunk i is copied.  Returns once the weights are on the device.
  // Throws HrmError Io for an unreadable or invalid file, InvalidInput for a
  // missing tensor, a gate_up smaller than its gate half, or any tensor of a
  // dtype other than BF16 / F32 / F16 (the reference converts every tensor
  // of the file and panics on those).
  // reader_threads 0: one per core this process may use, at most 16.
  ModelWeights load_safetensors(const std::string& path, size_t chunk_bytes = 128u << 20,
                                int reader_threads = 0) const;

  // ---- fused entry points that replace wrapper sequences of the reference
  // additive_inject -> rms_norm (src/lib.rs:976-979); weight may be null.
  void add_rms_norm(const CudaSlice<bf16>& x, const CudaSlice<bf16>& branch, CudaSlice<bf16>& residual_out,
                    CudaSlice<bf16>& normed_out, const CudaSlice<bf16>* weight, size_t rows,
                    size_t hidden_size) const;
  // embedding_lookup -> rms_norm (src/lib.rs:1191-1200, 969); hidden_out may be null.
  void embed_rms_norm(const CudaSlice<uint32_t>& input_ids, const CudaSlice<bf16>& embedding_table,
                      CudaSlice<bf16>* hidden_out, CudaSlice<bf16>& normed_out, const CudaSlice<bf16>* weight,
                      size_t rows, size_t hidden_size, size_t vocab_size, float embedding_scale) const;
  // split_gqkv -> rope_embed -> kv_cache_update in one pass (src/lib.rs:798-857);
  // k_cache / v_cache ([batch, heads, cache_len, head_dim]) may both be null.
  void split_gqkv_rope(const CudaSlice<bf16>& gqkv, CudaSlice<bf16>& gate, CudaSlice<bf16>& q, CudaSlice<bf16>& k,
                       CudaSlice<bf16>& v, CudaSlice<bf16>* k_cache, CudaSlice<bf16>* v_cache, size_t batch_size,
                       size_t seq_len, size_t num_heads, size_t head_dim, size_t position_offset, size_t cache_len,
                       size_t cache_offset) const;
  // ---- the layer loop's residual / norm schedule
  // Scratch of one module pass over `rows` tokens (the reference's
  // ScratchBuffers, src/lib.rs:86-112): the residual stream x, the normed
  // activations n / n2, the attention output a and the down projection d
  // ([rows x hidden]); the FFN gate, up and activation ([rows x intermediate]).
  struct ModuleScratch {
    ModuleScratch(const HrmLayerOps& ops, size_t rows);
    size_t rows;
    CudaSlice<bf16> x, n, n2, a, d, g, u, act;
  };
  // The caller's attention and FFN GEMMs, queued on cu_stream().
  struct LayerCallbacks {
    std::function<void(size_t layer, const CudaSlice<bf16>& normed, CudaSlice<bf16>& attn_out)> attention;
    std::function<void(size_t layer, const CudaSlice<bf16>& normed, CudaSlice<bf16>& gate, CudaSlice<bf16>& up)>
        gate_up;
    std::function<void(size_t layer, const CudaSlice<bf16>& act, CudaSlice<bf16>& down)> down;
  };
  // output = module(z_a + z_b): the cycle injection (src/lib.rs:1220-1229 or
  // 1248-1256) and transformer_module (src/lib.rs:1036-1105, layers as
  // src/lib.rs:955-1030) with every additive_inject -> rms_norm pair fused
  // and no device copies:
  //   (x, n) = add_rms_norm(z_a, z_b); per layer: attention(n) -> a,
  //   (x, n2) = add_rms_norm(x, a), gate_up(n2), swiglu_ffn, down -> d,
  //   (x, n) = add_rms_norm(x, d) -- into `output` after the last layer.
  // Bit-identical to the reference's order.  `output` may be z_a (z_L = L(z_L +
  // z_H) in place); it must not be z_b.
  void transformer_module(const CudaSlice<bf16>& z_a, const CudaSlice<bf16>& z_b, CudaSlice<bf16>& output,
                          size_t n_layers, const LayerCallbacks& layer, ModuleScratch& scratch) const;

  // One module (H or L) of recurrent_forward; its attention is also given the
  // KV-cache slot of the layer.
  struct ModuleCallbacks {
    size_t n_layers = 0;
    std::function<void(size_t layer, size_t kv_slot, const CudaSlice<bf16>& normed, CudaSlice<bf16>& attn_out)>
        attention;
    std::function<void(size_t layer, const CudaSlice<bf16>& normed, CudaSlice<bf16>& gate, CudaSlice<bf16>& up)>
        gate_up;
    std::function<void(size_t layer, const CudaSlice<bf16>& act, CudaSlice<bf16>& down)> down;
  };
  // The HRM recurrent loop over scratch.rows tokens (src/lib.rs:1189-1270):
  // z_h = embedding_lookup(input_ids) * config.embedding_scale (1189-1200),
  // z_l = broadcast(z_l_init) (1202-1203), then for each of h_cycles:
  // l_cycles x z_l = L(z_l + z_h), then z_h = H(z_h + z_l), each module pass
  // through transformer_module.  KV-cache slots are numbered as the reference's
  // kv_slot_counter: each module pass takes the next n_layers slots.
  void recurrent_forward(const CudaSlice<uint32_t>& input_ids, const CudaSlice<bf16>& embed_table,
                         size_t vocab_size, const CudaSlice<bf16>& z_l_init, size_t h_cycles, size_t l_cycles,
                         const ModuleCallbacks& l_module, const ModuleCallbacks& h_module, ModuleScratch& scratch,
                         CudaSlice<bf16>& z_h, CudaSlice<bf16>& z_l) const;

  // Builds the fp32 cos/sin table for config.head_dim / config.rope_theta
  // covering positions [0, max_positions); rope_embed uses it from then on
  // for every call it covers, and evaluates angles in-kernel otherwise.
  void build_rope_table(size_t max_positions);

 private:
  void check(int status, const char* op) const;
  int dev_ = 0;
  cudaStream_t stream_ = nullptr;
  CudaSlice<float> rope_table_;
  size_t rope_positions_ = 0;
};

}  // namespace hrm
