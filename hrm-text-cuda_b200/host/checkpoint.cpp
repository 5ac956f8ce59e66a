// HrmLayerOps::load_safetensors (src/lib.rs:2023-2125): checkpoint file ->
// bf16 device slices, converted on the GPU.
//
// The reference reads the whole file, converts every tensor to bf16 on the
// host one element at a time (raw_to_bf16, src/lib.rs:1981-2008), splits
// gate_up on the host and copies each tensor with a synchronous htod_copy.
// Here only the bytes of the tensors the model uses are read, in chunks of
// whole elements, into a ring of pinned host buffers by several threads at
// once; each chunk's tensors are uploaded raw and converted on the GPU
// (hrm_upload_to_bf16, one device staging buffer), and the next chunk is read
// while the GPU copies the previous one.  gate_up's two halves go straight to
// gate_proj and up_proj.
#include <fcntl.h>
#include <sched.h>
#include <unistd.h>

#include <algorithm>
#include <string>
#include <thread>
#include <vector>

#include "hrm_layer_ops.hpp"
#include "safetensors.hpp"

namespace hrm {

namespace {

[[noreturn]] void fail(HrmError::Kind kind, int status, const std::string& what) { throw HrmError(kind, status, what); }

void cuda_ok(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    fail(HrmError::Kind::Driver, HRM_ERR_CUDA + (int)e, std::string(what) + ": " + cudaGetErrorString(e));
}

int abi_dtype(StDtype d) {
  switch (d) {
    case StDtype::BF16: return HRM_DTYPE_BF16;
    case StDtype::F32: return HRM_DTYPE_F32;
    case StDtype::F16: return HRM_DTYPE_F16;
    default: return -1;
  }
}

// One contiguous byte range of the file that lands in one destination.
struct Piece {
  uint64_t off;    // file offset
  uint64_t bytes;  // a whole number of elements
  int dtype;       // HRM_DTYPE_*
  uint64_t esize;  // bytes per element
  bf16* dst;       // first destination element
};

// File-contiguous pieces read and uploaded together.
struct Chunk {
  uint64_t off = 0, bytes = 0;
  std::vector<Piece> pieces;
};

// Groups pieces (sorted by offset) into chunks of at most `cap` bytes, cutting
// a piece at whole elements where it crosses a chunk's end.
std::vector<Chunk> plan_chunks(std::vector<Piece> pieces, uint64_t cap) {
  std::sort(pieces.begin(), pieces.end(), [](const Piece& a, const Piece& b) { return a.off < b.off; });
  std::vector<Chunk> chunks;
  for (Piece p : pieces) {
    while (p.bytes > 0) {
      if (chunks.empty() || chunks.back().off + chunks.back().bytes != p.off ||
          cap - chunks.back().bytes < p.esize) {
        chunks.emplace_back();
        chunks.back().off = p.off;
      }
      Chunk& c = chunks.back();
      const uint64_t room = (cap - c.bytes) / p.esize * p.esize;
      const uint64_t take = std::min(room, p.bytes);
      Piece part = p;
      part.bytes = take;
      c.pieces.push_back(part);
      c.bytes += take;
      p.off += take;
      p.bytes -= take;
      p.dst += take / p.esize;
    }
  }
  return chunks;
}

// Reads [off, off + bytes) of fd into dst with `threads` concurrent preads.
bool read_parallel(int fd, uint8_t* dst, uint64_t off, uint64_t bytes, int threads) {
  const uint64_t per = (bytes + threads - 1) / threads;
  std::vector<std::thread> pool;
  std::vector<char> ok(threads, 1);
  for (int t = 0; t < threads; ++t) {
    const uint64_t b0 = std::min(bytes, per * t), b1 = std::min(bytes, per * (t + 1));
    if (b0 >= b1) continue;
    pool.emplace_back([=, &ok] {
      uint64_t done = b0;
      while (done < b1) {
        const ssize_t got = ::pread(fd, dst + done, (size_t)(b1 - done), (off_t)(off + done));
        if (got <= 0) { ok[t] = 0; return; }
        done += (uint64_t)got;
      }
    });
  }
  for (auto& th : pool) th.join();
  return std::all_of(ok.begin(), ok.end(), [](char c) { return c != 0; });
}

}  // namespace

HrmLayerOps::ModelWeights HrmLayerOps::load_safetensors(const std::string& path, size_t chunk_bytes,
                                                        int reader_threads) const {
  SafetensorsHeader hdr;
  try {
    hdr = SafetensorsHeader::read(path);
  } catch (const SafetensorsError& e) {
    fail(HrmError::Kind::Io, 0, std::string("safetensors: ") + e.what());
  }
  for (const auto& t : hdr.tensors)
    if (abi_dtype(t.dtype) < 0)
      fail(HrmError::Kind::InvalidInput, HRM_ERR_DTYPE,
           std::string("unsupported dtype ") + st_dtype_name(t.dtype) + " of tensor " + t.name);
  if (chunk_bytes < 64) chunk_bytes = 64;
  chunk_bytes = chunk_bytes / 16 * 16;
  if (reader_threads < 1) {
    cpu_set_t set;
    reader_threads = sched_getaffinity(0, sizeof(set), &set) == 0 ? CPU_COUNT(&set) : 1;
    reader_threads = std::max(1, std::min(16, reader_threads));
  }

  std::vector<Piece> pieces;
  auto tensor = [&](const std::string& name) -> const StTensor& {
    const StTensor* t = hdr.find(name);
    if (!t) {  // src/lib.rs:2011-2020
      std::string keys;
      for (const auto& x : hdr.tensors)
        if (x.name.find("layer") != std::string::npos || x.name.find("embed") != std::string::npos ||
            x.name.find("lm_head") != std::string::npos)
          keys += (keys.empty() ? "" : ", ") + x.name;
      fail(HrmError::Kind::InvalidInput, HRM_ERR_INVALID_SHAPE,
           "missing tensor: " + name + ". Available keys: [" + keys + "]");
    }
    return *t;
  };
  // `n` elements of t starting at element `first`, into a new slice.
  auto take = [&](const StTensor& t, uint64_t first, uint64_t n) {
    CudaSlice<bf16> s = alloc_zero_bf16((size_t)n);
    const uint64_t es = st_dtype_size(t.dtype);
    if (n > 0)
      pieces.push_back(Piece{hdr.data_offset() + t.begin + first * es, n * es, abi_dtype(t.dtype), es,
                             s.device_ptr()});
    return s;
  };
  auto whole = [&](const std::string& name) {
    const StTensor& t = tensor(name);
    return take(t, 0, t.numel());
  };

  const size_t L = config.n_layers, I = config.intermediate_size, H = config.hidden_size;
  const bool attn = hdr.find("model.H_module.layers.0.attn.gqkv_proj.weight") != nullptr;  // src/lib.rs:2043-2044
  auto module = [&](const std::string& prefix) {
    ModuleWeights m;
    for (size_t i = 0; i < L; ++i) {
      const std::string p = prefix + "." + std::to_string(i);
      LayerWeights lw;
      lw.gqkv_proj = whole(p + (attn ? ".attn" : "") + ".gqkv_proj.weight");
      lw.o_proj = whole(p + (attn ? ".attn" : "") + ".o_proj.weight");
      const StTensor& gu = tensor(p + (attn ? ".mlp" : "") + ".gate_up_proj.weight");
      const uint64_t split = (uint64_t)I * H;  // src/lib.rs:2072-2078
      if (gu.numel() < split)
        fail(HrmError::Kind::InvalidInput, HRM_ERR_INVALID_SHAPE,
             gu.name + ": " + std::to_string(gu.numel()) + " elements, fewer than intermediate x hidden");
      lw.gate_proj = take(gu, 0, split);
      lw.up_proj = take(gu, split, gu.numel() - split);
      lw.down_proj = whole(p + (attn ? ".mlp" : "") + ".down_proj.weight");
      m.layers.push_back(std::move(lw));
    }
    return m;
  };
  ModelWeights w;
  w.h_module = module("model.H_module.layers");
  w.l_module = module("model.L_module.layers");
  w.embed_tokens = whole("model.embed_tokens.weight");
  w.lm_head = whole(hdr.find("lm_head.weight") ? "lm_head.weight" : "model.lm_head.weight");
  w.z_l_init = whole("model.z_L_init");

  const std::vector<Chunk> chunks = plan_chunks(std::move(pieces), chunk_bytes);
  if (chunks.empty()) return w;
  const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) fail(HrmError::Kind::Io, 0, "cannot open " + path);
  constexpr int kRing = 3;
  uint8_t* host[kRing] = {nullptr, nullptr, nullptr};
  cudaEvent_t done[kRing] = {nullptr, nullptr, nullptr};
  void* staging = nullptr;
  const size_t staging_bytes = std::min<size_t>(chunk_bytes, 32u << 20);
  auto release = [&] {
    for (int r = 0; r < kRing; ++r) {
      if (done[r]) cudaEventDestroy(done[r]);
      if (host[r]) cudaFreeHost(host[r]);
    }
    if (staging) cudaFree(staging);
    ::close(fd);
  };
  try {
    for (int r = 0; r < kRing; ++r) {
      cuda_ok(cudaHostAlloc(reinterpret_cast<void**>(&host[r]), chunk_bytes, cudaHostAllocDefault), "cudaHostAlloc");
      cuda_ok(cudaEventCreateWithFlags(&done[r], cudaEventDisableTiming), "cudaEventCreate");
    }
    cuda_ok(cudaMalloc(&staging, staging_bytes), "cudaMalloc");
    for (size_t c = 0; c < chunks.size(); ++c) {
      const int r = (int)(c % kRing);
      if (c >= (size_t)kRing) cuda_ok(cudaEventSynchronize(done[r]), "cudaEventSynchronize");  // slot's copies done
      const Chunk& ch = chunks[c];
      if (!read_parallel(fd, host[r], ch.off, ch.bytes, reader_threads))
        fail(HrmError::Kind::Io, 0, "cannot read " + path);
      for (const Piece& p : ch.pieces)
        check(hrm_upload_to_bf16(host[r] + (p.off - ch.off), p.dtype, p.dst, (int64_t)(p.bytes / p.esize), staging,
                                 (int64_t)staging_bytes, stream_),
              "load_safetensors");
      cuda_ok(cudaEventRecord(done[r], stream_), "cudaEventRecord");
    }
    cuda_ok(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
  } catch (...) {
    cudaStreamSynchronize(stream_);
    release();
    throw;
  }
  release();
  return w;
}

}  // namespace hrm
