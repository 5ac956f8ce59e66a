// safetensors checkpoint headers: parsing and validation as the reference's
// loader gets them from the `safetensors` crate (Cargo.lock: safetensors
// 0.4.5, not vendored; its published format and validation rules restated):
//
//   [8 bytes: N, unsigned little-endian] [N bytes: UTF-8 JSON header] [data]
//
// The header is a JSON object mapping each tensor name to
// {"dtype": "F32" | "BF16" | ..., "shape": [d0, d1, ...],
//  "data_offsets": [begin, end]} (byte offsets into the data section), plus
// an optional "__metadata__" object of string values.  Validation, in the
// crate's order: at least 8 bytes; N <= 100,000,000; 8 + N within the file;
// the header is UTF-8, starts with '{' and deserialises; sorted by offsets,
// the tensors tile the data section from 0 with no gap or overlap and each
// spans exactly (product of its shape) x (dtype size) bytes; the data section
// ends at the end of the file.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace hrm {

// The crate's SafeTensorError variants that deserialisation can raise (plus
// Io for a file that cannot be read).
class SafetensorsError : public std::runtime_error {
 public:
  enum class Kind {
    HeaderTooSmall,
    HeaderTooLarge,
    InvalidHeaderLength,
    InvalidHeader,
    InvalidHeaderStart,
    InvalidHeaderDeserialization,
    InvalidOffset,
    TensorInvalidInfo,
    ValidationOverflow,
    MetadataIncompleteBuffer,
    Io,
  };
  SafetensorsError(Kind kind, const std::string& what) : std::runtime_error(what), kind_(kind) {}
  Kind kind() const { return kind_; }

 private:
  Kind kind_;
};

// The format's element types (the crate's Dtype, with its JSON names).
enum class StDtype { BOOL, U8, I8, F8_E5M2, F8_E4M3, I16, U16, F16, BF16, I32, U32, F32, F64, I64, U64 };
size_t st_dtype_size(StDtype d);
const char* st_dtype_name(StDtype d);

struct StTensor {
  std::string name;
  StDtype dtype = StDtype::U8;
  std::vector<uint64_t> shape;
  uint64_t begin = 0, end = 0;  // byte range within the data section
  uint64_t numel() const;
};

struct SafetensorsHeader {
  uint64_t header_len = 0;                      // N
  std::vector<StTensor> tensors;                // in data-offset order
  std::map<std::string, std::string> metadata;  // "__metadata__"
  uint64_t data_offset() const { return 8 + header_len; }
  uint64_t data_len() const { return tensors.empty() ? 0 : tensors.back().end; }
  const StTensor* find(const std::string& name) const;

  // Parses and validates the header of a file of file_len bytes; `prefix`
  // holds the file's first prefix_len bytes (at least 8 + N of them, or the
  // whole file if it is shorter).
  static SafetensorsHeader parse(const uint8_t* prefix, size_t prefix_len, uint64_t file_len);
  // Reads and validates the header of the file at `path`.
  static SafetensorsHeader read(const std::string& path);
};

}  // namespace hrm
