// safetensors header parsing and validation (see safetensors.hpp).
#include "safetensors.hpp"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <utility>

namespace hrm {

namespace {

using Kind = SafetensorsError::Kind;

constexpr uint64_t kMaxHeader = 100000000;  // the crate's MAX_HEADER_SIZE
constexpr int kMaxDepth = 128;              // serde_json's recursion limit

[[noreturn]] void fail(Kind k, const std::string& what) { throw SafetensorsError(k, what); }

const struct {
  const char* name;
  StDtype dtype;
  size_t size;
} kDtypes[] = {{"BOOL", StDtype::BOOL, 1}, {"U8", StDtype::U8, 1},         {"I8", StDtype::I8, 1},
               {"F8_E5M2", StDtype::F8_E5M2, 1}, {"F8_E4M3", StDtype::F8_E4M3, 1}, {"I16", StDtype::I16, 2},
               {"U16", StDtype::U16, 2},   {"F16", StDtype::F16, 2},       {"BF16", StDtype::BF16, 2},
               {"I32", StDtype::I32, 4},   {"U32", StDtype::U32, 4},       {"F32", StDtype::F32, 4},
               {"F64", StDtype::F64, 8},   {"I64", StDtype::I64, 8},       {"U64", StDtype::U64, 8}};

// Well-formed UTF-8 (no overlong forms, no surrogates, at most U+10FFFF).
bool valid_utf8(const uint8_t* s, size_t n) {
  size_t i = 0;
  while (i < n) {
    const uint8_t c = s[i];
    if (c < 0x80) { ++i; continue; }
    int len;
    uint32_t cp;
    if ((c & 0xE0) == 0xC0) { len = 2; cp = c & 0x1F; }
    else if ((c & 0xF0) == 0xE0) { len = 3; cp = c & 0x0F; }
    else if ((c & 0xF8) == 0xF0) { len = 4; cp = c & 0x07; }
    else return false;
    if (i + len > n) return false;
    for (int k = 1; k < len; ++k) {
      if ((s[i + k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (s[i + k] & 0x3F);
    }
    if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000)) return false;
    if (cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    i += len;
  }
  return true;
}

// ------------------------------------------------------------------- JSON
// A strict JSON (RFC 8259) reader for the header: values are kept as a small
// tree; numbers remember whether they are plain non-negative integers that
// fit 64 bits (the only numbers the schema accepts, as serde's usize).  A key
// repeated within an object, a lone surrogate escape or a control character
// in a string is an error.
struct JValue {
  enum class T { Null, Bool, Number, String, Array, Object } t = T::Null;
  bool b = false;
  bool is_u64 = false;
  uint64_t u = 0;
  std::string s;
  std::vector<JValue> arr;
  std::vector<std::pair<std::string, JValue>> obj;
};

class JsonReader {
 public:
  JsonReader(const char* p, size_t n) : p_(p), end_(p + n) {}

  JValue document() {
    JValue v = value(0);
    ws();
    if (p_ != end_) bad("trailing characters");
    return v;
  }

 private:
  [[noreturn]] void bad(const std::string& why) { fail(Kind::InvalidHeaderDeserialization, "header JSON: " + why); }

  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }

  bool lit(const char* word) {
    const size_t n = std::strlen(word);
    if ((size_t)(end_ - p_) >= n && std::memcmp(p_, word, n) == 0) {
      p_ += n;
      return true;
    }
    return false;
  }

  JValue value(int depth) {
    if (depth > kMaxDepth) bad("nested too deeply");
    ws();
    if (p_ == end_) bad("unexpected end");
    JValue v;
    const char c = *p_;
    if (c == '{') {
      v.t = JValue::T::Object;
      ++p_;
      ws();
      if (p_ < end_ && *p_ == '}') { ++p_; return v; }
      while (true) {
        ws();
        if (p_ == end_ || *p_ != '"') bad("expected a key");
        std::string key = string();
        for (const auto& kv : v.obj)
          if (kv.first == key) bad("duplicate key");
        ws();
        if (p_ == end_ || *p_ != ':') bad("expected ':'");
        ++p_;
        v.obj.emplace_back(std::move(key), value(depth + 1));
        ws();
        if (p_ < end_ && *p_ == ',') { ++p_; continue; }
        if (p_ < end_ && *p_ == '}') { ++p_; return v; }
        bad("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.t = JValue::T::Array;
      ++p_;
      ws();
      if (p_ < end_ && *p_ == ']') { ++p_; return v; }
      while (true) {
        v.arr.push_back(value(depth + 1));
        ws();
        if (p_ < end_ && *p_ == ',') { ++p_; continue; }
        if (p_ < end_ && *p_ == ']') { ++p_; return v; }
        bad("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.t = JValue::T::String;
      v.s = string();
      return v;
    }
    if (lit("true")) { v.t = JValue::T::Bool; v.b = true; return v; }
    if (lit("false")) { v.t = JValue::T::Bool; return v; }
    if (lit("null")) return v;
    if (c == '-' || (c >= '0' && c <= '9')) return number();
    bad("unexpected character");
  }

  JValue number() {
    JValue v;
    v.t = JValue::T::Number;
    const bool neg = *p_ == '-';
    if (neg) ++p_;
    if (p_ == end_ || *p_ < '0' || *p_ > '9') bad("bad number");
    bool overflow = false;
    uint64_t u = 0;
    if (*p_ == '0') {
      ++p_;
    } else {
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') {
        const uint64_t d = (uint64_t)(*p_ - '0');
        if (u > (UINT64_MAX - d) / 10) overflow = true;
        u = u * 10 + d;
        ++p_;
      }
    }
    bool plain = true;
    if (p_ < end_ && *p_ == '.') {
      plain = false;
      ++p_;
      if (p_ == end_ || *p_ < '0' || *p_ > '9') bad("bad fraction");
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
      plain = false;
      ++p_;
      if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
      if (p_ == end_ || *p_ < '0' || *p_ > '9') bad("bad exponent");
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    v.is_u64 = plain && !overflow && (!neg || u == 0);
    v.u = u;
    return v;
  }

  static void put_utf8(std::string& out, uint32_t cp) {
    if (cp < 0x80) {
      out += (char)cp;
    } else if (cp < 0x800) {
      out += (char)(0xC0 | (cp >> 6));
      out += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      out += (char)(0xE0 | (cp >> 12));
      out += (char)(0x80 | ((cp >> 6) & 0x3F));
      out += (char)(0x80 | (cp & 0x3F));
    } else {
      out += (char)(0xF0 | (cp >> 18));
      out += (char)(0x80 | ((cp >> 12) & 0x3F));
      out += (char)(0x80 | ((cp >> 6) & 0x3F));
      out += (char)(0x80 | (cp & 0x3F));
    }
  }

  uint32_t hex4() {
    if (end_ - p_ < 4) bad("short \\u escape");
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) {
      const char h = *p_++;
      v <<= 4;
      if (h >= '0' && h <= '9') v |= (uint32_t)(h - '0');
      else if (h >= 'a' && h <= 'f') v |= (uint32_t)(h - 'a' + 10);
      else if (h >= 'A' && h <= 'F') v |= (uint32_t)(h - 'A' + 10);
      else bad("bad \\u escape");
    }
    return v;
  }

  std::string string() {
    ++p_;  // opening quote
    std::string out;
    while (true) {
      if (p_ == end_) bad("unterminated string");
      const unsigned char c = (unsigned char)*p_++;
      if (c == '"') return out;
      if (c < 0x20) bad("control character in a string");
      if (c != '\\') { out += (char)c; continue; }
      if (p_ == end_) bad("unterminated escape");
      const char e = *p_++;
      switch (e) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp <= 0xDBFF) {  // a high surrogate needs its low half
            if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') bad("lone surrogate");
            p_ += 2;
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo > 0xDFFF) bad("lone surrogate");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp <= 0xDFFF) {
            bad("lone surrogate");
          }
          put_utf8(out, cp);
          break;
        }
        default: bad("bad escape");
      }
    }
  }

  const char* p_;
  const char* end_;
};

// Checked products (the crate's checked_mul chain: ValidationOverflow).
bool mul_ok(uint64_t a, uint64_t b, uint64_t* out) {
  if (a != 0 && b > UINT64_MAX / a) return false;
  *out = a * b;
  return true;
}

StTensor tensor_info(const std::string& name, const JValue& v) {
  auto need = [&](const std::string& why) -> void {
    fail(Kind::InvalidHeaderDeserialization, "tensor '" + name + "': " + why);
  };
  if (v.t != JValue::T::Object) need("not an object");
  const JValue *dtype = nullptr, *shape = nullptr, *offsets = nullptr;
  for (const auto& kv : v.obj) {
    const JValue** slot = kv.first == "dtype" ? &dtype
                          : kv.first == "shape" ? &shape
                          : kv.first == "data_offsets" ? &offsets : nullptr;
    if (slot) *slot = &kv.second;  // other fields are ignored
  }
  if (!dtype || !shape || !offsets) need("missing dtype, shape or data_offsets");
  StTensor t;
  t.name = name;
  bool known = false;
  if (dtype->t == JValue::T::String)
    for (const auto& d : kDtypes)
      if (dtype->s == d.name) { t.dtype = d.dtype; known = true; }
  if (!known) need("unknown dtype");
  if (shape->t != JValue::T::Array) need("shape is not an array");
  for (const auto& d : shape->arr) {
    if (d.t != JValue::T::Number || !d.is_u64) need("shape entries must be non-negative integers");
    t.shape.push_back(d.u);
  }
  if (offsets->t != JValue::T::Array || offsets->arr.size() != 2) need("data_offsets must be [begin, end]");
  for (const auto& d : offsets->arr)
    if (d.t != JValue::T::Number || !d.is_u64) need("data_offsets must be non-negative integers");
  t.begin = offsets->arr[0].u;
  t.end = offsets->arr[1].u;
  return t;
}

}  // namespace

size_t st_dtype_size(StDtype d) {
  for (const auto& x : kDtypes)
    if (x.dtype == d) return x.size;
  return 0;
}

const char* st_dtype_name(StDtype d) {
  for (const auto& x : kDtypes)
    if (x.dtype == d) return x.name;
  return "?";
}

uint64_t StTensor::numel() const {
  uint64_t n = 1;
  for (uint64_t d : shape) n *= d;
  return n;
}

const StTensor* SafetensorsHeader::find(const std::string& name) const {
  for (const auto& t : tensors)
    if (t.name == name) return &t;
  return nullptr;
}

SafetensorsHeader SafetensorsHeader::parse(const uint8_t* prefix, size_t prefix_len, uint64_t file_len) {
  if (file_len < 8 || prefix_len < 8) fail(Kind::HeaderTooSmall, "file shorter than the 8-byte header length");
  uint64_t n = 0;
  for (int i = 7; i >= 0; --i) n = (n << 8) | prefix[i];
  if (n > kMaxHeader) fail(Kind::HeaderTooLarge, "header length " + std::to_string(n) + " exceeds 100000000");
  if (8 + n > file_len || 8 + n > prefix_len)
    fail(Kind::InvalidHeaderLength, "header length " + std::to_string(n) + " runs past the end of the file");
  const uint8_t* h = prefix + 8;
  if (!valid_utf8(h, (size_t)n)) fail(Kind::InvalidHeader, "header is not UTF-8");
  if (n == 0 || h[0] != '{') fail(Kind::InvalidHeaderStart, "header does not start with '{'");

  const JValue doc = JsonReader(reinterpret_cast<const char*>(h), (size_t)n).document();
  if (doc.t != JValue::T::Object) fail(Kind::InvalidHeaderDeserialization, "header is not a JSON object");
  SafetensorsHeader out;
  out.header_len = n;
  for (const auto& kv : doc.obj) {  // keys are unique (the reader rejects duplicates)
    if (kv.first == "__metadata__") {
      if (kv.second.t == JValue::T::Null) continue;
      if (kv.second.t != JValue::T::Object) fail(Kind::InvalidHeaderDeserialization, "__metadata__ is not an object");
      for (const auto& m : kv.second.obj) {
        if (m.second.t != JValue::T::String)
          fail(Kind::InvalidHeaderDeserialization, "__metadata__ values must be strings");
        out.metadata[m.first] = m.second.s;
      }
      continue;
    }
    out.tensors.push_back(tensor_info(kv.first, kv.second));
  }
  // Metadata::new: order by data offsets, then validate.
  std::stable_sort(out.tensors.begin(), out.tensors.end(), [](const StTensor& a, const StTensor& b) {
    return a.begin != b.begin ? a.begin < b.begin : a.end < b.end;
  });
  uint64_t start = 0;
  for (const auto& t : out.tensors) {
    if (t.begin != start || t.end < t.begin) fail(Kind::InvalidOffset, "tensor '" + t.name + "' has invalid offsets");
    start = t.end;
    uint64_t nel = 1, nbytes = 0;
    for (uint64_t d : t.shape)
      if (!mul_ok(nel, d, &nel)) fail(Kind::ValidationOverflow, "tensor '" + t.name + "': shape overflows");
    if (!mul_ok(nel, st_dtype_size(t.dtype), &nbytes))
      fail(Kind::ValidationOverflow, "tensor '" + t.name + "': byte size overflows");
    if (t.end - t.begin != nbytes)
      fail(Kind::TensorInvalidInfo, "tensor '" + t.name + "': " + std::to_string(t.end - t.begin) +
                                        " bytes for shape x dtype " + std::to_string(nbytes));
  }
  if (file_len - 8 - n != start)
    fail(Kind::MetadataIncompleteBuffer, "data section of " + std::to_string(file_len - 8 - n) +
                                             " bytes, tensors cover " + std::to_string(start));
  return out;
}

SafetensorsHeader SafetensorsHeader::read(const std::string& path) {
  const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) fail(Kind::Io, "cannot open " + path);
  struct stat st;
  if (::fstat(fd, &st) != 0) {
    ::close(fd);
    fail(Kind::Io, "cannot stat " + path);
  }
  const uint64_t file_len = (uint64_t)st.st_size;
  std::vector<uint8_t> buf(8);
  ssize_t got = ::pread(fd, buf.data(), 8, 0);
  if (got < 8) {
    ::close(fd);
    return parse(buf.data(), got < 0 ? 0 : (size_t)got, file_len);  // HeaderTooSmall
  }
  uint64_t n = 0;
  for (int i = 7; i >= 0; --i) n = (n << 8) | buf[i];
  const uint64_t want = n > kMaxHeader ? 0 : std::min<uint64_t>(n, file_len - 8);
  buf.resize(8 + want);
  uint64_t done = 0;
  while (done < want) {
    got = ::pread(fd, buf.data() + 8 + done, (size_t)(want - done), (off_t)(8 + done));
    if (got <= 0) {
      ::close(fd);
      fail(Kind::Io, "cannot read the header of " + path);
    }
    done += (uint64_t)got;
  }
  ::close(fd);
  return parse(buf.data(), buf.size(), file_len);
}

}  // namespace hrm
