// gguf.h -- reader of Noor's GGUF v3 checkpoints (host code).
//
// The format is the one crates/noor-core/src/gguf.rs writes and reads
// (save_gguf :68-150, load_gguf :153-233):
//   header    u32 magic 0x46475547 ("GGUF"), u32 version 3, u64 tensor_count,
//             u64 metadata_count
//   metadata  metadata_count x (string key, u32 value type, value); value
//             types are Noor's own: 0 u32, 1 i32, 2 f32, 3 bool (1 byte),
//             4 string, 5 f64, 6 u64 (gguf.rs:323-347)
//   tensors   tensor_count x (string name, u32 n_dims, n_dims x u64 dims,
//             u32 type (0 F32, 1 F16), u64 offset)
//   data      from the header's end rounded up to 32 bytes; each tensor at
//             data start + offset, little-endian
// Strings are a u64 byte length and the bytes.  The file is memory-mapped:
// F32 tensors are used in place, F16 ones converted to f32 (the exact
// half-to-single conversion of tensor.rs:60-80).  Every read is bounds
// checked, so a truncated or malformed file gives an error, not a fault.
#pragma once

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace noor {
namespace gguf {

constexpr uint32_t kMagic = 0x46475547u;
constexpr uint32_t kVersion = 3;
constexpr uint64_t kAlignment = 32;
enum TensorType : uint32_t { TYPE_F32 = 0, TYPE_F16 = 1 };

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t type = 0;
  uint64_t offset = 0;
  uint64_t numel = 0;
};

inline float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1F;
  uint32_t man = h & 0x3FF;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: normalise the mantissa
      int e = -14;
      while ((man & 0x400) == 0) {
        man <<= 1;
        --e;
      }
      bits = sign | ((uint32_t)(e + 127) << 23) | ((man & 0x3FF) << 13);
    }
  } else if (exp == 31) {
    bits = sign | (0xFFu << 23) | (man << 13);
  } else {
    bits = sign | ((exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

class File {
 public:
  ~File() { close(); }

  bool open(const char* path) {
    close();
    fd_ = ::open(path, O_RDONLY);
    if (fd_ < 0) return set_error(std::string("cannot open ") + path);
    struct stat st;
    if (fstat(fd_, &st) != 0) return set_error("cannot stat the file");
    size_ = (size_t)st.st_size;
    if (size_ == 0) return set_error("empty file");
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (m == MAP_FAILED) return set_error("cannot map the file");
    base_ = static_cast<const uint8_t*>(m);
    return parse();
  }

  void close() {
    if (base_) munmap(const_cast<uint8_t*>(base_), size_);
    if (fd_ >= 0) ::close(fd_);
    base_ = nullptr;
    fd_ = -1;
    size_ = 0;
    tensors_.clear();
    index_.clear();
  }

  const std::string& error() const { return error_; }
  const std::vector<TensorInfo>& tensors() const { return tensors_; }

  const TensorInfo* find(const std::string& name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors_[it->second];
  }

  // The tensor as f32: in place for F32, else converted into `scratch`.
  const float* f32(const TensorInfo& t, std::vector<float>& scratch) const {
    const uint8_t* p = base_ + data_start_ + t.offset;
    if (t.type == TYPE_F32) return reinterpret_cast<const float*>(p);  // 32-byte aligned data, 4-byte offsets
    scratch.resize(t.numel);
    for (uint64_t i = 0; i < t.numel; ++i) {
      uint16_t v;
      std::memcpy(&v, p + 2 * i, 2);
      scratch[i] = half_to_float(v);
    }
    return scratch.data();
  }

 private:
  bool set_error(const std::string& e) {
    error_ = e;
    return false;
  }

  bool need(uint64_t n) const { return pos_ <= size_ && n <= size_ - pos_; }
  bool rd_u32(uint32_t* v) {
    if (!need(4)) return false;
    std::memcpy(v, base_ + pos_, 4);
    pos_ += 4;
    return true;
  }
  bool rd_u64(uint64_t* v) {
    if (!need(8)) return false;
    std::memcpy(v, base_ + pos_, 8);
    pos_ += 8;
    return true;
  }
  bool rd_string(std::string* s) {
    uint64_t n;
    if (!rd_u64(&n) || !need(n)) return false;
    s->assign(reinterpret_cast<const char*>(base_ + pos_), (size_t)n);
    pos_ += n;
    return true;
  }
  // skip one metadata value of Noor's value types
  bool skip_value() {
    uint32_t type;
    if (!rd_u32(&type)) return false;
    uint64_t n = 0;
    switch (type) {
      case 0: case 1: case 2: n = 4; break;
      case 3: n = 1; break;
      case 5: case 6: n = 8; break;
      case 4: {
        std::string s;
        return rd_string(&s);
      }
      default:
        error_ = "unknown metadata value type " + std::to_string(type);
        return false;
    }
    if (!need(n)) return false;
    pos_ += n;
    return true;
  }

  bool parse() {
    pos_ = 0;
    uint32_t magic, version;
    uint64_t n_tensors, n_meta;
    if (!rd_u32(&magic) || magic != kMagic) return set_error("not a GGUF file");
    if (!rd_u32(&version) || version != kVersion) return set_error("unsupported GGUF version");
    if (!rd_u64(&n_tensors) || !rd_u64(&n_meta)) return set_error("truncated header");
    if (n_tensors > size_ || n_meta > size_) return set_error("implausible counts in the header");
    for (uint64_t i = 0; i < n_meta; ++i) {
      std::string key;
      if (!rd_string(&key)) return set_error("truncated metadata");
      if (!skip_value()) return set_error(error_.empty() ? "truncated metadata" : error_);
    }
    tensors_.reserve((size_t)n_tensors);
    for (uint64_t i = 0; i < n_tensors; ++i) {
      TensorInfo t;
      uint32_t nd;
      if (!rd_string(&t.name) || !rd_u32(&nd) || nd > 8) return set_error("bad tensor info");
      t.numel = 1;
      for (uint32_t k = 0; k < nd; ++k) {
        uint64_t dim;
        if (!rd_u64(&dim)) return set_error("bad tensor info");
        if (dim > (1ull << 40) || (dim && t.numel > (1ull << 40) / dim)) return set_error("tensor too large");
        t.dims.push_back(dim);
        t.numel *= dim;
      }
      if (!rd_u32(&t.type) || !rd_u64(&t.offset)) return set_error("bad tensor info");
      if (t.type != TYPE_F32 && t.type != TYPE_F16)
        return set_error("tensor " + t.name + ": unknown dtype " + std::to_string(t.type));
      index_[t.name] = tensors_.size();
      tensors_.push_back(std::move(t));
    }
    data_start_ = (pos_ + kAlignment - 1) / kAlignment * kAlignment;
    for (const TensorInfo& t : tensors_) {
      const uint64_t bytes = t.numel * (t.type == TYPE_F32 ? 4 : 2);
      if (t.offset % (t.type == TYPE_F32 ? 4 : 2) != 0) return set_error("tensor " + t.name + ": misaligned data");
      if (data_start_ > size_ || t.offset > size_ - data_start_ || bytes > size_ - data_start_ - t.offset)
        return set_error("tensor " + t.name + ": data past the end of the file");
    }
    return true;
  }

  int fd_ = -1;
  const uint8_t* base_ = nullptr;
  size_t size_ = 0;
  uint64_t pos_ = 0;
  uint64_t data_start_ = 0;
  std::vector<TensorInfo> tensors_;
  std::unordered_map<std::string, size_t> index_;
  std::string error_;
};

}  // namespace gguf
}  // namespace noor
