#include "gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <stdexcept>

namespace mkb {

TypeSize type_size(uint32_t t) {
  switch (t) {
    case kF32:
      return {1, 4};
    case kF16:
    case kBF16:
      return {1, 2};
    case 2:  // Q4_0
      return {32, 18};
    case 3:  // Q4_1
      return {32, 20};
    case 6:  // Q5_0
      return {32, 22};
    case 7:  // Q5_1
      return {32, 24};
    case kQ8_0:
      return {32, 34};
    case 9:  // Q8_1
      return {32, 36};
    case 10:  // Q2_K
      return {256, 84};
    case 11:  // Q3_K
      return {256, 110};
    case kQ4_K:
      return {256, 144};
    case kQ5_K:
      return {256, 176};
    case kQ6_K:
      return {256, 210};
    case 15:  // Q8_K
      return {256, 292};
    case 39:  // MXFP4
      return {32, 17};
    default:
      return {0, 0};
  }
}

const char* type_name(uint32_t t) {
  switch (t) {
    case kF32:
      return "F32";
    case kF16:
      return "F16";
    case kBF16:
      return "BF16";
    case kQ8_0:
      return "Q8_0";
    case kQ4_K:
      return "Q4_K";
    case kQ5_K:
      return "Q5_K";
    case kQ6_K:
      return "Q6_K";
    default:
      return "unsupported";
  }
}

size_t row_bytes(uint32_t t, int64_t n) {
  const TypeSize s = type_size(t);
  if (s.block == 0) throw std::runtime_error("gguf: unknown ggml type " + std::to_string(t));
  if (n % s.block) throw std::runtime_error("gguf: row not a multiple of the block size");
  return static_cast<size_t>(n / s.block) * s.bytes;
}

int64_t Tensor::nelements() const {
  int64_t n = 1;
  for (int64_t d : ne) n *= d;
  return n;
}

float fp16_to_fp32(uint16_t h) {
  _Float16 f;
  std::memcpy(&f, &h, 2);
  return static_cast<float>(f);
}

uint16_t fp32_to_fp16(float f) {
  const _Float16 h = static_cast<_Float16>(f);
  uint16_t u;
  std::memcpy(&u, &h, 2);
  return u;
}

namespace {

// GGUF value type ids.
enum : uint32_t { kU8, kI8, kU16, kI16, kU32, kI32, kVF32, kBool, kStr, kArr, kU64, kI64, kF64 };

class Cursor {
 public:
  Cursor(const uint8_t* p, size_t n) : p_(p), end_(p + n), base_(p) {}
  template <typename T>
  T get() {
    need(sizeof(T));
    T v;
    std::memcpy(&v, p_, sizeof(T));
    p_ += sizeof(T);
    return v;
  }
  std::string str() {
    const auto n = get<uint64_t>();
    need(n);
    std::string s(reinterpret_cast<const char*>(p_), n);
    p_ += n;
    return s;
  }
  void skip(size_t n) {
    need(n);
    p_ += n;
  }
  size_t offset() const { return static_cast<size_t>(p_ - base_); }

 private:
  void need(size_t n) const {
    if (static_cast<size_t>(end_ - p_) < n) throw std::runtime_error("gguf: truncated header");
  }
  const uint8_t* p_;
  const uint8_t* end_;
  const uint8_t* base_;
};

bool is_int_type(uint32_t t) { return t <= kI32 || t == kU64 || t == kI64; }

int64_t read_int(Cursor& c, uint32_t t) {
  switch (t) {
    case kU8:
      return c.get<uint8_t>();
    case kI8:
      return c.get<int8_t>();
    case kU16:
      return c.get<uint16_t>();
    case kI16:
      return c.get<int16_t>();
    case kU32:
      return c.get<uint32_t>();
    case kI32:
      return c.get<int32_t>();
    case kU64:
      return static_cast<int64_t>(c.get<uint64_t>());
    case kI64:
      return c.get<int64_t>();
    default:
      throw std::runtime_error("gguf: not an integer type");
  }
}

size_t scalar_bytes(uint32_t t) {
  switch (t) {
    case kU8:
    case kI8:
    case kBool:
      return 1;
    case kU16:
    case kI16:
      return 2;
    case kU32:
    case kI32:
    case kVF32:
      return 4;
    case kU64:
    case kI64:
    case kF64:
      return 8;
    default:
      return 0;
  }
}

template <typename T>
void put(std::vector<uint8_t>& b, T v) {
  const auto* p = reinterpret_cast<const uint8_t*>(&v);
  b.insert(b.end(), p, p + sizeof(T));
}

void put_str(std::vector<uint8_t>& b, const std::string& s) {
  put<uint64_t>(b, s.size());
  b.insert(b.end(), s.begin(), s.end());
}

}  // namespace

Gguf::Gguf(const std::string& path) {
  fd_ = ::open(path.c_str(), O_RDONLY);
  if (fd_ < 0) throw std::runtime_error("cannot open " + path + ": " + std::strerror(errno));
  struct stat st {};
  if (fstat(fd_, &st) != 0) throw std::runtime_error("cannot stat " + path);
  size_ = static_cast<size_t>(st.st_size);
  void* m = mmap(nullptr, size_, PROT_READ, MAP_SHARED, fd_, 0);
  if (m == MAP_FAILED) {
    ::close(fd_);
    fd_ = -1;
    throw std::runtime_error("mmap failed: " + std::string(std::strerror(errno)));
  }
  base_ = static_cast<uint8_t*>(m);
  try {
    Cursor c(base_, size_);
    if (c.get<uint32_t>() != 0x46554747u) throw std::runtime_error(path + " is not a GGUF file");
    const auto version = c.get<uint32_t>();
    if (version < 3) throw std::runtime_error("GGUF v" + std::to_string(version) + " unsupported, need v3");
    const auto n_tensors = c.get<uint64_t>();
    const auto n_kv = c.get<uint64_t>();
    for (uint64_t i = 0; i < n_kv; ++i) {
      const std::string key = c.str();
      const auto t = c.get<uint32_t>();
      Value v;
      if (is_int_type(t)) {
        v.kind = Value::kInt;
        v.i = read_int(c, t);
      } else if (t == kVF32) {
        v.kind = Value::kFloat;
        v.f = c.get<float>();
      } else if (t == kF64) {
        v.kind = Value::kFloat;
        v.f = c.get<double>();
      } else if (t == kBool) {
        v.kind = Value::kBool;
        v.i = c.get<uint8_t>() != 0;
      } else if (t == kStr) {
        v.kind = Value::kStr;
        v.s = c.str();
      } else if (t == kArr) {
        v.kind = Value::kArr;
        const auto et = c.get<uint32_t>();
        const auto n = c.get<uint64_t>();
        v.arr_len = static_cast<int64_t>(n);
        if (et == kStr) {
          for (uint64_t j = 0; j < n; ++j) c.skip(c.get<uint64_t>());
        } else if (scalar_bytes(et)) {
          c.skip(scalar_bytes(et) * n);
        } else {
          throw std::runtime_error("gguf: nested arrays unsupported");
        }
      } else {
        throw std::runtime_error("gguf: bad value type " + std::to_string(t));
      }
      kv_[key] = std::move(v);
    }
    struct Info {
      Tensor t;
      uint64_t off;
    };
    std::vector<Info> infos;
    for (uint64_t i = 0; i < n_tensors; ++i) {
      Info in;
      in.t.name = c.str();
      const auto nd = c.get<uint32_t>();
      for (uint32_t d = 0; d < nd; ++d) in.t.ne.push_back(static_cast<int64_t>(c.get<uint64_t>()));
      in.t.type = c.get<uint32_t>();
      in.off = c.get<uint64_t>();
      infos.push_back(std::move(in));
    }
    const auto align = static_cast<size_t>(get_int("general.alignment").value_or(32));
    const size_t data_start = (c.offset() + align - 1) / align * align;
    for (auto& in : infos) {
      Tensor& t = in.t;
      t.nbytes = row_bytes(t.type, t.ne[0]) * static_cast<size_t>(t.nelements() / t.ne[0]);
      if (data_start + in.off + t.nbytes > size_) throw std::runtime_error("gguf: tensor " + t.name + " out of bounds");
      t.data = base_ + data_start + in.off;
      tensors_[t.name] = std::move(t);
    }
  } catch (...) {
    munmap(base_, size_);
    ::close(fd_);
    base_ = nullptr;
    fd_ = -1;
    throw;
  }
}

Gguf::~Gguf() {
  if (base_) munmap(base_, size_);
  if (fd_ >= 0) ::close(fd_);
}

std::optional<int64_t> Gguf::get_int(const std::string& key) const {
  auto it = kv_.find(key);
  if (it == kv_.end()) return std::nullopt;
  if (it->second.kind == Value::kInt || it->second.kind == Value::kBool) return it->second.i;
  return std::nullopt;
}

std::optional<double> Gguf::get_float(const std::string& key) const {
  auto it = kv_.find(key);
  if (it == kv_.end()) return std::nullopt;
  if (it->second.kind == Value::kFloat) return it->second.f;
  if (it->second.kind == Value::kInt) return static_cast<double>(it->second.i);
  return std::nullopt;
}

std::optional<std::string> Gguf::get_str(const std::string& key) const {
  auto it = kv_.find(key);
  if (it == kv_.end() || it->second.kind != Value::kStr) return std::nullopt;
  return it->second.s;
}

int64_t Gguf::array_len(const std::string& key) const {
  auto it = kv_.find(key);
  if (it == kv_.end() || it->second.kind != Value::kArr) return -1;
  return it->second.arr_len;
}

const Tensor* Gguf::tensor(const std::string& name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}

// ---- writer ----

void GgufWriter::add_str(const std::string& key, const std::string& v) {
  put_str(head_, key);
  put<uint32_t>(head_, kStr);
  put_str(head_, v);
  ++n_kv_;
}

void GgufWriter::add_u32(const std::string& key, uint32_t v) {
  put_str(head_, key);
  put<uint32_t>(head_, kU32);
  put<uint32_t>(head_, v);
  ++n_kv_;
}

void GgufWriter::add_f32(const std::string& key, float v) {
  put_str(head_, key);
  put<uint32_t>(head_, kVF32);
  put<float>(head_, v);
  ++n_kv_;
}

void GgufWriter::add_str_array(const std::string& key, const std::vector<std::string>& v) {
  put_str(head_, key);
  put<uint32_t>(head_, kArr);
  put<uint32_t>(head_, kStr);
  put<uint64_t>(head_, v.size());
  for (const auto& s : v) put_str(head_, s);
  ++n_kv_;
}

int GgufWriter::add_tensor(const std::string& name, uint32_t type, const std::vector<int64_t>& ne) {
  Info in;
  in.name = name;
  in.type = type;
  in.ne = ne;
  int64_t n = 1;
  for (int64_t d : ne) n *= d;
  in.nbytes = row_bytes(type, ne[0]) * static_cast<size_t>(n / ne[0]);
  in.offset = 0;
  infos_.push_back(in);
  return static_cast<int>(infos_.size()) - 1;
}

void GgufWriter::open(const std::string& path) {
  constexpr size_t kAlign = 32;
  std::vector<uint8_t> hdr;
  put<uint32_t>(hdr, 0x46554747u);
  put<uint32_t>(hdr, 3);
  put<uint64_t>(hdr, infos_.size());
  put<uint64_t>(hdr, n_kv_ + 1);
  hdr.insert(hdr.end(), head_.begin(), head_.end());
  put_str(hdr, "general.alignment");
  put<uint32_t>(hdr, kU32);
  put<uint32_t>(hdr, static_cast<uint32_t>(kAlign));
  size_t off = 0;
  for (auto& in : infos_) {
    in.offset = off;
    off += (in.nbytes + kAlign - 1) / kAlign * kAlign;
    put_str(hdr, in.name);
    put<uint32_t>(hdr, static_cast<uint32_t>(in.ne.size()));
    for (int64_t d : in.ne) put<uint64_t>(hdr, static_cast<uint64_t>(d));
    put<uint32_t>(hdr, in.type);
    put<uint64_t>(hdr, in.offset);
  }
  data_start_ = (hdr.size() + kAlign - 1) / kAlign * kAlign;
  map_size_ = data_start_ + off;
  fd_ = ::open(path.c_str(), O_RDWR | O_CREAT | O_TRUNC, 0644);
  if (fd_ < 0) throw std::runtime_error("cannot create " + path + ": " + std::strerror(errno));
  if (ftruncate(fd_, static_cast<off_t>(map_size_)) != 0) throw std::runtime_error("ftruncate failed: " + path);
  void* m = mmap(nullptr, map_size_, PROT_READ | PROT_WRITE, MAP_SHARED, fd_, 0);
  if (m == MAP_FAILED) throw std::runtime_error("mmap failed: " + std::string(std::strerror(errno)));
  map_ = static_cast<uint8_t*>(m);
  std::memcpy(map_, hdr.data(), hdr.size());
  std::memset(map_ + hdr.size(), 0, data_start_ - hdr.size());
}

uint8_t* GgufWriter::data(int i) { return map_ + data_start_ + infos_[static_cast<size_t>(i)].offset; }

void GgufWriter::close() {
  if (map_) {
    msync(map_, map_size_, MS_SYNC);
    munmap(map_, map_size_);
    map_ = nullptr;
  }
  if (fd_ >= 0) {
    ::close(fd_);
    fd_ = -1;
  }
}

GgufWriter::~GgufWriter() { close(); }

}  // namespace mkb
