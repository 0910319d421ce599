#include "gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdio>
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

// GGUF metadata value types (format constants).
enum MetaType : uint32_t {
  kMetaU8 = 0,
  kMetaI8,
  kMetaU16,
  kMetaI16,
  kMetaU32,
  kMetaI32,
  kMetaF32,
  kMetaBool,
  kMetaString,
  kMetaArray,
  kMetaU64,
  kMetaI64,
  kMetaF64,
  kMetaTypeCount
};

// Per metadata type: fixed byte width (0: variable length), and whether it is an integer / a signed one.
struct MetaTypeInfo {
  uint8_t width;
  bool integer;
  bool is_signed;
};
constexpr MetaTypeInfo kMetaTypes[kMetaTypeCount] = {
    {1, true, false}, {1, true, true},   {2, true, false},  {2, true, true}, {4, true, false},
    {4, true, true},  {4, false, false}, {1, false, false}, {0, false, false}, {0, false, false},
    {8, true, false}, {8, true, true},   {8, false, false},
};

constexpr uint32_t kGgufMagic = 0x46554747u;  // "GGUF" read as a little-endian u32
constexpr uint32_t kMaxDims = 4;

// Bounds-checked little-endian decoding of the header bytes. Each read names the field it reads, so a truncated
// or corrupt file reports that field and the byte offset where decoding stopped.
class HeaderDecoder {
 public:
  HeaderDecoder(const uint8_t* bytes, size_t len, const std::string& path) : bytes_(bytes), len_(len), path_(path) {}

  [[noreturn]] void fail(const std::string& msg) const {
    throw std::runtime_error("gguf: " + path_ + ": " + msg + " (header byte " + std::to_string(pos_) + ")");
  }
  size_t pos() const { return pos_; }
  size_t left() const { return len_ - pos_; }

  const uint8_t* take(uint64_t n, const char* what) {
    if (n > left()) fail(std::string(what) + " runs past the end of the file");
    const uint8_t* p = bytes_ + pos_;
    pos_ += static_cast<size_t>(n);
    return p;
  }
  uint32_t u32(const char* what) { return static_cast<uint32_t>(unsigned_of(4, what)); }
  uint64_t u64(const char* what) { return unsigned_of(8, what); }
  std::string_view text(const char* what) {
    const uint64_t n = u64(what);
    return {reinterpret_cast<const char*>(take(n, what)), static_cast<size_t>(n)};
  }
  // An integer metadata value of type t, widened to int64 (u64 values above INT64_MAX are rejected).
  int64_t integer(uint32_t t, const char* what) {
    const MetaTypeInfo& info = kMetaTypes[t];
    const uint64_t raw = unsigned_of(info.width, what);
    if (info.is_signed && info.width < 8) {
      const int shift = 64 - 8 * info.width;
      return static_cast<int64_t>(raw << shift) >> shift;
    }
    if (!info.is_signed && raw > static_cast<uint64_t>(INT64_MAX)) fail(std::string(what) + " exceeds int64");
    return static_cast<int64_t>(raw);
  }

 private:
  uint64_t unsigned_of(int width, const char* what) {
    uint64_t v = 0;
    std::memcpy(&v, take(static_cast<uint64_t>(width), what), static_cast<size_t>(width));  // little-endian host
    return v;
  }
  const uint8_t* bytes_;
  size_t len_;
  size_t pos_ = 0;
  const std::string& path_;
};

struct CloseOnExit {
  int fd;
  ~CloseOnExit() {
    if (fd >= 0) ::close(fd);
  }
};

}  // namespace

int64_t TensorView::nelements() const {
  int64_t n = 1;
  for (int64_t d : ne) n *= d;
  return n;
}

GgufReader::GgufReader(const std::string& path) {
  CloseOnExit file{::open(path.c_str(), O_RDONLY | O_CLOEXEC)};
  if (file.fd < 0) throw std::runtime_error("gguf: " + path + ": open: " + std::strerror(errno));
  struct stat st {};
  if (fstat(file.fd, &st) != 0) throw std::runtime_error("gguf: " + path + ": stat: " + std::strerror(errno));
  if (!S_ISREG(st.st_mode)) throw std::runtime_error("gguf: " + path + ": not a regular file");
  map_len_ = static_cast<size_t>(st.st_size);
  if (map_len_ < 24) throw std::runtime_error("gguf: " + path + ": " + std::to_string(map_len_) +
                                              " bytes, shorter than a GGUF header");
  void* m = mmap(nullptr, map_len_, PROT_READ, MAP_PRIVATE, file.fd, 0);
  if (m == MAP_FAILED) throw std::runtime_error("gguf: " + path + ": mmap: " + std::strerror(errno));
  map_ = static_cast<const uint8_t*>(m);  // the mapping outlives the descriptor
  try {
    decode(path);
  } catch (...) {
    munmap(const_cast<uint8_t*>(map_), map_len_);
    map_ = nullptr;
    throw;
  }
}

GgufReader::~GgufReader() {
  if (map_) munmap(const_cast<uint8_t*>(map_), map_len_);
}

void GgufReader::decode(const std::string& path) {
  HeaderDecoder d(map_, map_len_, path);
  const uint32_t magic = d.u32("magic");
  if (magic != kGgufMagic) {
    char hex[16];
    std::snprintf(hex, sizeof hex, "0x%08x", magic);
    d.fail(std::string("not a GGUF file (magic ") + hex + ")");
  }
  version_ = d.u32("version");
  if (version_ != 3) d.fail("GGUF version " + std::to_string(version_) + "; this reader handles version 3");
  const uint64_t n_tensors = d.u64("tensor count");
  const uint64_t n_meta = d.u64("metadata count");
  // every metadata entry takes at least 13 bytes (key length, type, 1-byte value), every tensor info 28
  if (n_meta > d.left() / 13 || n_tensors > d.left() / 28) d.fail("entry counts exceed the file size");

  meta_.reserve(static_cast<size_t>(n_meta));
  for (uint64_t i = 0; i < n_meta; ++i) {
    const std::string key(d.text("metadata key"));
    const uint32_t t = d.u32("metadata value type");
    if (t >= kMetaTypeCount) d.fail("metadata " + key + ": unknown value type " + std::to_string(t));
    MetaValue v;
    if (kMetaTypes[t].integer) {
      v = d.integer(t, "metadata integer");
    } else if (t == kMetaF32) {
      float f;
      std::memcpy(&f, d.take(4, "metadata f32"), 4);
      v = static_cast<double>(f);
    } else if (t == kMetaF64) {
      double f;
      std::memcpy(&f, d.take(8, "metadata f64"), 8);
      v = f;
    } else if (t == kMetaBool) {
      v = *d.take(1, "metadata bool") != 0;
    } else if (t == kMetaString) {
      v = std::string(d.text("metadata string"));
    } else {  // array: element type, count, elements (skipped; only the count is kept)
      const uint32_t et = d.u32("array element type");
      const uint64_t count = d.u64("array length");
      if (et >= kMetaTypeCount || et == kMetaArray) d.fail("metadata " + key + ": unsupported array element type");
      if (et == kMetaString) {
        for (uint64_t j = 0; j < count; ++j) d.text("array string");
      } else {
        const uint64_t w = kMetaTypes[et].width;
        if (count > d.left() / w) d.fail("metadata " + key + ": array runs past the end of the file");
        d.take(count * w, "array data");
      }
      v = ArrayInfo{et, static_cast<int64_t>(count)};
    }
    meta_.insert_or_assign(key, std::move(v));
  }

  if (const auto a = meta_int("general.alignment")) {
    if (*a <= 0 || (*a & (*a - 1)) || *a > (1 << 20)) d.fail("general.alignment " + std::to_string(*a) + " is not a power of two");
    alignment_ = static_cast<size_t>(*a);
  }

  std::vector<uint64_t> rel_off(static_cast<size_t>(n_tensors));
  dir_.resize(static_cast<size_t>(n_tensors));
  for (uint64_t i = 0; i < n_tensors; ++i) {
    TensorView& t = dir_[static_cast<size_t>(i)];
    t.name = std::string(d.text("tensor name"));
    const uint32_t nd = d.u32("tensor rank");
    if (nd == 0 || nd > kMaxDims) d.fail("tensor " + t.name + ": rank " + std::to_string(nd) + " outside 1..4");
    int64_t elems = 1;
    for (uint32_t k = 0; k < nd; ++k) {
      const uint64_t e = d.u64("tensor dimension");
      if (e == 0 || e > (uint64_t{1} << 40) || static_cast<uint64_t>(elems) > (uint64_t{1} << 50) / e)
        d.fail("tensor " + t.name + ": dimension " + std::to_string(e) + " out of range");
      elems *= static_cast<int64_t>(e);
      t.ne.push_back(static_cast<int64_t>(e));
    }
    t.type = d.u32("tensor type");
    const TypeSize ts = type_size(t.type);
    if (ts.block == 0) d.fail("tensor " + t.name + ": unknown ggml type " + std::to_string(t.type));
    if (t.ne[0] % ts.block)
      d.fail("tensor " + t.name + ": row of " + std::to_string(t.ne[0]) + " values is not whole " + type_name(t.type) +
             " blocks");
    t.nbytes = static_cast<size_t>(elems / ts.block) * ts.bytes;
    rel_off[static_cast<size_t>(i)] = d.u64("tensor data offset");
  }

  const size_t data_begin = (d.pos() + alignment_ - 1) / alignment_ * alignment_;
  for (size_t i = 0; i < dir_.size(); ++i) {
    TensorView& t = dir_[i];
    const uint64_t off = rel_off[i];
    if (off % alignment_) d.fail("tensor " + t.name + ": data offset " + std::to_string(off) + " not aligned");
    if (data_begin > map_len_ || off > map_len_ - data_begin || t.nbytes > map_len_ - data_begin - off)
      d.fail("tensor " + t.name + ": data lies outside the file");
    t.data = map_ + data_begin + off;
  }
  index_.reserve(dir_.size());
  for (size_t i = 0; i < dir_.size(); ++i)
    if (!index_.emplace(std::string_view(dir_[i].name), i).second) d.fail("tensor " + dir_[i].name + " appears twice");
}

std::optional<int64_t> GgufReader::meta_int(std::string_view key) const {
  const auto it = meta_.find(std::string(key));
  if (it == meta_.end()) return std::nullopt;
  if (const auto* i = std::get_if<int64_t>(&it->second)) return *i;
  if (const auto* b = std::get_if<bool>(&it->second)) return *b ? 1 : 0;
  return std::nullopt;
}

std::optional<double> GgufReader::meta_real(std::string_view key) const {
  const auto it = meta_.find(std::string(key));
  if (it == meta_.end()) return std::nullopt;
  if (const auto* f = std::get_if<double>(&it->second)) return *f;
  if (const auto* i = std::get_if<int64_t>(&it->second)) return static_cast<double>(*i);
  return std::nullopt;
}

std::optional<std::string> GgufReader::meta_text(std::string_view key) const {
  const auto it = meta_.find(std::string(key));
  if (it == meta_.end()) return std::nullopt;
  if (const auto* s = std::get_if<std::string>(&it->second)) return *s;
  return std::nullopt;
}

int64_t GgufReader::meta_count(std::string_view key) const {
  const auto it = meta_.find(std::string(key));
  if (it == meta_.end()) return -1;
  if (const auto* a = std::get_if<ArrayInfo>(&it->second)) return a->count;
  return -1;
}

const TensorView* GgufReader::find(std::string_view name) const {
  const auto it = index_.find(name);
  return it == index_.end() ? nullptr : &dir_[it->second];
}

// ---- writer ----

namespace {

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

void GgufWriter::add_str(const std::string& key, const std::string& v) {
  put_str(head_, key);
  put<uint32_t>(head_, kMetaString);
  put_str(head_, v);
  ++n_kv_;
}

void GgufWriter::add_u32(const std::string& key, uint32_t v) {
  put_str(head_, key);
  put<uint32_t>(head_, kMetaU32);
  put<uint32_t>(head_, v);
  ++n_kv_;
}

void GgufWriter::add_f32(const std::string& key, float v) {
  put_str(head_, key);
  put<uint32_t>(head_, kMetaF32);
  put<float>(head_, v);
  ++n_kv_;
}

void GgufWriter::add_str_array(const std::string& key, const std::vector<std::string>& v) {
  put_str(head_, key);
  put<uint32_t>(head_, kMetaArray);
  put<uint32_t>(head_, kMetaString);
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
  put<uint32_t>(hdr, kMetaU32);
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
