// GGUF v3 container, host side: a read-only mapped view (GgufReader) and a streaming writer (GgufWriter).
//
// Format (GGUF v3, little-endian; the ggml project's gguf.md):
//   u32 magic "GGUF" | u32 version | u64 tensor_count | u64 metadata_kv_count
//   metadata_kv_count x { string key | u32 value_type | value }
//   tensor_count x { string name | u32 n_dims | n_dims x u64 ne | u32 ggml_type | u64 offset }
//   padding to general.alignment (default 32) | tensor data (offsets relative to here, each aligned)
// where string = u64 length + bytes, and an array value = u32 element type + u64 count + elements.
// The reader keeps what the verify path needs: every metadata scalar and string, array element counts, and a
// directory of tensor views into the mapping. malkin reads the same files (gguf.cpp:205-249); both sides must
// agree on the bytes, not on the parser.
#pragma once
#include <cstddef>
#include <cstdint>
#include <optional>
#include <string>
#include <string_view>
#include <unordered_map>
#include <variant>
#include <vector>

namespace mkb {

// ggml tensor type ids (format constants, gguf.h:12-29).
enum GgmlType : uint32_t {
  kF32 = 0,
  kF16 = 1,
  kQ8_0 = 8,
  kQ4_K = 12,
  kQ5_K = 13,
  kQ6_K = 14,
  kBF16 = 30,
};

// Elements per block and bytes per block of a ggml type; block 0 = unknown type.
struct TypeSize {
  int64_t block;
  size_t bytes;
};
TypeSize type_size(uint32_t t);
const char* type_name(uint32_t t);
// Bytes of n elements of type t; throws if the type is unknown or n is not a multiple of its block.
size_t row_bytes(uint32_t t, int64_t n);

// One tensor of a mapped file: shape (ne[0] contiguous), type and its bytes inside the mapping.
struct TensorView {
  std::string name;
  uint32_t type = 0;
  std::vector<int64_t> ne;
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
  int64_t nelements() const;
  int64_t cols() const { return ne.empty() ? 0 : ne[0]; }
  int64_t rows() const { return ne.empty() ? 0 : nelements() / ne[0]; }
};

class GgufReader {
 public:
  // Maps `path` read-only and decodes its header; throws std::runtime_error("gguf: <path>: ...") on any
  // malformed or truncated header, unknown tensor type or tensor outside the file.
  explicit GgufReader(const std::string& path);
  ~GgufReader();
  GgufReader(const GgufReader&) = delete;
  GgufReader& operator=(const GgufReader&) = delete;

  // Metadata lookups; std::nullopt when the key is absent or holds another kind of value (booleans read as 0/1
  // integers, integers also read as reals).
  std::optional<int64_t> meta_int(std::string_view key) const;
  std::optional<double> meta_real(std::string_view key) const;
  std::optional<std::string> meta_text(std::string_view key) const;
  // Element count of an array-valued key, or -1.
  int64_t meta_count(std::string_view key) const;

  const TensorView* find(std::string_view name) const;
  const std::vector<TensorView>& directory() const { return dir_; }
  uint32_t version() const { return version_; }
  size_t alignment() const { return alignment_; }

 private:
  struct ArrayInfo {
    uint32_t elem_type;
    int64_t count;
  };
  using MetaValue = std::variant<int64_t, double, bool, std::string, ArrayInfo>;

  void decode(const std::string& path);

  const uint8_t* map_ = nullptr;
  size_t map_len_ = 0;
  uint32_t version_ = 0;
  size_t alignment_ = 32;
  std::unordered_map<std::string, MetaValue> meta_;
  std::vector<TensorView> dir_;
  std::unordered_map<std::string_view, size_t> index_;  // views into dir_[i].name
};

// Streaming GGUF writer: metadata and tensor infos first, then the data region, which callers fill in place
// through a writable mapping of the file (so multi-GB models are generated without a second copy).
class GgufWriter {
 public:
  void add_str(const std::string& key, const std::string& v);
  void add_u32(const std::string& key, uint32_t v);
  void add_f32(const std::string& key, float v);
  void add_str_array(const std::string& key, const std::vector<std::string>& v);
  // Declares a tensor; returns its index. ne[0] is the contiguous dimension.
  int add_tensor(const std::string& name, uint32_t type, const std::vector<int64_t>& ne);
  // Creates the file, writes header + infos, sizes the data region, maps it writable.
  void open(const std::string& path);
  // Writable pointer to tensor i's bytes (valid between open and close).
  uint8_t* data(int i);
  size_t nbytes(int i) const { return infos_[i].nbytes; }
  void close();
  ~GgufWriter();

 private:
  struct Info {
    std::string name;
    uint32_t type;
    std::vector<int64_t> ne;
    size_t nbytes, offset;
  };
  std::vector<uint8_t> head_;  // serialized key/values
  uint64_t n_kv_ = 0;
  std::vector<Info> infos_;
  int fd_ = -1;
  uint8_t* map_ = nullptr;
  size_t map_size_ = 0, data_start_ = 0;
};

// fp16 <-> fp32 (IEEE binary16, round to nearest even).
float fp16_to_fp32(uint16_t h);
uint16_t fp32_to_fp16(float f);

}  // namespace mkb
