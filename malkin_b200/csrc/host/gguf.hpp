// GGUF v3 reader and writer (host). The reader covers what malkin's GgufFile reads (gguf.cpp:205-249):
// magic, version >= 3, key/value metadata of every GGUF value type, tensor infos, data aligned to
// general.alignment (default 32). The writer emits files that reader (and malkin's) accept.
#pragma once
#include <cstddef>
#include <cstdint>
#include <map>
#include <optional>
#include <string>
#include <vector>

namespace mkb {

enum GgmlType : uint32_t {
  kF32 = 0,
  kF16 = 1,
  kQ8_0 = 8,
  kQ4_K = 12,
  kQ5_K = 13,
  kQ6_K = 14,
  kBF16 = 30,
};

// Elements per block and bytes per block of a ggml type (gguf.cpp:60-95); block 0 = unknown type.
struct TypeSize {
  int64_t block;
  size_t bytes;
};
TypeSize type_size(uint32_t t);
const char* type_name(uint32_t t);
// Bytes of n elements of type t; throws if n is not a multiple of the block.
size_t row_bytes(uint32_t t, int64_t n);

struct Tensor {
  std::string name;
  uint32_t type = 0;
  std::vector<int64_t> ne;  // ne[0] contiguous
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
  int64_t nelements() const;
  int64_t cols() const { return ne.empty() ? 0 : ne[0]; }
  int64_t rows() const { return ne.empty() ? 0 : nelements() / ne[0]; }
};

class Gguf {
 public:
  explicit Gguf(const std::string& path);
  ~Gguf();
  Gguf(const Gguf&) = delete;
  Gguf& operator=(const Gguf&) = delete;

  std::optional<int64_t> get_int(const std::string& key) const;
  std::optional<double> get_float(const std::string& key) const;
  std::optional<std::string> get_str(const std::string& key) const;
  // Entries of an array-valued key (any element type), or -1 if absent.
  int64_t array_len(const std::string& key) const;
  const Tensor* tensor(const std::string& name) const;
  const std::map<std::string, Tensor>& tensors() const { return tensors_; }

 private:
  struct Value {
    enum Kind { kInt, kFloat, kBool, kStr, kArr } kind = kInt;
    int64_t i = 0;
    double f = 0;
    std::string s;
    int64_t arr_len = 0;
  };
  int fd_ = -1;
  uint8_t* base_ = nullptr;
  size_t size_ = 0;
  std::map<std::string, Value> kv_;
  std::map<std::string, Tensor> tensors_;
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
