// GGUF v1-v3 reader over a read-only mmap.  Restates woolly-gguf's parser
// (format.rs:79-105, metadata.rs:86-179, tensor_info.rs:206-255,
// loader.rs:141-199) so that the same files load with the same errors.
#pragma once
#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace wl {

struct GgufValue {
  uint32_t type = 0;  // MetadataValueType (metadata.rs:13-44)
  uint64_t u = 0;     // unsigned / bool payload
  int64_t i = 0;      // signed payload
  double f = 0;       // float payload
  std::string s;      // string payload
  uint32_t array_type = 0;
  uint64_t array_len = 0;
};

struct GgufTensor {
  std::string name;
  uint32_t n_dims = 0;
  uint64_t dims[4] = {1, 1, 1, 1};
  uint32_t type = 0;
  uint64_t offset = 0;
  uint64_t nelems() const;
  uint64_t nbytes() const;
};

struct GgufFile {
  ~GgufFile();
  uint8_t* map = nullptr;  // mmap'd file or owned copy
  size_t size = 0;
  bool mapped = false;
  uint32_t version = 0;
  uint64_t tensor_count = 0, kv_count = 0;
  uint32_t alignment = 32;
  uint64_t data_start = 0;
  std::map<std::string, GgufValue> kv;
  std::vector<GgufTensor> tensors;
  std::map<std::string, size_t> index;

  const GgufTensor* find(const std::string& n) const;
  const uint8_t* data(const GgufTensor& t) const;  // nullptr if out of bounds
  bool get_u32(const std::string& k, uint32_t* v) const;
  bool get_f32(const std::string& k, float* v) const;
  bool get_str(const std::string& k, std::string* v) const;
};

// returns WL_OK or a wl_status; on failure the error message is set
int gguf_open_file(const std::string& path, GgufFile** out);
int gguf_open_bytes(const uint8_t* p, size_t n, GgufFile** out);

size_t type_block_size(uint32_t t);
size_t type_size(uint32_t t);
bool type_valid(uint32_t t);
bool type_quantized(uint32_t t);

}  // namespace wl
