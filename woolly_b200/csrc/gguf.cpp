// GGUF reader (host).  See gguf.h for the reference functions restated here.
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdlib>
#include <cstring>

#include "common.h"

namespace wl {

// GGMLType::block_size (tensor_info.rs:128-145)
size_t type_block_size(uint32_t t) {
  switch (t) {
    case 2: case 3: case 6: case 7: case 8: case 9: return 32;
    case 10: case 11: case 12: case 13: case 14: case 15: case 16: case 17: case 18:
    case 19: case 20: case 21: case 22: case 23: case 29: return 256;
    default: return 1;
  }
}

// GGMLType::type_size (tensor_info.rs:148-177)
size_t type_size(uint32_t t) {
  static const int sz[31] = {4,  2,  18, 20, 0,  0,  22, 24, 34, 36, 82,  110, 144, 176, 210, 292,
                             66, 74, 98, 50, 130, 110, 82, 136, 1,  2,  4,   8,   8,   56,  2};
  return t < 31 ? (size_t)sz[t] : 0;
}

bool type_valid(uint32_t t) { return t <= 3 || (t >= 6 && t <= 30); }

bool type_quantized(uint32_t t) {
  return !(t == 0 || t == 1 || t == 30 || t == 28 || (t >= 24 && t <= 27));
}

uint64_t GgufTensor::nelems() const {
  uint64_t n = 1;
  for (uint32_t d = 0; d < n_dims; d++) n *= dims[d];
  return n;
}

// TensorInfo::data_size (tensor_info.rs:244-255)
uint64_t GgufTensor::nbytes() const {
  uint64_t n = nelems();
  if (type_quantized(type)) {
    uint64_t bs = type_block_size(type);
    return (n + bs - 1) / bs * type_size(type);
  }
  return n * type_size(type);
}

GgufFile::~GgufFile() {
  if (map) {
    if (mapped)
      munmap(map, size);
    else
      free(map);
  }
}

const GgufTensor* GgufFile::find(const std::string& n) const {
  auto it = index.find(n);
  return it == index.end() ? nullptr : &tensors[it->second];
}

// loader.rs:265-274: absolute offset = data_start + offset, bounds-checked
const uint8_t* GgufFile::data(const GgufTensor& t) const {
  uint64_t off = data_start + t.offset;
  if (off > size || t.nbytes() > size - off) return nullptr;
  return map + off;
}

bool GgufFile::get_u32(const std::string& k, uint32_t* v) const {
  auto it = kv.find(k);
  if (it == kv.end() || it->second.type != 4) return false;
  *v = (uint32_t)it->second.u;
  return true;
}

bool GgufFile::get_f32(const std::string& k, float* v) const {
  auto it = kv.find(k);
  if (it == kv.end() || it->second.type != 6) return false;
  *v = (float)it->second.f;
  return true;
}

bool GgufFile::get_str(const std::string& k, std::string* v) const {
  auto it = kv.find(k);
  if (it == kv.end() || it->second.type != 8) return false;
  *v = it->second.s;
  return true;
}

namespace {

struct Reader {
  const uint8_t* p;
  size_t n, pos = 0;
  bool short_read = false;
  bool take(void* dst, size_t k) {
    if (short_read || k > n - pos) {
      short_read = true;
      return false;
    }
    if (dst) memcpy(dst, p + pos, k);
    pos += k;
    return true;
  }
  template <class T>
  T get() {
    T v{};
    take(&v, sizeof(T));
    return v;
  }
};

// MetadataValue::read_from (metadata.rs:86-120)
int read_value(Reader& r, uint32_t type, GgufValue* v, int depth) {
  v->type = type;
  switch (type) {
    case 0: v->u = r.get<uint8_t>(); break;
    case 1: v->i = r.get<int8_t>(); break;
    case 2: v->u = r.get<uint16_t>(); break;
    case 3: v->i = r.get<int16_t>(); break;
    case 4: v->u = r.get<uint32_t>(); break;
    case 5: v->i = r.get<int32_t>(); break;
    case 6: v->f = r.get<float>(); break;
    case 7: v->u = r.get<uint8_t>() != 0; break;
    case 8: {
      uint64_t len = r.get<uint64_t>();
      if (r.short_read || len > r.n - r.pos) {
        r.short_read = true;
        break;
      }
      v->s.assign((const char*)r.p + r.pos, (size_t)len);
      r.pos += (size_t)len;
      break;
    }
    case 9: {
      uint32_t at = r.get<uint32_t>();
      uint64_t len = r.get<uint64_t>();
      if (r.short_read) break;
      if (at > 12 || depth > 8)
        return fail(WL_ERR_INVALID_FORMAT, "Invalid metadata: Invalid array type: " +
                                               std::to_string(at));
      v->array_type = at;
      v->array_len = len;
      for (uint64_t i = 0; i < len && !r.short_read; i++) {
        GgufValue tmp;
        int st = read_value(r, at, &tmp, depth + 1);
        if (st) return st;
      }
      break;
    }
    case 10: v->u = r.get<uint64_t>(); break;
    case 11: v->i = r.get<int64_t>(); break;
    case 12: v->f = r.get<double>(); break;
    default:
      return fail(WL_ERR_INVALID_FORMAT,
                  "Invalid metadata: Invalid value type: " + std::to_string(type));
  }
  return WL_OK;
}

int parse(GgufFile* g) {
  Reader r{g->map, g->size};
  // GGUFHeader::read_from (format.rs:79-105)
  uint8_t magic[4];
  if (!r.take(magic, 4)) return fail(WL_ERR_IO, "I/O error: failed to fill whole buffer");
  if (memcmp(magic, "GGUF", 4) != 0)
    return fail(WL_ERR_INVALID_MAGIC, "Invalid GGUF magic: expected 'GGUF'");
  g->version = r.get<uint32_t>();
  if (r.short_read) return fail(WL_ERR_IO, "I/O error: failed to fill whole buffer");
  if (g->version < 1 || g->version > 3)
    return fail(WL_ERR_UNSUPPORTED_VERSION,
                "Unsupported GGUF version: " + std::to_string(g->version));
  g->tensor_count = r.get<uint64_t>();
  g->kv_count = r.get<uint64_t>();
  if (r.short_read) return fail(WL_ERR_IO, "I/O error: failed to fill whole buffer");
  // GGUFMetadata::read_from (metadata.rs:156-179)
  for (uint64_t i = 0; i < g->kv_count; i++) {
    uint64_t kl = r.get<uint64_t>();
    if (r.short_read || kl > r.n - r.pos) return fail(WL_ERR_IO, "I/O error: truncated metadata");
    std::string key((const char*)r.p + r.pos, (size_t)kl);
    r.pos += (size_t)kl;
    uint32_t vt = r.get<uint32_t>();
    GgufValue v;
    int st = read_value(r, vt, &v, 0);
    if (st) return st;
    if (r.short_read) return fail(WL_ERR_IO, "I/O error: truncated metadata");
    g->kv[key] = v;
  }
  uint32_t al;
  g->alignment = g->get_u32("general.alignment", &al) ? al : 32;
  // TensorInfo::read_from (tensor_info.rs:206-236)
  if (g->tensor_count > g->size) return fail(WL_ERR_IO, "I/O error: truncated tensor table");
  g->tensors.reserve((size_t)g->tensor_count);
  for (uint64_t i = 0; i < g->tensor_count; i++) {
    GgufTensor t;
    uint64_t nl = r.get<uint64_t>();
    if (r.short_read || nl > r.n - r.pos) return fail(WL_ERR_IO, "I/O error: truncated tensor info");
    t.name.assign((const char*)r.p + r.pos, (size_t)nl);
    r.pos += (size_t)nl;
    t.n_dims = r.get<uint32_t>();
    if (t.n_dims > 4)
      return fail(WL_ERR_INVALID_FORMAT, "Invalid tensor info: n_dims " + std::to_string(t.n_dims));
    for (uint32_t d = 0; d < t.n_dims; d++) t.dims[d] = r.get<uint64_t>();
    t.type = r.get<uint32_t>();
    if (!r.short_read && !type_valid(t.type))
      return fail(WL_ERR_INVALID_TENSOR_TYPE, "Invalid tensor type: " + std::to_string(t.type));
    t.offset = r.get<uint64_t>();
    if (r.short_read) return fail(WL_ERR_IO, "I/O error: truncated tensor info");
    g->index[t.name] = g->tensors.size();
    g->tensors.push_back(std::move(t));
  }
  uint64_t a = g->alignment;
  g->data_start = a ? (r.pos + a - 1) / a * a : r.pos;  // align_offset, loader.rs:661-666
  return WL_OK;
}

}  // namespace

int gguf_open_file(const std::string& path, GgufFile** out) {
  *out = nullptr;
  int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) return fail(WL_ERR_IO, "I/O error: cannot open " + path);
  struct stat st;
  if (fstat(fd, &st) != 0) {
    close(fd);
    return fail(WL_ERR_IO, "I/O error: cannot stat " + path);
  }
  auto* g = new GgufFile();
  g->size = (size_t)st.st_size;
  if (g->size > 0) {
    void* p = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (p == MAP_FAILED) {
      close(fd);
      delete g;
      return fail(WL_ERR_IO, "I/O error: mmap failed for " + path);
    }
    g->map = (uint8_t*)p;
    g->mapped = true;
  }
  close(fd);
  int s = parse(g);
  if (s) {
    delete g;
    return s;
  }
  *out = g;
  return WL_OK;
}

int gguf_open_bytes(const uint8_t* p, size_t n, GgufFile** out) {
  *out = nullptr;
  auto* g = new GgufFile();
  g->size = n;
  g->map = (uint8_t*)malloc(n ? n : 1);
  if (n) memcpy(g->map, p, n);
  int s = parse(g);
  if (s) {
    delete g;
    return s;
  }
  *out = g;
  return WL_OK;
}

}  // namespace wl
