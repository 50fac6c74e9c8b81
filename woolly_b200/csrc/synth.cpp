// Seeded synthetic GGUF writer and GGUF block quantizers (host).
//
// woolly ships no quantizer (Q4_0Quantizer::quantize returns Err,
// woolly-tensor/src/quantization.rs:303-307), so the block encoders below
// implement the published ggml block schemes from the format definition:
//   Q4_0: d = v_absmax / -8, q = clamp(trunc(x/d + 8.5), 0, 15)
//   Q4_1: d = (max - min) / 15, m = min, q = clamp(trunc((x - m)/d + 0.5), 0, 15)
//   Q8_0: d = absmax / 127, q = round(x / d)
// (K-quant encoders below, for the reference's own reading of those blocks)
// with d (and m) stored as IEEE f16.  The file layout follows the GGUF v3
// container that woolly-gguf reads (and its MockGGUFBuilder writes,
// woolly-gguf/tests/load_model.rs:51-144), with every tensor offset aligned
// to general.alignment = 32.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "common.h"
#include "gguf.h"

namespace wl {

uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to infinity
  if (ax < 0x38800000u) {                                     // f16 subnormal range
    float v;
    memcpy(&v, &ax, 4);
    return (uint16_t)(sign | (uint32_t)lrintf(v * 16777216.0f));
  }
  uint32_t e = (ax >> 23) - 127 + 15;
  uint32_t man = ax & 0x7FFFFFu;
  uint32_t h = (e << 10) | (man >> 13);
  uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

static void put16(uint8_t* p, uint16_t v) {
  p[0] = (uint8_t)(v & 0xFF);
  p[1] = (uint8_t)(v >> 8);
}

static void quant_q4_0(const float* x, uint8_t* b) {
  float amax = 0.0f, vmax = 0.0f;
  for (int j = 0; j < 32; j++)
    if (fabsf(x[j]) > amax) amax = fabsf(x[j]), vmax = x[j];
  float d = vmax / -8.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  put16(b, f32_to_f16(d));
  for (int j = 0; j < 16; j++) {
    int lo = (int)(int8_t)(x[j] * id + 8.5f);
    int hi = (int)(int8_t)(x[j + 16] * id + 8.5f);
    lo = lo > 15 ? 15 : lo;
    hi = hi > 15 ? 15 : hi;
    b[2 + j] = (uint8_t)(lo | (hi << 4));
  }
}

static void quant_q4_1(const float* x, uint8_t* b) {
  float mn = INFINITY, mx = -INFINITY;
  for (int j = 0; j < 32; j++) mn = x[j] < mn ? x[j] : mn, mx = x[j] > mx ? x[j] : mx;
  float d = (mx - mn) / 15.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  put16(b, f32_to_f16(d));
  put16(b + 2, f32_to_f16(mn));
  for (int j = 0; j < 16; j++) {
    int lo = (int)(int8_t)((x[j] - mn) * id + 0.5f);
    int hi = (int)(int8_t)((x[j + 16] - mn) * id + 0.5f);
    lo = lo > 15 ? 15 : lo;
    hi = hi > 15 ? 15 : hi;
    b[4 + j] = (uint8_t)(lo | (hi << 4));
  }
}

static void quant_q8_0(const float* x, uint8_t* b) {
  float amax = 0.0f;
  for (int j = 0; j < 32; j++) amax = fabsf(x[j]) > amax ? fabsf(x[j]) : amax;
  float d = amax / 127.0f;
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  put16(b, f32_to_f16(d));
  for (int j = 0; j < 32; j++) b[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
}

static float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 31u, man = h & 1023u;
  float v;
  if (e == 0) {
    v = (float)man * (1.0f / 16777216.0f);  // subnormal: man * 2^-24 (exact)
  } else if (e == 31) {
    uint32_t x = 0x7F800000u | (man << 13);
    memcpy(&v, &x, 4);
  } else {
    uint32_t x = ((e + 112u) << 23) | (man << 13);
    memcpy(&v, &x, 4);
  }
  uint32_t x;
  memcpy(&x, &v, 4);
  x |= sign;
  memcpy(&v, &x, 4);
  return v;
}

// K-quant encoders for the values woolly_gguf::dequantize reads back
// (dequantize.rs:381-537), 256 values per super-block:
//   Q4_K: w = d*sc[j]*q + dmin (dmin added as stored), so dmin = the block
//     minimum, d*sc[j]*15 spans sub-block j's range above it, q = round((x -
//     dmin)/(d*sc[j])); sc[j] six bits at the reference's bit positions.
//   Q6_K: w = d*sc[j]*(q - 32)/64 with unsigned sc per 16 values, d*sc[j]/64
//     = absmax_j/31, q = round(x/step) + 32 written to the ql/qh bits the
//     reference reads (values whose bits it reads from one place share them).
static void quant_q4_k(const float* x, uint8_t* b) {
  memset(b, 0, 144);
  float mn = x[0];
  for (int i = 1; i < 256; i++) mn = x[i] < mn ? x[i] : mn;
  const uint16_t hm = f32_to_f16(mn);
  const float dmin = f16_to_f32(hm);
  float rng[8], rmax = 0.0f;
  for (int j = 0; j < 8; j++) {
    float mx = x[32 * j];
    for (int i = 1; i < 32; i++) mx = x[32 * j + i] > mx ? x[32 * j + i] : mx;
    rng[j] = mx - dmin > 0.0f ? mx - dmin : 0.0f;
    rmax = rng[j] > rmax ? rng[j] : rmax;
  }
  const uint16_t hd = f32_to_f16(rmax / 945.0f);
  const float d = f16_to_f32(hd);
  put16(b + 12, hd);
  put16(b + 14, hm);
  for (int j = 0; j < 8; j++) {
    int sc = d > 0.0f ? (int)(rng[j] / (15.0f * d) + 0.5f) : 0;
    sc = sc > 63 ? 63 : sc;
    const int src = (j * 3) / 2;
    if (j % 2 == 0) {
      b[src] = (uint8_t)(b[src] | sc);
    } else {
      b[src] = (uint8_t)(b[src] | ((sc & 3) << 6));
      b[src + 1] = (uint8_t)(b[src + 1] | (sc >> 2));
    }
    const float step = d * (float)sc, inv = step > 0.0f ? 1.0f / step : 0.0f;
    for (int i = 32 * j; i < 32 * j + 32; i++) {
      int q = (int)((x[i] - dmin) * inv + 0.5f);
      q = q < 0 ? 0 : q > 15 ? 15 : q;
      b[16 + i / 2] = (uint8_t)(b[16 + i / 2] | (i % 2 == 0 ? q : q << 4));
    }
  }
}

static void set_bits(uint8_t* p, int shift, int width, int v) {
  const int mask = ((1 << width) - 1) << shift;
  *p = (uint8_t)((*p & ~mask) | ((v << shift) & mask));
}

static void quant_q6_k(const float* x, uint8_t* b) {
  memset(b, 0, 210);
  float am[16], m = 0.0f;
  for (int j = 0; j < 16; j++) {
    am[j] = 0.0f;
    for (int i = 16 * j; i < 16 * j + 16; i++) am[j] = fabsf(x[i]) > am[j] ? fabsf(x[i]) : am[j];
    m = am[j] > m ? am[j] : m;
  }
  const uint16_t hd = f32_to_f16(m * 64.0f / (31.0f * 255.0f));
  const float d = f16_to_f32(hd);
  put16(b + 208, hd);
  uint8_t *ql = b, *qh = b + 128;
  for (int j = 0; j < 16; j++) {
    int sc = d > 0.0f ? (int)(am[j] * 64.0f / (31.0f * d) + 0.5f) : 0;
    sc = sc > 255 ? 255 : sc;
    b[192 + j] = (uint8_t)sc;
    const float step = d * (float)sc / 64.0f, inv = step > 0.0f ? 1.0f / step : 0.0f;
    for (int i = 16 * j; i < 16 * j + 16; i++) {
      int q = (int)(x[i] * inv + 32.5f);
      q = q < 0 ? 0 : q > 63 ? 63 : q;
      const int ql_idx = 64 * (i / 128) + 32 * ((i % 128) / 64) + 16 * ((i % 64) / 32) + (i % 16);
      const int qh_idx = 32 * (i / 128) + 16 * ((i % 128) / 64) + 8 * ((i % 64) / 32) + (i % 32) / 4;
      const int sh = 2 * ((i % 32) % 4);
      if (i < 128) {
        set_bits(ql + ql_idx, 0, 4, q & 15);
        set_bits(qh + qh_idx, sh, 2, q >> 4);
      } else {
        set_bits(ql + ql_idx, 4, 4, q & 15);
        if (sh < 6)
          set_bits(qh + qh_idx, sh + 2, 2, q >> 4);
        else if (qh_idx + 1 < 64)
          set_bits(qh + qh_idx + 1, 0, 2, q >> 4);
      }
    }
  }
}

static int quantize_blocks(uint32_t type, const float* src, size_t n, uint8_t* dst) {
  if (type == WL_Q4_K || type == WL_Q6_K) {
    const size_t ts = type_size(type);
    for (size_t i = 0; i < n / 256; i++)
      (type == WL_Q4_K ? quant_q4_k : quant_q6_k)(src + 256 * i, dst + ts * i);
    return WL_OK;
  }
  size_t nb = n / 32, ts = type_size(type);
  for (size_t i = 0; i < nb; i++) {
    if (type == WL_Q4_0)
      quant_q4_0(src + 32 * i, dst + ts * i);
    else if (type == WL_Q4_1)
      quant_q4_1(src + 32 * i, dst + ts * i);
    else if (type == WL_Q8_0)
      quant_q8_0(src + 32 * i, dst + ts * i);
    else
      return WL_ERR_UNSUPPORTED;
  }
  return WL_OK;
}

// ---- seeded normal stream: splitmix64 per 64K-element chunk, Box-Muller ----
static inline uint64_t splitmix(uint64_t& s) {
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static const size_t kChunk = 65536;

static void normal_chunk(uint64_t seed, uint64_t stream, uint64_t chunk, float mean, float sd,
                         float* out, size_t n) {
  uint64_t s = seed * 0xD1B54A32D192ED03ull ^ (stream + 1) * 0x8CB92BA72F3D8DD7ull ^
               (chunk + 1) * 0xABC98388FB8FAC03ull;
  for (size_t i = 0; i < n; i += 2) {
    double u1 = ((splitmix(s) >> 11) + 1.0) * (1.0 / 9007199254740992.0);  // (0, 1]
    double u2 = (splitmix(s) >> 11) * (1.0 / 9007199254740992.0);
    double r = sqrt(-2.0 * log(u1));
    double t = 6.283185307179586 * u2;
    out[i] = (float)(mean + sd * r * cos(t));
    if (i + 1 < n) out[i + 1] = (float)(mean + sd * r * sin(t));
  }
}

template <class F>
static void parallel_chunks(size_t nchunks, F fn) {
  unsigned nt = std::thread::hardware_concurrency();
  if (nt == 0) nt = 4;
  if (nt > 64) nt = 64;
  if (nchunks < nt) nt = (unsigned)nchunks;
  if (nt <= 1) {
    for (size_t c = 0; c < nchunks; c++) fn(c);
    return;
  }
  std::vector<std::thread> th;
  for (unsigned t = 0; t < nt; t++)
    th.emplace_back([&, t] {
      for (size_t c = t; c < nchunks; c += nt) fn(c);
    });
  for (auto& x : th) x.join();
}

static void gen_normal(uint64_t seed, uint64_t stream, float mean, float sd, size_t n, float* out) {
  size_t nch = (n + kChunk - 1) / kChunk;
  parallel_chunks(nch, [&](size_t c) {
    size_t o = c * kChunk, k = n - o < kChunk ? n - o : kChunk;
    normal_chunk(seed, stream, c, mean, sd, out + o, k);
  });
}

// ---- GGUF writer ----
struct W {
  FILE* f;
  bool ok = true;
  void raw(const void* p, size_t n) {
    if (ok && n && fwrite(p, 1, n, f) != n) ok = false;
  }
  void u32(uint32_t v) { raw(&v, 4); }
  void u64(uint64_t v) { raw(&v, 8); }
  void f32(float v) { raw(&v, 4); }
  void str(const std::string& s) {
    u64(s.size());
    raw(s.data(), s.size());
  }
  void kv_u32(const std::string& k, uint32_t v) { str(k), u32(4), u32(v); }
  void kv_f32(const std::string& k, float v) { str(k), u32(6), f32(v); }
  void kv_str(const std::string& k, const std::string& v) { str(k), u32(8), str(v); }
  void pad(uint64_t n) {
    static const uint8_t z[64] = {0};
    while (n) {
      uint64_t k = n < 64 ? n : 64;
      raw(z, (size_t)k);
      n -= k;
    }
  }
};

struct TSpec {
  std::string name;
  uint64_t d0, d1;  // dims [d0, d1]; d1 == 0 -> 1-D
  uint32_t type;
  int kind;  // 0 projection N(0,.02), 1 embedding N(0,.02) f32, 2 norm 1+N(0,.02)
  uint64_t nelems() const { return d1 ? d0 * d1 : d0; }
  uint64_t nbytes() const {
    uint64_t n = nelems();
    return type_quantized(type) ? n / type_block_size(type) * type_size(type) : n * type_size(type);
  }
};

int synth_gguf(const char* path, const wl_synth_config* c) {
  if (!path || !c) return fail(WL_ERR_INVALID_ARGUMENT, "synth_gguf: null argument");
  if (!c->hidden || !c->layers || !c->heads || !c->kv_heads || !c->ff || !c->vocab ||
      c->hidden % c->heads || c->heads % c->kv_heads)
    return fail(WL_ERR_INVALID_ARGUMENT, "synth_gguf: inconsistent shape");
  auto ok_type = [](uint32_t t) {
    return t == WL_Q4_0 || t == WL_Q4_1 || t == WL_Q8_0 || t == WL_Q4_K || t == WL_Q6_K || t == WL_F32;
  };
  uint32_t wt = c->weight_type, vt = c->vd_type ? c->vd_type : wt;
  if (!ok_type(wt) || !ok_type(vt))
    return fail(WL_ERR_UNSUPPORTED, "synth_gguf: weight type must be F32/Q4_0/Q4_1/Q8_0/Q4_K/Q6_K");
  uint64_t d = c->hidden, hd = d / c->heads, kvd = hd * c->kv_heads, ff = c->ff, V = c->vocab;
  // quantization blocks run along the output columns (the second dim)
  auto blk = [](uint32_t t) -> uint64_t { return t == WL_F32 ? 1 : type_block_size(t); };
  if (d % blk(wt) || kvd % blk(wt) || ff % blk(wt) || d % blk(vt) || kvd % blk(vt) ||
      (c->output_type != 0xFFFFFFFFu && ok_type(c->output_type) && V % blk(c->output_type)))
    return fail(WL_ERR_INVALID_ARGUMENT,
                "synth_gguf: quantized output dims must be multiples of the block size (32; 256 for K-quants)");
  const uint32_t et = c->embd_type;
  if (!ok_type(et) || (et != WL_F32 && (d * V) % blk(et)))
    return fail(WL_ERR_UNSUPPORTED, "synth_gguf: bad token_embd type");
  std::vector<TSpec> ts;
  ts.push_back({"token_embd.weight", d, V, et, 1});
  for (uint32_t l = 0; l < c->layers; l++) {
    std::string p = "blk." + std::to_string(l) + ".";
    ts.push_back({p + "attn_norm.weight", d, 0, WL_F32, 2});
    ts.push_back({p + "attn_q.weight", d, d, wt, 0});
    ts.push_back({p + "attn_k.weight", d, kvd, wt, 0});
    ts.push_back({p + "attn_v.weight", d, kvd, vt, 0});
    ts.push_back({p + "attn_output.weight", d, d, wt, 0});
    ts.push_back({p + "ffn_norm.weight", d, 0, WL_F32, 2});
    ts.push_back({p + "ffn_gate.weight", d, ff, wt, 0});
    ts.push_back({p + "ffn_up.weight", d, ff, wt, 0});
    ts.push_back({p + "ffn_down.weight", ff, d, vt, 0});
  }
  ts.push_back({"output_norm.weight", d, 0, WL_F32, 2});
  if (c->output_type != 0xFFFFFFFFu) {
    uint32_t ot = c->output_type;
    if (!ok_type(ot))
      return fail(WL_ERR_UNSUPPORTED, "synth_gguf: output type must be F32/Q4_0/Q4_1/Q8_0/Q4_K/Q6_K");
    ts.push_back({"output.weight", d, V, ot, 0});
  }
  FILE* f = fopen(path, "wb");
  if (!f) return fail(WL_ERR_IO, std::string("I/O error: cannot create ") + path);
  W w{f};
  const std::string arch = "llama";
  uint32_t nkv = 12 + (c->sliding_window ? 1 : 0);
  w.raw("GGUF", 4);
  w.u32(3);
  w.u64(ts.size());
  w.u64(nkv);
  w.kv_str("general.architecture", arch);
  w.kv_str("general.name", "woolly-b200 synthetic");
  w.kv_u32("general.alignment", 32);
  w.kv_u32(arch + ".vocab_size", c->vocab);
  w.kv_u32(arch + ".context_length", c->context_length ? c->context_length : 4096);
  w.kv_u32(arch + ".embedding_length", c->hidden);
  w.kv_u32(arch + ".block_count", c->layers);
  w.kv_u32(arch + ".feed_forward_length", c->ff);
  w.kv_u32(arch + ".attention.head_count", c->heads);
  w.kv_u32(arch + ".attention.head_count_kv", c->kv_heads);
  w.kv_f32(arch + ".rope.freq_base", c->rope_theta > 0 ? c->rope_theta : 10000.0f);
  // woolly reads this key (model/loader.rs:144-146), not the standard *_rms_* one
  w.kv_f32(arch + ".attention.layer_norm_epsilon", c->norm_eps > 0 ? c->norm_eps : 1e-5f);
  if (c->sliding_window) w.kv_u32(arch + ".attention.sliding_window", c->sliding_window);
  uint64_t off = 0;
  for (auto& t : ts) {
    w.str(t.name);
    w.u32(t.d1 ? 2 : 1);
    w.u64(t.d0);
    if (t.d1) w.u64(t.d1);
    w.u32(t.type);
    w.u64(off);
    off = (off + t.nbytes() + 31) / 32 * 32;
  }
  long pos = ftell(f);
  w.pad((uint64_t)((pos + 31) / 32 * 32 - pos));
  std::vector<float> buf;
  std::vector<uint8_t> q;
  for (size_t i = 0; i < ts.size() && w.ok; i++) {
    auto& t = ts[i];
    uint64_t n = t.nelems();
    buf.resize((size_t)n);
    float mean = t.kind == 2 ? 1.0f : 0.0f;
    gen_normal(c->seed, i, mean, 0.02f, (size_t)n, buf.data());
    if (type_quantized(t.type)) {
      q.resize((size_t)t.nbytes());
      size_t nch = (size_t)((n + kChunk - 1) / kChunk);  // kChunk is a multiple of 32
      int err = WL_OK;
      parallel_chunks(nch, [&](size_t ch) {
        size_t o = ch * kChunk, k = n - o < kChunk ? (size_t)(n - o) : kChunk;
        int s = quantize_blocks(t.type, buf.data() + o, k,
                                q.data() + o / type_block_size(t.type) * type_size(t.type));
        if (s) err = s;
      });
      if (err) {
        fclose(f);
        return fail(err, "synth_gguf: quantization failed");
      }
      w.raw(q.data(), q.size());
    } else {
      w.raw(buf.data(), (size_t)n * 4);
    }
    uint64_t nb = t.nbytes();
    w.pad((nb + 31) / 32 * 32 - nb);
  }
  bool ok = w.ok;
  if (fclose(f) != 0) ok = false;
  if (!ok) return fail(WL_ERR_IO, std::string("I/O error: short write to ") + path);
  return WL_OK;
}

}  // namespace wl

extern "C" int wl_synth_gguf(const char* path, const wl_synth_config* cfg) {
  return wl::synth_gguf(path, cfg);
}

extern "C" int wl_quantize(int type, const float* src, size_t n, void* dst) {
  if (!src || !dst || n % 32) return wl::fail(WL_ERR_INVALID_ARGUMENT, "wl_quantize: n % 32 != 0");
  if ((type == WL_Q4_K || type == WL_Q6_K) && n % 256)
    return wl::fail(WL_ERR_INVALID_ARGUMENT, "wl_quantize: K-quants need n % 256 == 0");
  int s = wl::quantize_blocks((uint32_t)type, src, n, (uint8_t*)dst);
  if (s) return wl::fail(s, "wl_quantize: unsupported type " + std::to_string(type));
  return WL_OK;
}

extern "C" int wl_synth_normal(uint64_t seed, uint64_t stream, float mean, float sd, size_t n,
                               float* out) {
  if (!out && n) return wl::fail(WL_ERR_INVALID_ARGUMENT, "wl_synth_normal: null output");
  wl::gen_normal(seed, stream, mean, sd, n, out);
  return WL_OK;
}
