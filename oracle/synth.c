/*
 * Seeded synthetic GGUF writer for the CPU oracle side.
 *
 * TEST INFRASTRUCTURE ONLY.  bench.py's reference arm and CPU baseline build
 * their model file with this writer so that they never load the product
 * library; tests/test_oracle.py checks that it writes files byte-identical to
 * the product's writer (wl_synth_gguf) for the same configuration.
 *
 * Tensor set and layout: the LLaMA-shape file woolly's loader reads
 * (GGUF v3, crates/woolly-gguf/src/format.rs:79-105; key/value types
 * metadata.rs:86-120; tensor table tensor_info.rs:206-236; data aligned to
 * general.alignment = 32, loader.rs:151-164), with the model keys of
 * crates/woolly-core/src/model/loader.rs:104-156 (including woolly's
 * `.attention.layer_norm_epsilon`).  Weights are N(0, 0.02) draws (norms
 * 1 + N(0, 0.02)) from one seeded stream per tensor: splitmix64 state per
 * 65536-value chunk, Box-Muller pairs.  Quantizers: the published ggml block
 * schemes (woolly's own encoders are stubs, woolly-tensor/src/quantization.rs:
 * 303-307): Q4_0 d = vmax/-8, q = min(15, (int8)(x/d + 8.5)); Q4_1
 * d = (max-min)/15, m = min, q = min(15, (int8)((x-m)/d + 0.5)); Q8_0
 * d = amax/127, q = round(x/d); d and m stored as IEEE f16 (round to nearest
 * even).  K-quants are encoded for the values woolly_gguf::dequantize reads
 * back from them (dequantize.rs:381-537; 256 values per super-block):
 * Q4_K w = d*sc[j]*q + dmin (dmin as stored: the block minimum; d*sc[j]*15
 * spans sub-block j's range above it; six-bit sc at the reference's bit
 * positions); Q6_K w = d*sc[j]*(q-32)/64 with d*sc[j]/64 = absmax_j/31 and q
 * written to the ql/qh bits the reference reads.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

static uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
  if (ax < 0x38800000u) { /* subnormal: value * 2^24, rounded to nearest even */
    float v;
    memcpy(&v, &ax, 4);
    return (uint16_t)(sign | (uint32_t)lrintf(v * 16777216.0f));
  }
  uint32_t e = (ax >> 23) - 127 + 15, man = ax & 0x7FFFFFu;
  uint32_t h = (e << 10) | (man >> 13), rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

static void put16(uint8_t* p, uint16_t v) {
  p[0] = (uint8_t)(v & 0xFF);
  p[1] = (uint8_t)(v >> 8);
}

static int clamp15(int v) { return v > 15 ? 15 : v; }

static void enc_q4_0(const float* x, uint8_t* b) {
  float amax = 0.0f, vmax = 0.0f;
  for (int j = 0; j < 32; j++)
    if (fabsf(x[j]) > amax) amax = fabsf(x[j]), vmax = x[j];
  float d = vmax / -8.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
  put16(b, f32_to_f16(d));
  for (int j = 0; j < 16; j++) {
    int lo = clamp15((int)(int8_t)(x[j] * id + 8.5f));
    int hi = clamp15((int)(int8_t)(x[j + 16] * id + 8.5f));
    b[2 + j] = (uint8_t)(lo | (hi << 4));
  }
}

static void enc_q4_1(const float* x, uint8_t* b) {
  float mn = INFINITY, mx = -INFINITY;
  for (int j = 0; j < 32; j++) {
    if (x[j] < mn) mn = x[j];
    if (x[j] > mx) mx = x[j];
  }
  float d = (mx - mn) / 15.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
  put16(b, f32_to_f16(d));
  put16(b + 2, f32_to_f16(mn));
  for (int j = 0; j < 16; j++) {
    int lo = clamp15((int)(int8_t)((x[j] - mn) * id + 0.5f));
    int hi = clamp15((int)(int8_t)((x[j + 16] - mn) * id + 0.5f));
    b[4 + j] = (uint8_t)(lo | (hi << 4));
  }
}

static void enc_q8_0(const float* x, uint8_t* b) {
  float amax = 0.0f;
  for (int j = 0; j < 32; j++)
    if (fabsf(x[j]) > amax) amax = fabsf(x[j]);
  float d = amax / 127.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
  put16(b, f32_to_f16(d));
  for (int j = 0; j < 32; j++) b[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
}

static float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 31u, man = h & 1023u, x;
  float v;
  if (e == 0) {
    v = (float)man * (1.0f / 16777216.0f);
    memcpy(&x, &v, 4);
  } else if (e == 31) {
    x = 0x7F800000u | (man << 13);
  } else {
    x = ((e + 112u) << 23) | (man << 13);
  }
  x |= sign;
  memcpy(&v, &x, 4);
  return v;
}

static void enc_q4_k(const float* x, uint8_t* b) {
  memset(b, 0, 144);
  float mn = x[0], rng[8], rmax = 0.0f;
  for (int i = 1; i < 256; i++)
    if (x[i] < mn) mn = x[i];
  uint16_t hm = f32_to_f16(mn);
  float dmin = f16_to_f32(hm);
  for (int j = 0; j < 8; j++) {
    float mx = x[32 * j];
    for (int i = 1; i < 32; i++)
      if (x[32 * j + i] > mx) mx = x[32 * j + i];
    rng[j] = mx - dmin > 0.0f ? mx - dmin : 0.0f;
    if (rng[j] > rmax) rmax = rng[j];
  }
  uint16_t hd = f32_to_f16(rmax / 945.0f);
  float d = f16_to_f32(hd);
  put16(b + 12, hd);
  put16(b + 14, hm);
  for (int j = 0; j < 8; j++) {
    int sc = d > 0.0f ? (int)(rng[j] / (15.0f * d) + 0.5f) : 0;
    if (sc > 63) sc = 63;
    int src = (j * 3) / 2;
    if (j % 2 == 0) {
      b[src] |= (uint8_t)sc;
    } else {
      b[src] |= (uint8_t)((sc & 3) << 6);
      b[src + 1] |= (uint8_t)(sc >> 2);
    }
    float step = d * (float)sc, inv = step > 0.0f ? 1.0f / step : 0.0f;
    for (int i = 32 * j; i < 32 * j + 32; i++) {
      int q = (int)((x[i] - dmin) * inv + 0.5f);
      q = q < 0 ? 0 : (q > 15 ? 15 : q);
      b[16 + i / 2] |= (uint8_t)(i % 2 == 0 ? q : q << 4);
    }
  }
}

static void set_bits(uint8_t* p, int shift, int width, int v) {
  int mask = ((1 << width) - 1) << shift;
  *p = (uint8_t)((*p & ~mask) | ((v << shift) & mask));
}

static void enc_q6_k(const float* x, uint8_t* b) {
  memset(b, 0, 210);
  float am[16], m = 0.0f;
  for (int j = 0; j < 16; j++) {
    am[j] = 0.0f;
    for (int i = 16 * j; i < 16 * j + 16; i++)
      if (fabsf(x[i]) > am[j]) am[j] = fabsf(x[i]);
    if (am[j] > m) m = am[j];
  }
  uint16_t hd = f32_to_f16(m * 64.0f / (31.0f * 255.0f));
  float d = f16_to_f32(hd);
  put16(b + 208, hd);
  uint8_t *ql = b, *qh = b + 128;
  for (int j = 0; j < 16; j++) {
    int sc = d > 0.0f ? (int)(am[j] * 64.0f / (31.0f * d) + 0.5f) : 0;
    if (sc > 255) sc = 255;
    b[192 + j] = (uint8_t)sc;
    float step = d * (float)sc / 64.0f, inv = step > 0.0f ? 1.0f / step : 0.0f;
    for (int i = 16 * j; i < 16 * j + 16; i++) {
      int q = (int)(x[i] * inv + 32.5f);
      q = q < 0 ? 0 : (q > 63 ? 63 : q);
      int ql_idx = 64 * (i / 128) + 32 * ((i % 128) / 64) + 16 * ((i % 64) / 32) + (i % 16);
      int qh_idx = 32 * (i / 128) + 16 * ((i % 128) / 64) + 8 * ((i % 64) / 32) + (i % 32) / 4;
      int sh = 2 * ((i % 32) % 4);
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

static uint64_t splitmix(uint64_t* s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

enum { CHUNK = 65536 };

/* values [c*CHUNK, c*CHUNK + n) of stream `stream` */
static void normal_chunk(uint64_t seed, uint64_t stream, uint64_t c, float mean, float sd,
                         float* out, size_t n) {
  uint64_t s = seed * 0xD1B54A32D192ED03ull ^ (stream + 1) * 0x8CB92BA72F3D8DD7ull ^
               (c + 1) * 0xABC98388FB8FAC03ull;
  for (size_t i = 0; i < n; i += 2) {
    double u1 = ((splitmix(&s) >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    double u2 = (splitmix(&s) >> 11) * (1.0 / 9007199254740992.0);
    double r = sqrt(-2.0 * log(u1)), t = 6.283185307179586 * u2;
    out[i] = (float)(mean + sd * r * cos(t));
    if (i + 1 < n) out[i + 1] = (float)(mean + sd * r * sin(t));
  }
}

typedef struct {
  FILE* f;
  int ok;
} wr;

static void wraw(wr* w, const void* p, size_t n) {
  if (w->ok && n && fwrite(p, 1, n, w->f) != n) w->ok = 0;
}
static void wu32(wr* w, uint32_t v) { wraw(w, &v, 4); }
static void wu64(wr* w, uint64_t v) { wraw(w, &v, 8); }
static void wstr(wr* w, const char* s) {
  wu64(w, strlen(s));
  wraw(w, s, strlen(s));
}
static void kv_u32(wr* w, const char* k, uint32_t v) { wstr(w, k), wu32(w, 4), wu32(w, v); }
static void kv_f32(wr* w, const char* k, float v) { wstr(w, k), wu32(w, 6), wraw(w, &v, 4); }
static void kv_str(wr* w, const char* k, const char* v) { wstr(w, k), wu32(w, 8), wstr(w, v); }
static void wpad(wr* w, uint64_t n) {
  static const uint8_t z[64];
  while (n) {
    uint64_t k = n < 64 ? n : 64;
    wraw(w, z, (size_t)k);
    n -= k;
  }
}

typedef struct {
  char name[64];
  uint64_t d0, d1; /* d1 == 0: 1-D */
  uint32_t type;
  int kind; /* 0 weight, 1 embedding (f32), 2 norm (mean 1) */
} tspec;

static int quantized(uint32_t t) {
  return t == OR_Q4_0 || t == OR_Q4_1 || t == OR_Q8_0 || t == OR_Q4_K || t == OR_Q6_K;
}
static uint64_t blk(uint32_t t) { return t == OR_Q4_K || t == OR_Q6_K ? 256 : (t == OR_F32 ? 1 : 32); }
static uint64_t nelems(const tspec* t) { return t->d1 ? t->d0 * t->d1 : t->d0; }
static uint64_t nbytes(const tspec* t) {
  return quantized(t->type) ? nelems(t) / blk(t->type) * or_type_size((int)t->type) : nelems(t) * 4;
}

int or_synth_gguf(const char* path, const or_synth_cfg* c) {
  if (!path || !c || !c->hidden || !c->layers || !c->heads || !c->kv_heads || !c->ff ||
      !c->vocab || c->hidden % c->heads || c->heads % c->kv_heads)
    return OR_ERR_INVALID;
  uint32_t wt = c->weight_type, vt = c->vd_type ? c->vd_type : wt;
  if (!(quantized(wt) || wt == OR_F32) || !(quantized(vt) || vt == OR_F32)) return OR_ERR_UNSUPPORTED;
  uint64_t d = c->hidden, kvd = d / c->heads * c->kv_heads, ff = c->ff, V = c->vocab;
  int has_out = c->output_type != 0xFFFFFFFFu;
  if (has_out && !(quantized(c->output_type) || c->output_type == OR_F32)) return OR_ERR_UNSUPPORTED;
  if (!(quantized(c->embd_type) || c->embd_type == OR_F32) || (d * V) % blk(c->embd_type)) return OR_ERR_UNSUPPORTED;
  if (d % blk(wt) || kvd % blk(wt) || ff % blk(wt) || d % blk(vt) || kvd % blk(vt) ||
      (has_out && V % blk(c->output_type)))
    return OR_ERR_INVALID;
  size_t nt = 2 + 9 * (size_t)c->layers + (has_out ? 1 : 0), i = 0;
  tspec* ts = (tspec*)calloc(nt, sizeof(tspec));
  if (!ts) return OR_ERR_IO;
#define T(nm, a, b, ty, k)                                                                    \
  (snprintf(ts[i].name, sizeof ts[i].name, "%s", nm), ts[i].d0 = a, ts[i].d1 = b, ts[i].type = ty, \
   ts[i].kind = k, i++)
  T("token_embd.weight", d, V, c->embd_type, 1);
  for (uint32_t l = 0; l < c->layers; l++) {
    static const char* names[9] = {"attn_norm", "attn_q",   "attn_k", "attn_v",  "attn_output",
                                   "ffn_norm",  "ffn_gate", "ffn_up", "ffn_down"};
    uint64_t a[9] = {d, d, d, d, d, d, d, d, ff}, b[9] = {0, d, kvd, kvd, d, 0, ff, ff, d};
    for (int j = 0; j < 9; j++) {
      char nm[64];
      snprintf(nm, sizeof nm, "blk.%u.%s.weight", l, names[j]);
      T(nm, a[j], b[j], b[j] ? (j == 3 || j == 8 ? vt : wt) : OR_F32, b[j] ? 0 : 2);
    }
  }
  T("output_norm.weight", d, 0, OR_F32, 2);
  if (has_out) T("output.weight", d, V, c->output_type, 0);
#undef T
  FILE* f = fopen(path, "wb");
  if (!f) {
    free(ts);
    return OR_ERR_IO;
  }
  wr w = {f, 1};
  wraw(&w, "GGUF", 4);
  wu32(&w, 3);
  wu64(&w, nt);
  wu64(&w, 12 + (c->sliding_window ? 1 : 0));
  kv_str(&w, "general.architecture", "llama");
  kv_str(&w, "general.name", "woolly-b200 synthetic");
  kv_u32(&w, "general.alignment", 32);
  kv_u32(&w, "llama.vocab_size", c->vocab);
  kv_u32(&w, "llama.context_length", c->context_length ? c->context_length : 4096);
  kv_u32(&w, "llama.embedding_length", c->hidden);
  kv_u32(&w, "llama.block_count", c->layers);
  kv_u32(&w, "llama.feed_forward_length", c->ff);
  kv_u32(&w, "llama.attention.head_count", c->heads);
  kv_u32(&w, "llama.attention.head_count_kv", c->kv_heads);
  kv_f32(&w, "llama.rope.freq_base", c->rope_theta > 0 ? c->rope_theta : 10000.0f);
  kv_f32(&w, "llama.attention.layer_norm_epsilon", c->norm_eps > 0 ? c->norm_eps : 1e-5f);
  if (c->sliding_window) kv_u32(&w, "llama.attention.sliding_window", c->sliding_window);
  uint64_t off = 0;
  for (i = 0; i < nt; i++) {
    wstr(&w, ts[i].name);
    wu32(&w, ts[i].d1 ? 2 : 1);
    wu64(&w, ts[i].d0);
    if (ts[i].d1) wu64(&w, ts[i].d1);
    wu32(&w, ts[i].type);
    wu64(&w, off);
    off = (off + nbytes(&ts[i]) + 31) / 32 * 32;
  }
  long pos = ftell(f);
  wpad(&w, (uint64_t)((pos + 31) / 32 * 32 - pos));
  for (i = 0; i < nt && w.ok; i++) {
    const tspec* t = &ts[i];
    uint64_t n = nelems(t), nb = nbytes(t);
    float mean = t->kind == 2 ? 1.0f : 0.0f;
    uint8_t* out = (uint8_t*)malloc((size_t)nb);
    if (!out) {
      w.ok = 0;
      break;
    }
    long nch = (long)((n + CHUNK - 1) / CHUNK);
    int qt = quantized(t->type);
    size_t tsz = qt ? or_type_size((int)t->type) : 4;
#pragma omp parallel
    {
      float* buf = (float*)malloc(sizeof(float) * CHUNK);
#pragma omp for schedule(static)
      for (long ch = 0; ch < nch; ch++) {
        uint64_t c0 = (uint64_t)ch * CHUNK;
        size_t k = n - c0 < CHUNK ? (size_t)(n - c0) : CHUNK;
        if (!qt) {
          normal_chunk(c->seed, i, (uint64_t)ch, mean, 0.02f, (float*)(out + c0 * 4), k);
          continue;
        }
        normal_chunk(c->seed, i, (uint64_t)ch, mean, 0.02f, buf, k);
        uint8_t* q = out + c0 / blk(t->type) * tsz;
        if (t->type == OR_Q4_K || t->type == OR_Q6_K) {
          for (size_t b = 0; b < k / 256; b++)
            (t->type == OR_Q4_K ? enc_q4_k : enc_q6_k)(buf + 256 * b, q + tsz * b);
          continue;
        }
        for (size_t b = 0; b < k / 32; b++) {
          if (t->type == OR_Q4_0) enc_q4_0(buf + 32 * b, q + tsz * b);
          else if (t->type == OR_Q4_1) enc_q4_1(buf + 32 * b, q + tsz * b);
          else enc_q8_0(buf + 32 * b, q + tsz * b);
        }
      }
      free(buf);
    }
    wraw(&w, out, (size_t)nb);
    free(out);
    wpad(&w, (nb + 31) / 32 * 32 - nb);
  }
  free(ts);
  int ok = w.ok;
  if (fclose(f) != 0) ok = 0;
  return ok ? OR_OK : OR_ERR_IO;
}
