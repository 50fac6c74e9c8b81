/*
 * CPU oracle: plain-C restatement of woolly's quantized transformer forward.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Each function names the reference
 * file:line it restates.  Compile with -ffp-contract=off: Rust does not fuse
 * a*b+c into an FMA, and the Q4_1 dequant (q*d + m) must round twice, as the
 * reference does, to stay bit-exact.
 */
#include "oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ */
/* f16 -> f32, exact (the `half` crate's f16::to_f32 is an exact IEEE
 * widening; dequantize.rs:307 / :366 / :574 rely on it).              */
float or_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do {
        man <<= 1;
        e++;
      } while ((man & 0x400u) == 0);
      man &= 0x3FFu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* GGMLType::block_size / type_size: crates/woolly-gguf/src/tensor_info.rs:128-177 */
size_t or_block_size(int t) {
  switch (t) {
    case 2: case 3: case 6: case 7: case 8: case 9: return 32;
    case 10: case 11: case 12: case 13: case 14: case 15:
    case 16: case 17: case 18: case 19: case 20: case 21: case 22: case 23: case 29:
      return 256;
    default: return 1;
  }
}

size_t or_type_size(int t) {
  switch (t) {
    case 0: return 4;
    case 1: case 30: return 2;
    case 28: return 8;
    case 24: return 1;
    case 25: return 2;
    case 26: return 4;
    case 27: return 8;
    case 2: return 18;
    case 3: return 20;
    case 6: return 22;
    case 7: return 24;
    case 8: return 34;
    case 9: return 36;
    case 10: return 82;
    case 11: return 110;
    case 12: return 144;
    case 13: return 176;
    case 14: return 210;
    case 15: return 292;
    case 16: return 66;
    case 17: return 74;
    case 18: return 98;
    case 19: return 50;
    case 20: return 130;
    case 21: return 110;
    case 22: return 82;
    case 23: return 136;
    case 29: return 56;
    default: return 0;
  }
}

static int type_valid(uint32_t t) { return t <= 3 || (t >= 6 && t <= 30); }
static int type_quantized(uint32_t t) {
  return !(t == 0 || t == 1 || t == 30 || t == 28 || (t >= 24 && t <= 27));
}

/* loader.rs:661-666 */
uint64_t or_align_offset(uint64_t off, uint64_t a) {
  if (a == 0) return off;
  return (off + a - 1) & ~(a - 1);
}

/* ------------------------------------------------------------------ */
/* dequantize.rs:189-205 and the per-type functions it dispatches to.  */
int or_dequantize(const uint8_t* data, size_t len, int type, size_t n, float* out) {
  size_t nb = (n + 31) / 32;
  switch (type) {
    case OR_F32: /* dequantize.rs:250-265: exact length required */
      if (len != n * 4) return OR_ERR_BUFFER_TOO_SMALL;
      memcpy(out, data, n * 4);
      return OR_OK;
    case OR_F16: /* :268-283 */
      if (len != n * 2) return OR_ERR_BUFFER_TOO_SMALL;
      for (size_t i = 0; i < n; i++) out[i] = or_half_to_float(rd16(data + 2 * i));
      return OR_OK;
    case OR_Q4_0: { /* :286-327 */
      if (len < nb * 18) return OR_ERR_BUFFER_TOO_SMALL;
      size_t o = 0;
      for (size_t b = 0; b < nb; b++) {
        const uint8_t* blk = data + b * 18;
        float d = or_half_to_float(rd16(blk));
        for (int i = 0; i < 32 && o < n; i++) {
          int q = i < 16 ? (blk[2 + i] & 0x0F) - 8 : ((blk[2 + i - 16] >> 4) & 0x0F) - 8;
          out[o++] = (float)q * d;
        }
      }
      return OR_OK;
    }
    case OR_Q4_1: { /* :337-378 */
      if (len < nb * 20) return OR_ERR_BUFFER_TOO_SMALL;
      size_t o = 0;
      for (size_t b = 0; b < nb; b++) {
        const uint8_t* blk = data + b * 20;
        float d = or_half_to_float(rd16(blk));
        float m = or_half_to_float(rd16(blk + 2));
        for (int i = 0; i < 32 && o < n; i++) {
          int q = i < 16 ? (blk[4 + i] & 0x0F) : ((blk[4 + i - 16] >> 4) & 0x0F);
          float p = (float)q * d; /* two roundings, no FMA (Rust semantics) */
          out[o++] = p + m;
        }
      }
      return OR_OK;
    }
    case OR_Q8_0: { /* :553-586 */
      if (len < nb * 34) return OR_ERR_BUFFER_TOO_SMALL;
      size_t o = 0;
      for (size_t b = 0; b < nb; b++) {
        const uint8_t* blk = data + b * 34;
        float d = or_half_to_float(rd16(blk));
        for (int i = 0; i < 32 && o < n; i++) out[o++] = (float)(int8_t)blk[2 + i] * d;
      }
      return OR_OK;
    }
    case 12: { /* Q4_K, dequantize.rs:381-462 (the scalar path the x86 build runs) */
      size_t nbk = (n + 255) / 256;
      if (len < nbk * 144) return OR_ERR_INVALID; /* InvalidTensorInfo("Q4_K data too small") */
      size_t o = 0;
      for (size_t b = 0; b < nbk; b++) {
        const uint8_t* blk = data + b * 144;
        uint8_t sc[8];
        for (int i = 0; i < 8; i++) { /* 8 six-bit scales from the first 12 bytes */
          int src = (i * 3) / 2;
          sc[i] = (i % 2 == 0) ? (uint8_t)(blk[src] & 63)
                               : (uint8_t)(((blk[src] >> 6) | ((blk[src + 1] & 15) << 2)) & 63);
        }
        float d = or_half_to_float(rd16(blk + 12));
        float dmin = or_half_to_float(rd16(blk + 14));
        const uint8_t* qs = blk + 16;
        for (int i = 0; i < 256 && o < n; i++) {
          int q = (i % 2 == 0) ? (qs[i / 2] & 0x0F) : ((qs[i / 2] >> 4) & 0x0F);
          float t = d * (float)sc[i / 32];
          t = t * (float)q;
          out[o++] = t + dmin;
        }
      }
      return OR_OK;
    }
    case 14: { /* Q6_K, dequantize.rs:465-537 */
      size_t nbk = (n + 255) / 256;
      if (len < nbk * 210) return OR_ERR_INVALID; /* InvalidTensorInfo("Q6_K data too small") */
      size_t o = 0;
      for (size_t b = 0; b < nbk; b++) {
        const uint8_t* blk = data + b * 210;
        const uint8_t *ql = blk, *qh = blk + 128, *scales = blk + 192;
        float d = or_half_to_float(rd16(blk + 208));
        for (int i = 0; i < 256 && o < n; i++) {
          int is = i / 16;
          int ql_idx = 64 * (i / 128) + 32 * ((i % 128) / 64) + 16 * ((i % 64) / 32) + (i % 16);
          int qh_idx = 32 * (i / 128) + 16 * ((i % 128) / 64) + 8 * ((i % 64) / 32) + (i % 32) / 4;
          int qh_shift = 2 * ((i % 32) % 4);
          uint8_t qh_val = qh[qh_idx];
          uint8_t q1_ext = (qh_val >> qh_shift) & 3;
          uint8_t q2_ext = qh_shift < 6 ? (uint8_t)((qh_val >> (qh_shift + 2)) & 3)
                                        : (uint8_t)(qh_idx + 1 < 64 ? (qh[qh_idx + 1] & 3) : 0);
          uint8_t q1 = (uint8_t)((ql[ql_idx] & 0x0F) | (q1_ext << 4));
          uint8_t q2 = (uint8_t)((ql[ql_idx] >> 4) | (q2_ext << 4));
          uint8_t q = i < 128 ? q1 : q2;
          float t = d * (float)scales[is];
          t = t * (float)((int8_t)q - 32);
          out[o++] = t / 64.0f;
        }
      }
      return OR_OK;
    }
    case 6: case 7: case 13: case 15: /* Q5_0/Q5_1/Q5_K/Q8_K: zero stubs (:539-551,:595-607) */
      memset(out, 0, n * sizeof(float));
      return OR_OK;
    default:
      return type_valid((uint32_t)type) ? OR_ERR_UNSUPPORTED : OR_ERR_INVALID_TYPE;
  }
}

/* quantization.rs:869-909 (dispatch), :1100-1163 (scalar Q4_0 / Q8_0) */
int or_quantized_matvec(int type, const uint8_t* blocks, const float* x, float* y, size_t m,
                        size_t k) {
  if (k % 32 != 0) return OR_ERR_INVALID;
  size_t nbr = k / 32;
  if (type == OR_Q4_0) {
    for (size_t r = 0; r < m; r++) {
      float sum = 0.0f;
      for (size_t b = 0; b < nbr; b++) {
        const uint8_t* blk = blocks + (r * nbr + b) * 18;
        float d = or_half_to_float(rd16(blk));
        const float* in = x + b * 32;
        for (int j = 0; j < 16; j++) {
          int x0 = (blk[2 + j] & 0x0F) - 8;
          int x1 = (blk[2 + j] >> 4) - 8;
          sum += ((float)x0 * d) * in[j];
          sum += ((float)x1 * d) * in[j + 16];
        }
      }
      y[r] = sum;
    }
    return OR_OK;
  }
  if (type == OR_Q8_0) {
    for (size_t r = 0; r < m; r++) {
      float sum = 0.0f;
      for (size_t b = 0; b < nbr; b++) {
        const uint8_t* blk = blocks + (r * nbr + b) * 34;
        float d = or_half_to_float(rd16(blk));
        const float* in = x + b * 32;
        for (int j = 0; j < 32; j++) sum += ((float)(int8_t)blk[2 + j] * d) * in[j];
      }
      y[r] = sum;
    }
    return OR_OK;
  }
  return OR_ERR_UNSUPPORTED; /* :905-907: Q4_1 and the rest -> UnsupportedScheme */
}

/* ------------------------------------------------------------------ */
/* GGUF parsing: format.rs:79-105, metadata.rs:86-179, tensor_info.rs:206-236,
 * loader.rs:141-199.                                                   */
typedef struct cur {
  const uint8_t* p;
  size_t n, pos;
  int err;
} cur;

static int need(cur* c, size_t k) {
  if (c->err) return 0;
  if (c->pos + k > c->n) {
    c->err = OR_ERR_TRUNCATED;
    return 0;
  }
  return 1;
}
static uint8_t g8(cur* c) { return need(c, 1) ? c->p[c->pos++] : 0; }
static uint32_t g32(cur* c) {
  if (!need(c, 4)) return 0;
  uint32_t v;
  memcpy(&v, c->p + c->pos, 4);
  c->pos += 4;
  return v;
}
static uint64_t g64(cur* c) {
  if (!need(c, 8)) return 0;
  uint64_t v;
  memcpy(&v, c->p + c->pos, 8);
  c->pos += 8;
  return v;
}
static void gskip(cur* c, uint64_t k) {
  if (k > c->n - c->pos) {
    c->err = OR_ERR_TRUNCATED;
    return;
  }
  c->pos += (size_t)k;
}

typedef struct kvval {
  uint32_t type;
  uint32_t u32;
  float f32;
  const uint8_t* str;
  uint64_t slen;
} kvval;

/* reads one metadata value of the given type (metadata.rs:86-120) */
static void read_value(cur* c, uint32_t type, kvval* v, int depth) {
  v->type = type;
  switch (type) {
    case 0: case 1: case 7: g8(c); break;
    case 2: case 3: gskip(c, 2); break;
    case 4: v->u32 = g32(c); break;
    case 5: g32(c); break;
    case 6: {
      uint32_t b = g32(c);
      memcpy(&v->f32, &b, 4);
      break;
    }
    case 8: {
      v->slen = g64(c);
      if (!need(c, (size_t)(v->slen > c->n ? c->n + 1 : v->slen))) return;
      v->str = c->p + c->pos;
      c->pos += v->slen;
      break;
    }
    case 9: {
      uint32_t at = g32(c);
      uint64_t len = g64(c);
      if (at > 12) {
        c->err = OR_ERR_INVALID;
        return;
      }
      if (depth > 4) {
        c->err = OR_ERR_INVALID;
        return;
      }
      for (uint64_t i = 0; i < len && !c->err; i++) {
        kvval tmp;
        read_value(c, at, &tmp, depth + 1);
      }
      v->slen = len;
      break;
    }
    case 10: case 11: case 12: gskip(c, 8); break;
    default: c->err = OR_ERR_INVALID; /* metadata.rs:166-167: invalid value type */
  }
}

static int key_is(const uint8_t* k, uint64_t kl, const char* s) {
  return strlen(s) == kl && memcmp(k, s, kl) == 0;
}

int or_gguf_open_mem(const uint8_t* bytes, size_t n, or_gguf** out) {
  *out = NULL;
  cur c = {bytes, n, 0, 0};
  /* header, format.rs:79-105 */
  if (n < 4) return OR_ERR_IO; /* read_exact on a short file is an Io error */
  if (memcmp(bytes, "GGUF", 4) != 0) return OR_ERR_INVALID_MAGIC;
  c.pos = 4;
  uint32_t ver = g32(&c);
  if (c.err) return OR_ERR_IO;
  if (ver < 1 || ver > 3) return OR_ERR_UNSUPPORTED_VERSION;
  uint64_t nt = g64(&c), nkv = g64(&c);
  if (c.err) return OR_ERR_IO;
  or_gguf* g = (or_gguf*)calloc(1, sizeof(or_gguf));
  g->version = ver;
  g->n_tensors = nt;
  g->n_kv = nkv;
  g->eps = 1e-5f;
  uint32_t alignment = 32;
  /* all key-value pairs are scanned; the ones the config needs are kept.
   * Typed getters (metadata.rs:195-224) only match the exact value type. */
  kvval* kvs = NULL;
  const uint8_t** keys = NULL;
  uint64_t* klens = NULL;
  if (nkv > n) { /* each pair needs at least 12 bytes */
    free(g);
    return OR_ERR_IO;
  }
  kvs = (kvval*)calloc(nkv ? nkv : 1, sizeof(kvval));
  keys = (const uint8_t**)calloc(nkv ? nkv : 1, sizeof(*keys));
  klens = (uint64_t*)calloc(nkv ? nkv : 1, sizeof(uint64_t));
  for (uint64_t i = 0; i < nkv && !c.err; i++) {
    uint64_t kl = g64(&c);
    if (kl > c.n - c.pos) {
      c.err = OR_ERR_TRUNCATED;
      break;
    }
    keys[i] = c.p + c.pos;
    klens[i] = kl;
    c.pos += kl;
    uint32_t vt = g32(&c);
    if (c.err) break;
    read_value(&c, vt, &kvs[i], 0);
  }
  if (c.err) {
    int e = c.err == OR_ERR_TRUNCATED ? OR_ERR_IO : c.err;
    free(kvs), free(keys), free(klens), free(g);
    return e;
  }
  /* general.architecture, then "{arch}.*" keys (model/loader.rs:104-156) */
  for (uint64_t i = 0; i < nkv; i++)
    if (key_is(keys[i], klens[i], "general.architecture") && kvs[i].type == 8 &&
        kvs[i].slen < sizeof(g->arch)) {
      memcpy(g->arch, kvs[i].str, kvs[i].slen);
      g->arch[kvs[i].slen] = 0;
      g->has_arch = 1;
    }
  int have[10] = {0};
  uint32_t alt_vocab = 0, alt_hidden = 0, alt_layers = 0, alt_ctx = 0;
  float alt_theta = 0, alt_eps = 0;
  int have_alt[6] = {0};
  char buf[160];
  for (uint64_t i = 0; i < nkv; i++) {
    const uint8_t* k = keys[i];
    uint64_t kl = klens[i];
    kvval* v = &kvs[i];
    if (key_is(k, kl, "general.alignment") && v->type == 4) alignment = v->u32;
    if (key_is(k, kl, "tokenizer.ggml.tokens.len") && v->type == 4) alt_vocab = v->u32, have_alt[0] = 1;
    if (key_is(k, kl, "tokenizer.ggml.context_length") && v->type == 4) alt_ctx = v->u32, have_alt[3] = 1;
    if (!g->has_arch) continue;
#define AK(suffix) (snprintf(buf, sizeof buf, "%s." suffix, g->arch), key_is(k, kl, buf))
    if (AK("vocab_size") && v->type == 4) g->vocab = v->u32, have[0] = 1;
    if (AK("embedding_length") && v->type == 4) g->hidden = v->u32, have[1] = 1;
    if (AK("embed_dim") && v->type == 4) alt_hidden = v->u32, have_alt[1] = 1;
    if (AK("block_count") && v->type == 4) g->layers = v->u32, have[2] = 1;
    if (AK("layer_count") && v->type == 4) alt_layers = v->u32, have_alt[2] = 1;
    if (AK("attention.head_count") && v->type == 4) g->heads = v->u32, have[3] = 1;
    if (AK("context_length") && v->type == 4) g->ctx = v->u32, have[4] = 1;
    if (AK("feed_forward_length") && v->type == 4) g->ff = v->u32, have[5] = 1;
    if (AK("attention.head_count_kv") && v->type == 4) g->kv_heads = v->u32, g->has_kv_heads = 1;
    if (AK("rope.freq_base") && v->type == 6) g->theta = v->f32, g->has_theta = 1;
    if (AK("attention.rope_theta") && v->type == 6) alt_theta = v->f32, have_alt[4] = 1;
    if (AK("attention.layer_norm_epsilon") && v->type == 6) g->eps = v->f32, have[6] = 1;
    if (AK("layer_norm_epsilon") && v->type == 6) alt_eps = v->f32, have_alt[5] = 1;
#undef AK
  }
  if (!have[0]) g->vocab = have_alt[0] ? alt_vocab : 32000;
  if (!have[1]) g->hidden = have_alt[1] ? alt_hidden : 4096;
  if (!have[2]) g->layers = have_alt[2] ? alt_layers : 32;
  if (!have[3]) g->heads = 32;
  if (!have[4]) g->ctx = have_alt[3] ? alt_ctx : 2048;
  if (!have[5]) g->ff = g->hidden * 4;
  if (!g->has_theta && have_alt[4]) g->theta = alt_theta, g->has_theta = 1;
  if (!have[6] && have_alt[5]) g->eps = alt_eps;
  free(kvs), free(keys), free(klens);

  /* tensor table, tensor_info.rs:206-236 */
  if (nt > n) {
    free(g);
    return OR_ERR_IO;
  }
  g->tensors = (or_tensor*)calloc(nt ? nt : 1, sizeof(or_tensor));
  for (uint64_t i = 0; i < nt && !c.err; i++) {
    or_tensor* t = &g->tensors[i];
    uint64_t nl = g64(&c);
    if (nl > c.n - c.pos) {
      c.err = OR_ERR_TRUNCATED;
      break;
    }
    size_t cp = nl < sizeof(t->name) - 1 ? (size_t)nl : sizeof(t->name) - 1;
    memcpy(t->name, c.p + c.pos, cp);
    c.pos += nl;
    t->n_dims = g32(&c);
    if (t->n_dims > 4) {
      c.err = OR_ERR_INVALID;
      break;
    }
    for (uint32_t d = 0; d < t->n_dims; d++) t->dims[d] = g64(&c);
    t->type = g32(&c);
    if (!c.err && !type_valid(t->type)) {
      c.err = OR_ERR_INVALID_TYPE;
      break;
    }
    t->offset = g64(&c);
  }
  if (c.err) {
    int e = c.err == OR_ERR_TRUNCATED ? OR_ERR_IO : c.err;
    free(g->tensors), free(g);
    return e;
  }
  g->alignment = alignment;
  g->data_start = or_align_offset(c.pos, alignment); /* loader.rs:151-164 */
  g->file = (uint8_t*)malloc(n ? n : 1);
  memcpy(g->file, bytes, n);
  g->file_size = n;
  *out = g;
  return OR_OK;
}

int or_gguf_open(const char* path, or_gguf** out) {
  FILE* f = fopen(path, "rb");
  if (!f) return OR_ERR_IO;
  fseek(f, 0, SEEK_END);
  long sz = ftell(f);
  fseek(f, 0, SEEK_SET);
  uint8_t* buf = (uint8_t*)malloc(sz > 0 ? (size_t)sz : 1);
  size_t got = sz > 0 ? fread(buf, 1, (size_t)sz, f) : 0;
  fclose(f);
  if ((long)got != sz) {
    free(buf);
    return OR_ERR_IO;
  }
  int st = or_gguf_open_mem(buf, got, out);
  free(buf);
  return st;
}

void or_gguf_close(or_gguf* g) {
  if (!g) return;
  free(g->file);
  free(g->tensors);
  free(g);
}

int or_gguf_find(const or_gguf* g, const char* name) {
  for (uint64_t i = 0; i < g->n_tensors; i++)
    if (strcmp(g->tensors[i].name, name) == 0) return (int)i;
  return -1;
}

uint64_t or_tensor_nelems(const or_tensor* t) {
  uint64_t n = 1;
  for (uint32_t d = 0; d < t->n_dims; d++) n *= t->dims[d];
  return n;
}

/* tensor_info.rs:244-255 */
uint64_t or_tensor_nbytes(const or_tensor* t) {
  uint64_t n = or_tensor_nelems(t);
  if (type_quantized(t->type)) {
    uint64_t bs = or_block_size((int)t->type), ts = or_type_size((int)t->type);
    return (n + bs - 1) / bs * ts;
  }
  return n * or_type_size((int)t->type);
}

/* loader.rs:265-274: data_start + offset, bounds-checked */
const uint8_t* or_tensor_data(const or_gguf* g, const or_tensor* t) {
  uint64_t off = g->data_start + t->offset;
  if (off + or_tensor_nbytes(t) > g->file_size) return NULL;
  return g->file + off;
}

/* ------------------------------------------------------------------ */
/* ops                                                                  */

/* tensor_utils.rs:446-480 */
void or_rms_norm(const float* x, const float* w, int rows, int d, float eps, float* y) {
  for (int r = 0; r < rows; r++) {
    const float* xr = x + (size_t)r * d;
    float ss = 0.0f;
    for (int i = 0; i < d; i++) ss += xr[i] * xr[i];
    float rms = sqrtf(ss / (float)d + eps);
    for (int i = 0; i < d; i++) {
      float nv = xr[i] / rms;
      y[(size_t)r * d + i] = nv * w[i];
    }
  }
}

/* tensor_utils.rs:512-532 (exact); simd_matmul.rs:1086-1097 (AVX2, exp(-g)~1-g);
 * simd_matmul.rs:1050-1061 (NEON, sigmoid(g)~0.5+0.5*(0.5g)).  The SIMD
 * variants only apply to full 8- (AVX2) or 4-wide (NEON) groups; tails are exact. */
void or_swiglu(const float* g, const float* u, size_t n, int mode, float* out) {
  size_t vec = mode == 1 ? 8 : (mode == 2 ? 4 : 0);
  size_t nv = vec ? n / vec * vec : 0;
  for (size_t i = 0; i < n; i++) {
    float gi = g[i], s;
    if (i < nv && mode == 1) {
      float e = 1.0f + (0.0f - gi);
      s = gi * (1.0f / (1.0f + e));
    } else if (i < nv && mode == 2) {
      float sc = gi * 0.5f;
      s = gi * (0.5f + 0.5f * sc);
    } else {
      s = gi * (1.0f / (1.0f + expf(-gi)));
    }
    out[i] = s * u[i];
  }
}

/* RoPE::apply_f32 (crates/woolly-tensor/src/ops/mod.rs:476-527), in place.
 * x is [batch, seq, heads, hd]; pairs (i, i + hd/2) rotate by pos*base^(-2i/hd). */
void or_rope_neox(float* x, const size_t* positions, int batch, int seq, int heads, int hd,
                  float base) {
  int half = hd / 2;
  float* freqs = (float*)malloc(sizeof(float) * (size_t)half);
  for (int i = 0; i < half; i++) freqs[i] = 1.0f / powf(base, 2.0f * (float)i / (float)hd);
  for (int b = 0; b < batch; b++)
    for (int s = 0; s < seq; s++) {
      float pos = (float)positions[s];
      for (int h = 0; h < heads; h++) {
        float* v = x + (((size_t)b * seq + s) * heads + h) * hd;
        for (int i = 0; i < half; i++) {
          float ang = pos * freqs[i];
          float c = cosf(ang), sn = sinf(ang);
          float x1 = v[i], x2 = v[i + half];
          v[i] = x1 * c - x2 * sn;
          v[i + half] = x1 * sn + x2 * c;
        }
      }
    }
  free(freqs);
}

static int g_threads = 0;

/* Layout-B projection, tensor_utils.rs:118-157 (matmul_simple):
 * y[s, o] = sum_k x[s, k] * W[k*N + o], summed in k order per output.
 * Blocked over (row chunk, output chunk) so the accumulators stay in L1; the
 * order of the sum for each output is unchanged (k = 0, 1, ..., K-1). */
void or_matmul_b(const float* x, int rows, int K, const float* W, int N, float* y) {
  enum { OC = 64, RC = 32 };
  int noc = (N + OC - 1) / OC, nrc = (rows + RC - 1) / RC;
#pragma omp parallel for collapse(2) schedule(dynamic) num_threads(g_threads > 0 ? g_threads : omp_get_max_threads())
  for (int rc = 0; rc < nrc; rc++)
    for (int c = 0; c < noc; c++) {
      int o0 = c * OC, on = o0 + OC < N ? OC : N - o0;
      int r0 = rc * RC, rn = r0 + RC < rows ? RC : rows - r0;
      float acc[RC][OC];
      for (int s = 0; s < rn; s++)
        for (int o = 0; o < OC; o++) acc[s][o] = 0.0f;
      for (int k = 0; k < K; k++) {
        const float* wr = W + (size_t)k * N + o0;
        if (on == OC) {
          for (int s = 0; s < rn; s++) {
            float xv = x[(size_t)(r0 + s) * K + k];
            for (int o = 0; o < OC; o++) acc[s][o] += xv * wr[o];
          }
        } else {
          for (int s = 0; s < rn; s++) {
            float xv = x[(size_t)(r0 + s) * K + k];
            for (int o = 0; o < on; o++) acc[s][o] += xv * wr[o];
          }
        }
      }
      for (int s = 0; s < rn; s++)
        memcpy(y + (size_t)(r0 + s) * N + o0, acc[s], sizeof(float) * (size_t)on);
    }
}

/* GQA attention with a KV cache: lazy_transformer.rs:360-434.
 * q [rows, H*hd]; kc/vc [past+rows, KVH*hd]; row i is at absolute position
 * past+i and attends keys 0..=past+i (window W > 0 keeps only j > pos-W). */
void or_attention(const float* q, const float* kc, const float* vc, int rows, int past,
                  int heads, int kv_heads, int hd, int window, float* out) {
  int groups = heads / kv_heads;
  int d = heads * hd, kvd = kv_heads * hd;
  int total = past + rows;
  float scale = 1.0f / sqrtf((float)hd);
  memset(out, 0, sizeof(float) * (size_t)rows * d);
#pragma omp parallel num_threads(g_threads > 0 ? g_threads : omp_get_max_threads())
  {
    float* sc = (float*)malloc(sizeof(float) * (size_t)(total > 0 ? total : 1));
#pragma omp for collapse(2) schedule(static)
    for (int pos = 0; pos < rows; pos++)
      for (int qh = 0; qh < heads; qh++) {
        int kvh = qh / groups;
        int abs = past + pos;
        int j0 = window > 0 && abs - window + 1 > 0 ? abs - window + 1 : 0;
        const float* qv = q + (size_t)pos * d + (size_t)qh * hd;
        for (int j = j0; j <= abs; j++) {
          const float* kv = kc + (size_t)j * kvd + (size_t)kvh * hd;
          float s = 0.0f;
          for (int t = 0; t < hd; t++) s += qv[t] * kv[t];
          sc[j] = s * scale;
        }
        float mx = -INFINITY;
        for (int j = j0; j <= abs; j++) mx = sc[j] > mx ? sc[j] : mx;
        float sum = 0.0f;
        for (int j = j0; j <= abs; j++) {
          sc[j] = expf(sc[j] - mx);
          sum += sc[j];
        }
        if (sum > 0.0f) {
          float inv = 1.0f / sum;
          float* o = out + (size_t)pos * d + (size_t)qh * hd;
          for (int j = j0; j <= abs; j++) {
            float wgt = sc[j] * inv;
            const float* vv = vc + (size_t)j * kvd + (size_t)kvh * hd;
            for (int t = 0; t < hd; t++) o[t] += wgt * vv[t];
          }
        }
      }
    free(sc);
  }
  (void)total;
}

/* ------------------------------------------------------------------ */
/* model                                                                */
typedef struct or_layer {
  float *attn_norm, *ffn_norm, *wq, *wk, *wv, *wo, *wg, *wu, *wd;
} or_layer;

struct or_model {
  int d, L, H, KVH, hd, kvd, ff, V;
  float eps, theta;
  or_opts opts;
  float* embd; /* [d][V] as stored (token_embd dims [d, V]) */
  float* out_norm;
  float* out_w; /* [d][V]; the tied embedding when output.weight is absent */
  int tied;
  or_layer* layers;
};

struct or_kv {
  int max_ctx, len, L, kvd;
  float** k;
  float** v;
};

static float* load_f32(const or_gguf* g, const char* name, uint64_t expect, int* st) {
  int i = or_gguf_find(g, name);
  if (i < 0) {
    *st = OR_ERR_NOT_FOUND;
    return NULL;
  }
  const or_tensor* t = &g->tensors[i];
  uint64_t n = or_tensor_nelems(t);
  if (expect && n != expect) {
    *st = OR_ERR_INVALID;
    return NULL;
  }
  const uint8_t* p = or_tensor_data(g, t);
  if (!p) {
    *st = OR_ERR_BUFFER_TOO_SMALL;
    return NULL;
  }
  float* out = (float*)malloc(sizeof(float) * (size_t)n);
  if (!out) {
    *st = OR_ERR_INVALID;
    return NULL;
  }
  *st = or_dequantize(p, (size_t)or_tensor_nbytes(t), (int)t->type, (size_t)n, out);
  if (*st) {
    free(out);
    return NULL;
  }
  return out;
}

/* ggml orientation: a [ne0 = K, ne1 = N] tensor holds N rows of K values
 * (row o, column k at o*K + k); the forward reads [K][N] (k*N + o), so
 * layout A transposes once at load.  For token_embd [d, V] this turns token
 * rows E[t*d + j] into the reference's E[j*V + t]. */
static int to_layout_b(float** p, size_t K, size_t N) {
  float* t = (float*)malloc(sizeof(float) * K * N);
  if (!t) return OR_ERR_INVALID;
  const float* s = *p;
  for (size_t o = 0; o < N; o++)
    for (size_t k = 0; k < K; k++) t[k * N + o] = s[o * K + k];
  free(*p);
  *p = t;
  return OR_OK;
}

void or_model_free(or_model* m) {
  if (!m) return;
  for (int l = 0; m->layers && l < m->L; l++) {
    or_layer* y = &m->layers[l];
    free(y->attn_norm), free(y->ffn_norm), free(y->wq), free(y->wk), free(y->wv);
    free(y->wo), free(y->wg), free(y->wu), free(y->wd);
  }
  free(m->layers);
  free(m->embd);
  free(m->out_norm);
  if (!m->tied) free(m->out_w);
  free(m);
}

/* LazyTransformer::from_gguf (lazy_transformer.rs:29-95) with every weight
 * dequantized to f32 up front, which is what the reference's dequantization
 * cache holds after preload (lazy_loader.rs:377-396). */
int or_model_load(const char* path, const or_opts* opts, or_model** out) {
  *out = NULL;
  or_gguf* g = NULL;
  int st = or_gguf_open(path, &g);
  if (st) return st;
  if (!g->has_arch) {
    or_gguf_close(g);
    return OR_ERR_INVALID; /* model/loader.rs:108-109 */
  }
  or_model* m = (or_model*)calloc(1, sizeof(or_model));
  if (opts) m->opts = *opts;
  g_threads = m->opts.threads;
  m->d = (int)g->hidden;
  m->L = (int)g->layers;
  if (m->opts.max_layers > 0 && m->opts.max_layers < m->L) m->L = m->opts.max_layers;
  m->H = (int)g->heads;
  m->hd = m->d / m->H;
  m->V = (int)g->vocab;
  m->eps = g->eps;
  m->theta = g->has_theta ? g->theta : 10000.0f;
  /* KV width from the attn_k shape, lazy_transformer.rs:284-287 */
  int ki = or_gguf_find(g, "blk.0.attn_k.weight");
  if (ki < 0 || g->tensors[ki].n_dims != 2) {
    or_gguf_close(g), free(m);
    return OR_ERR_NOT_FOUND;
  }
  m->kvd = (int)g->tensors[ki].dims[1];
  m->KVH = m->kvd / m->hd;
  int gi = or_gguf_find(g, "blk.0.ffn_gate.weight");
  if (gi < 0) {
    or_gguf_close(g), free(m);
    return OR_ERR_NOT_FOUND;
  }
  m->ff = (int)g->tensors[gi].dims[1]; /* gate_shape[1], lazy_transformer.rs:496 */
  size_t d = (size_t)m->d, kvd = (size_t)m->kvd, ff = (size_t)m->ff, V = (size_t)m->V;
  m->embd = load_f32(g, "token_embd.weight", d * V, &st);
  if (st) goto fail;
  if (m->opts.layout_a && (st = to_layout_b(&m->embd, d, V))) goto fail;
  m->out_norm = load_f32(g, "output_norm.weight", d, &st);
  if (st) goto fail;
  if (or_gguf_find(g, "output.weight") >= 0) {
    m->out_w = load_f32(g, "output.weight", d * V, &st);
    if (st) goto fail;
    if (m->opts.layout_a && (st = to_layout_b(&m->out_w, d, V))) goto fail;
  } else {
    m->out_w = m->embd;
    m->tied = 1;
  }
  m->layers = (or_layer*)calloc((size_t)m->L, sizeof(or_layer));
  for (int l = 0; l < m->L; l++) {
    char nm[128];
    or_layer* y = &m->layers[l];
#define LD(field, suffix, K, N)                                                   \
  snprintf(nm, sizeof nm, "blk.%d." suffix, l);                                   \
  y->field = load_f32(g, nm, (K) * (N), &st);                                     \
  if (st) goto fail;                                                              \
  if ((N) > 1 && m->opts.layout_a && (st = to_layout_b(&y->field, (K), (N)))) goto fail;
    LD(attn_norm, "attn_norm.weight", d, 1)
    LD(ffn_norm, "ffn_norm.weight", d, 1)
    LD(wq, "attn_q.weight", d, d)
    LD(wk, "attn_k.weight", d, kvd)
    LD(wv, "attn_v.weight", d, kvd)
    LD(wo, "attn_output.weight", d, d)
    LD(wg, "ffn_gate.weight", d, ff)
    LD(wu, "ffn_up.weight", d, ff)
    LD(wd, "ffn_down.weight", ff, d)
#undef LD
  }
  or_gguf_close(g);
  *out = m;
  return OR_OK;
fail:
  or_gguf_close(g);
  or_model_free(m);
  return st;
}

void or_model_dims(const or_model* m, int* hidden, int* layers, int* heads, int* kv_heads,
                   int* ff, int* vocab) {
  if (hidden) *hidden = m->d;
  if (layers) *layers = m->L;
  if (heads) *heads = m->H;
  if (kv_heads) *kv_heads = m->KVH;
  if (ff) *ff = m->ff;
  if (vocab) *vocab = m->V;
}

or_kv* or_kv_new(const or_model* m, int max_ctx) {
  or_kv* kv = (or_kv*)calloc(1, sizeof(or_kv));
  kv->max_ctx = max_ctx;
  kv->L = m->L;
  kv->kvd = m->kvd;
  kv->k = (float**)calloc((size_t)m->L, sizeof(float*));
  kv->v = (float**)calloc((size_t)m->L, sizeof(float*));
  for (int l = 0; l < m->L; l++) {
    kv->k[l] = (float*)calloc((size_t)max_ctx * m->kvd, sizeof(float));
    kv->v[l] = (float*)calloc((size_t)max_ctx * m->kvd, sizeof(float));
  }
  return kv;
}

void or_kv_free(or_kv* kv) {
  if (!kv) return;
  for (int l = 0; l < kv->L; l++) free(kv->k[l]), free(kv->v[l]);
  free(kv->k), free(kv->v), free(kv);
}

int or_kv_len(const or_kv* kv) { return kv->len; }

int or_kv_fill_synthetic(or_kv* kv, int len, uint64_t seed) {
  if (len > kv->max_ctx) return OR_ERR_INVALID;
  uint64_t s = seed * 0x9E3779B97F4A7C15ull + 1;
  for (int l = 0; l < kv->L; l++)
    for (size_t i = 0; i < (size_t)len * kv->kvd; i++) {
      s ^= s << 13, s ^= s >> 7, s ^= s << 17;
      kv->k[l][i] = (float)((int64_t)(s >> 40) - (1 << 23)) / (float)(1 << 23);
      s ^= s << 13, s ^= s >> 7, s ^= s << 17;
      kv->v[l][i] = (float)((int64_t)(s >> 40) - (1 << 23)) / (float)(1 << 23);
    }
  kv->len = len;
  return OR_OK;
}

/* process_layer's attention half for one session's rows (lazy_transformer.rs:131-179) */
static void attn_block(or_model* m, or_layer* y, int l, or_kv* kv, const float* xn, int rows,
                       float* h, float* q, float* kn, float* vn, float* att, float* o) {
  int d = m->d, kvd = m->kvd;
  int past = kv->len;
  or_matmul_b(xn, rows, d, y->wq, d, q);
  or_matmul_b(xn, rows, d, y->wk, kvd, kn);
  or_matmul_b(xn, rows, d, y->wv, kvd, vn);
  if (m->opts.rope == 1) { /* not on the reference forward; helper semantics only */
    size_t* pos = (size_t*)malloc(sizeof(size_t) * (size_t)rows);
    for (int i = 0; i < rows; i++) pos[i] = (size_t)(past + i);
    or_rope_neox(q, pos, 1, rows, m->H, m->hd, m->theta);
    or_rope_neox(kn, pos, 1, rows, m->KVH, m->hd, m->theta);
    free(pos);
  }
  /* KV store: cached ++ new (lazy_transformer.rs:322-349) */
  memcpy(kv->k[l] + (size_t)past * kvd, kn, sizeof(float) * (size_t)rows * kvd);
  memcpy(kv->v[l] + (size_t)past * kvd, vn, sizeof(float) * (size_t)rows * kvd);
  or_attention(q, kv->k[l], kv->v[l], rows, past, m->H, m->KVH, m->hd, m->opts.window, att);
  or_matmul_b(att, rows, d, y->wo, d, o);
  for (size_t i = 0; i < (size_t)rows * d; i++) h[i] += o[i];
}

/* the FFN half (lazy_transformer.rs:186-230, compute_swiglu_ffn :459-534) */
static void ffn_block(or_model* m, or_layer* y, const float* xn, int rows, float* h, float* gt,
                      float* up, float* o) {
  int d = m->d, ff = m->ff;
  or_matmul_b(xn, rows, d, y->wg, ff, gt);
  or_matmul_b(xn, rows, d, y->wu, ff, up);
  or_swiglu(gt, up, (size_t)rows * ff, m->opts.swiglu, gt);
  or_matmul_b(gt, rows, ff, y->wd, d, o);
  for (size_t i = 0; i < (size_t)rows * d; i++) h[i] += o[i];
}

/* Model::forward for LazyTransformer (lazy_transformer.rs:1155-1336) on the
 * KV-cache path: embedding gather (E[j*V + t], :1252-1262), layers, final
 * RMSNorm and the layout-B LM head (:1293-1316). */
int or_forward(or_model* m, or_kv* kv, const uint32_t* ids, int n, float* logits, int all_rows) {
  int d = m->d, V = m->V;
  if (n <= 0) return OR_ERR_INVALID;
  if (kv->len + n > kv->max_ctx) return OR_ERR_INVALID;
  for (int i = 0; i < n; i++)
    if (ids[i] >= (uint32_t)V) return OR_ERR_INVALID; /* tensor_utils.rs:569-576 */
  size_t nd = (size_t)n * d;
  float* h = (float*)malloc(sizeof(float) * nd);
  float* xn = (float*)malloc(sizeof(float) * nd);
  float* q = (float*)malloc(sizeof(float) * nd);
  float* kn = (float*)malloc(sizeof(float) * (size_t)n * m->kvd);
  float* vn = (float*)malloc(sizeof(float) * (size_t)n * m->kvd);
  float* att = (float*)malloc(sizeof(float) * nd);
  float* o = (float*)malloc(sizeof(float) * nd);
  float* gt = (float*)malloc(sizeof(float) * (size_t)n * m->ff);
  float* up = (float*)malloc(sizeof(float) * (size_t)n * m->ff);
  for (int i = 0; i < n; i++)
    for (int j = 0; j < d; j++) h[(size_t)i * d + j] = m->embd[(size_t)j * V + ids[i]];
  for (int l = 0; l < m->L; l++) {
    or_layer* y = &m->layers[l];
    or_rms_norm(h, y->attn_norm, n, d, m->eps, xn);
    attn_block(m, y, l, kv, xn, n, h, q, kn, vn, att, o);
    or_rms_norm(h, y->ffn_norm, n, d, m->eps, xn);
    ffn_block(m, y, xn, n, h, gt, up, o);
  }
  kv->len += n;
  int first = all_rows ? 0 : n - 1;
  int rows = n - first;
  or_rms_norm(h + (size_t)first * d, m->out_norm, rows, d, m->eps, xn);
  or_matmul_b(xn, rows, d, m->out_w, V, logits);
  free(h), free(xn), free(q), free(kn), free(vn), free(att), free(o), free(gt), free(up);
  return OR_OK;
}

/* B independent sessions, one token each, sharing each weight pass. */
int or_decode_batch(or_model* m, or_kv** kvs, int B, const uint32_t* ids, float* logits) {
  int d = m->d, V = m->V, kvd = m->kvd;
  for (int b = 0; b < B; b++) {
    if (ids[b] >= (uint32_t)V) return OR_ERR_INVALID;
    if (kvs[b]->len + 1 > kvs[b]->max_ctx) return OR_ERR_INVALID;
  }
  size_t nd = (size_t)B * d;
  float* h = (float*)malloc(sizeof(float) * nd);
  float* xn = (float*)malloc(sizeof(float) * nd);
  float* q = (float*)malloc(sizeof(float) * nd);
  float* kn = (float*)malloc(sizeof(float) * (size_t)B * kvd);
  float* vn = (float*)malloc(sizeof(float) * (size_t)B * kvd);
  float* att = (float*)malloc(sizeof(float) * nd);
  float* o = (float*)malloc(sizeof(float) * nd);
  float* gt = (float*)malloc(sizeof(float) * (size_t)B * m->ff);
  float* up = (float*)malloc(sizeof(float) * (size_t)B * m->ff);
  for (int b = 0; b < B; b++)
    for (int j = 0; j < d; j++) h[(size_t)b * d + j] = m->embd[(size_t)j * V + ids[b]];
  for (int l = 0; l < m->L; l++) {
    or_layer* y = &m->layers[l];
    or_rms_norm(h, y->attn_norm, B, d, m->eps, xn);
    or_matmul_b(xn, B, d, y->wq, d, q);
    or_matmul_b(xn, B, d, y->wk, kvd, kn);
    or_matmul_b(xn, B, d, y->wv, kvd, vn);
    for (int b = 0; b < B; b++) {
      or_kv* kv = kvs[b];
      int past = kv->len;
      if (m->opts.rope == 1) {
        size_t pos = (size_t)past;
        or_rope_neox(q + (size_t)b * d, &pos, 1, 1, m->H, m->hd, m->theta);
        or_rope_neox(kn + (size_t)b * kvd, &pos, 1, 1, m->KVH, m->hd, m->theta);
      }
      memcpy(kv->k[l] + (size_t)past * kvd, kn + (size_t)b * kvd, sizeof(float) * kvd);
      memcpy(kv->v[l] + (size_t)past * kvd, vn + (size_t)b * kvd, sizeof(float) * kvd);
      or_attention(q + (size_t)b * d, kv->k[l], kv->v[l], 1, past, m->H, m->KVH, m->hd,
                   m->opts.window, att + (size_t)b * d);
    }
    or_matmul_b(att, B, d, y->wo, d, o);
    for (size_t i = 0; i < nd; i++) h[i] += o[i];
    or_rms_norm(h, y->ffn_norm, B, d, m->eps, xn);
    ffn_block(m, y, xn, B, h, gt, up, o);
  }
  for (int b = 0; b < B; b++) kvs[b]->len += 1;
  or_rms_norm(h, m->out_norm, B, d, m->eps, xn);
  or_matmul_b(xn, B, d, m->out_w, V, logits);
  free(h), free(xn), free(q), free(kn), free(vn), free(att), free(o), free(gt), free(up);
  return OR_OK;
}
