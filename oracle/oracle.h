/*
 * CPU oracle for the quantized transformer forward of woolly.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference's
 * CPU algorithm, used by tests/ as the parity checker, by the smoke() entry
 * point, and by bench.py's cpu_baseline / --impl reference legs as the timed
 * CPU baseline.  Nothing in the product (woolly_b200/) links or calls it.
 *
 * The reference is Rust (crates/woolly-gguf, woolly-tensor, woolly-core) and
 * cannot be compiled in this image (no cargo/rustc, no vendored crates), so
 * there is no oracle/_ref build.  Parity is pinned by the reference's own
 * known-answer tests (dequant KATs, GGUF builder layout, align table, 2x2
 * matmul) which tests/test_oracle.py replays against this file.  The model
 * forward has no golden vector in the reference; it is pinned only by this
 * restatement.
 */
#ifndef WOOLLY_ORACLE_H
#define WOOLLY_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids: crates/woolly-gguf/src/tensor_info.rs:15-60 */
enum { OR_F32 = 0, OR_F16 = 1, OR_Q4_0 = 2, OR_Q4_1 = 3, OR_Q8_0 = 8, OR_Q4_K = 12, OR_Q6_K = 14 };

/* status codes mirror woolly_gguf::Error kinds (crates/woolly-gguf/src/error.rs) */
enum {
  OR_OK = 0,
  OR_ERR_IO = 1,
  OR_ERR_INVALID_MAGIC = 2,
  OR_ERR_UNSUPPORTED_VERSION = 3,
  OR_ERR_TRUNCATED = 4,
  OR_ERR_INVALID_TYPE = 5,
  OR_ERR_BUFFER_TOO_SMALL = 6,
  OR_ERR_NOT_FOUND = 7,
  OR_ERR_INVALID = 8,
  OR_ERR_UNSUPPORTED = 9,
};

float or_half_to_float(uint16_t h);
size_t or_block_size(int type);
size_t or_type_size(int type);
uint64_t or_align_offset(uint64_t off, uint64_t align);

/* woolly_gguf::dequantize (crates/woolly-gguf/src/dequantize.rs:189-205) */
int or_dequantize(const uint8_t* data, size_t len, int type, size_t n, float* out);

/* woolly_tensor quantization::simd::quantized_matvec, scalar path
 * (crates/woolly-tensor/src/quantization.rs:869-909, 1100-1163):
 * layout A, y[r] = sum_k W[r*k + kk] * x[kk]; Q4_0 and Q8_0 only. */
int or_quantized_matvec(int type, const uint8_t* blocks, const float* x, float* y,
                        size_t m, size_t k);

/* ---- GGUF (format.rs, metadata.rs, tensor_info.rs, loader.rs) ---- */
typedef struct or_tensor {
  char name[256];
  uint32_t n_dims;
  uint64_t dims[4];
  uint32_t type;
  uint64_t offset;
} or_tensor;

typedef struct or_gguf {
  uint8_t* file;
  size_t file_size;
  uint32_t version;
  uint64_t n_tensors, n_kv;
  uint32_t alignment;
  uint64_t data_start;
  or_tensor* tensors;
  /* metadata picked up for the model config (model/loader.rs:104-156) */
  char arch[64];
  int has_arch;
  uint32_t vocab, hidden, layers, heads, ctx, ff;
  int has_kv_heads;
  uint32_t kv_heads;
  float eps;
  float theta;
  int has_theta;
} or_gguf;

int or_gguf_open(const char* path, or_gguf** out);
int or_gguf_open_mem(const uint8_t* bytes, size_t n, or_gguf** out);
void or_gguf_close(or_gguf* g);
int or_gguf_find(const or_gguf* g, const char* name);
uint64_t or_tensor_nelems(const or_tensor* t);
uint64_t or_tensor_nbytes(const or_tensor* t);
const uint8_t* or_tensor_data(const or_gguf* g, const or_tensor* t);

/* ---- model forward (model/lazy_transformer.rs) ---- */
typedef struct or_opts {
  int rope;        /* 0 off (reference forward), 1 NeoX half-split */
  int window;      /* 0 = full causal prefix; W > 0: keys j in (i-W, i] */
  int swiglu;      /* 0 exact, 1 AVX2 approximation, 2 NEON approximation */
  int threads;     /* OpenMP threads, <=0: library default */
  int max_layers;  /* 0 = all layers; >0 loads only the first N (baseline sampling) */
  int layout_a;    /* 0: the reference's reading of every 2-D weight as [ne0][ne1]
                      (layout B); 1: ggml's, ne1 rows of ne0 (llama.cpp files) */
} or_opts;

typedef struct or_model or_model;
typedef struct or_kv or_kv;

int or_model_load(const char* path, const or_opts* opts, or_model** out);
void or_model_free(or_model* m);
void or_model_dims(const or_model* m, int* hidden, int* layers, int* heads, int* kv_heads,
                   int* ff, int* vocab);
or_kv* or_kv_new(const or_model* m, int max_ctx);
void or_kv_free(or_kv* kv);
int or_kv_len(const or_kv* kv);
/* Fill the cache with deterministic synthetic values up to len (baseline timing only). */
int or_kv_fill_synthetic(or_kv* kv, int len, uint64_t seed);

/* forward n tokens appended after the cached prefix; logits for every row
 * (all_rows=1, n*V floats) or just the last row (V floats). */
int or_forward(or_model* m, or_kv* kv, const uint32_t* ids, int n, float* logits, int all_rows);
/* one decode step for B independent sessions (batched over the weights) */
int or_decode_batch(or_model* m, or_kv** kvs, int B, const uint32_t* ids, float* logits);

/* ---- individual ops (for op-level parity) ---- */
void or_rms_norm(const float* x, const float* w, int rows, int d, float eps, float* y);
void or_swiglu(const float* g, const float* u, size_t n, int mode, float* out);
void or_rope_neox(float* x, const size_t* positions, int batch, int seq, int heads, int hd,
                  float base);
void or_matmul_b(const float* x, int rows, int K, const float* W, int N, float* y);
void or_attention(const float* q, const float* kc, const float* vc, int rows, int past,
                  int heads, int kv_heads, int hd, int window, float* out);


/* ---- seeded synthetic GGUF writer (synth.c; byte-identical to the
 * product's wl_synth_gguf for the same configuration) ---- */
typedef struct or_synth_cfg {
  uint32_t hidden, layers, heads, kv_heads, ff, vocab, context_length;
  uint32_t weight_type;    /* OR_Q4_0 / OR_Q4_1 / OR_Q8_0 / OR_Q4_K / OR_Q6_K / OR_F32 */
  uint32_t output_type;    /* 0xFFFFFFFF: tied (no output.weight) */
  uint32_t sliding_window; /* 0 = none */
  float rope_theta, norm_eps;
  uint64_t seed;
  uint32_t vd_type;        /* 0 = weight_type; else the type of attn_v and ffn_down */
  uint32_t embd_type;      /* type of token_embd.weight (OR_F32 = 0 by default) */
} or_synth_cfg;
int or_synth_gguf(const char* path, const or_synth_cfg* cfg);

#ifdef __cplusplus
}
#endif
#endif
