// Device kernels other than the quantized GEMV: attention, norms, misc ops.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "qgemv.cuh"

namespace wl {

// Attention over a paged f16 KV cache for `rows` query rows.
struct AttnArgs {
  const float* q = nullptr;  // [rows][H*hd] f32
  int ldq = 0;
  KvPages kv{};                   // page size must be 16 tokens
  const int* row_pos = nullptr;   // [rows]
  const int* row_sess = nullptr;  // [rows]
  int rows = 0, heads = 0, kv_heads = 0, head_dim = 0;
  int window = 0;   // 0 = full causal prefix
  int nsplit = 1;
  float* part_o = nullptr;   // [rows][H][nsplit][hd]   (nsplit > 1)
  float* part_ml = nullptr;  // [rows][H][nsplit][2]
  void* out = nullptr;       // [rows][ldo]: f32, or f16 hi/lo planes when out_plane != 0
  int ldo = 0;
  size_t out_plane = 0;      // planes: offset of the lo plane (elements)
  int* err = nullptr;        // set (bit 1) if a bounded wait gave up
};
int launch_attention_paged(const AttnArgs& a, cudaStream_t st);
// Prompt rows of ONE session at consecutive positions (a prefill chunk) on
// tensor cores (mma.sync, flash-attention style); same math and outputs as
// launch_attention_paged (nsplit / part buffers unused).  Needs head_dim 64 or
// 128 and 1, 2, 4 or 8 heads per KV head (attention_prefill_ok).
bool attention_prefill_ok(int heads, int kv_heads, int head_dim);
int launch_attention_prefill(const AttnArgs& a, cudaStream_t st);

// Same math over contiguous f32 K/V [past+rows][KVH*hd] (the reference's KV
// cache layout, lazy_transformer.rs:322-434).
int launch_attention_f32(const float* q, const float* k, const float* v, int rows, int past,
                         int heads, int kv_heads, int hd, int window, float* out,
                         cudaStream_t st);

// Context splits per (KV head, row) for the paged kernel; the partial buffers
// need rows * splits <= kAttnSplitCtasPerSm * num_sms + rows.
constexpr int kAttnSplitCtasPerSm = 12;
int attention_plan_splits(int rows, int kv_heads, int max_len, int num_sms);

// y = x / sqrt(mean(x^2) + eps) * w per row; optional NeoX rope per head.
// y_mode: 0 f32, 1 f16, 2 f16 hi/lo planes (lo plane y_plane elements after hi).
int launch_rmsnorm(const float* x, const float* w, int rows, int dim, float eps, int rope,
                   const int* pos, int head_dim, float theta, void* y, int y_mode,
                   size_t y_plane, cudaStream_t st);

// Tensor-parallel variant: x[r] += sum over ranks of the pushed partial rows
// (written back to x), then the RMSNorm into f16 hi/lo planes.  rows may be 0
// (waits and re-arms the counters only).
int launch_rmsnorm_peer(float* x, const float* w, int rows, int dim, float eps, void* y,
                        size_t y_plane, const PeerReduce& pr, cudaStream_t st);

// h[r][j] = E[j*V + ids[r]] (token_embd stored [d][V], lazy_transformer.rs:1252-1262)
// token_rows: E holds one row of d values per token, h[r][j] = E[ids[r]*d + j]
// (ggml orientation, llama.cpp files)
int launch_embed(const float* E, int d, int V, const uint32_t* ids, int rows, float* h,
                 int* err_flag, cudaStream_t st, int token_rows = 0);

int launch_qkv_post(float* q, const float* k, const float* v, int rows, int H, int KVH, int hd,
                    int rope, float theta, const int* row_pos, const int* row_sess, const KvPages& kv,
                    cudaStream_t st);

int launch_swiglu(const float* g, const float* u, size_t n, float* out, cudaStream_t st);
int launch_rope(const float* x, float* out, const int* pos, float base, int batch, int seq,
                int heads, int hd, cudaStream_t st);
int launch_dequant(int type, const void* blocks, size_t n, float* out, cudaStream_t st);

// GPU next-token sampling (sample.cu); vocab <= kSampleMaxVocab
constexpr int kSampleMaxVocab = 51200;
int launch_sample(const float* logits, int rows, int V, int ld, const wl_sample_params* prm,
                  uint32_t* out, cudaStream_t st);

// dst[r][t * cols + c] = src[t][r][c]: the rank-major blocks of an all-gather
// of column shards back into whole rows
int launch_gather_cols(const float* src, int T, int rows, int cols, float* dst, cudaStream_t st);

// *err &= ~bits (stream-ordered): clears the error bits the host has reported
int launch_err_clear(int* err, int bits, cudaStream_t st);

}  // namespace wl
