// Quantized GEMV / skinny GEMM (decode path) — shared declarations.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace wl {

// Epilogue kinds for the layout-B GEMV (applied once the full K sum is known).
enum EpiKind : int {
  EPI_F32 = 0,     // y[b][col] = v                      (f32)
  EPI_ADD = 1,     // y[b][col] += v                     (residual, f32)
  EPI_F16 = 2,     // y[b][col] = half(v)
  EPI_QKV = 3,     // seg0 -> q f32 (+rope), seg1 -> K pages f16 (+rope), seg2 -> V pages
  EPI_SWIGLU = 4,  // seg0 = gate, seg1 = up: y[b][col] = half(silu(g) * u)
};

// Paged KV cache addressing for one layer.
struct KvPages {
  __half* k;              // [n_pages][page][kvd]
  __half* v;
  const int* page_table;  // [n_sessions_max][max_pages]
  int max_pages;          // row stride of page_table
  int page;               // tokens per page
  int kvd;
};

struct Epilogue {
  int kind = EPI_F32;
  void* y = nullptr;  // output base (kind-dependent)
  int ldy = 0;        // row stride of y (elements)
  // QKV / rope
  int rope = 0;
  int head_dim = 0;
  float theta = 10000.f;
  const int* row_pos = nullptr;   // [B] absolute position of each row
  const int* row_sess = nullptr;  // [B] session slot of each row (page table row)
  KvPages kv{};
};

struct GemvSeg {
  const uint8_t* W = nullptr;
  int N = 0;         // columns (layout B) or rows (layout A)
  int pitch = 0;     // bytes per matrix row
  int groups = 0;    // column groups (tiles) in this segment
  int group_base = 0;
};

struct GemvArgs {
  int type = 2;  // WL_Q4_0 / WL_Q4_1 / WL_Q8_0
  int nseg = 1;
  GemvSeg seg[3];
  int K = 0;            // reduction length
  int B = 0;            // rows of x (<= 32 per launch)
  const __half* x = nullptr;
  int ldx = 0;
  int ksplit = 1;
  int kchunk = 0;       // rows of K per split (multiple of 16)
  float* ws = nullptr;  // [ksplit][B][total_cols] partial sums
  unsigned* counters = nullptr;
  int total_cols = 0;
  Epilogue epi;
};

// Host launchers (stream-ordered).  Return a wl_status.
int launch_qgemv_b(const GemvArgs& a, cudaStream_t st);
int launch_qgemv_a(const GemvArgs& a, cudaStream_t st);
// generic (any alignment) fallback, f32 math, plain loads; EPI_F32/EPI_ADD only
int launch_qgemv_generic(int type, int layout, const uint8_t* W, int K, int N, int pitch,
                         const __half* x, int ldx, int B, float* y, int ldy, bool add,
                         cudaStream_t st);
bool qgemv_b_fast_ok(int type, int K, int N, int pitch, const void* W);
bool qgemv_a_fast_ok(int type, int K, int N, int pitch, const void* W);
// scratch needs: floats of partial sums and counters for a launch
void qgemv_plan(const GemvArgs& a, int layout, int num_sms, int* ksplit, int* kchunk);
size_t qgemv_ws_floats(int ksplit, int B, int total_cols);
int qgemv_group_cols(int layout);

int launch_f32_to_f16(const float* x, __half* y, size_t n, cudaStream_t st);

}  // namespace wl
