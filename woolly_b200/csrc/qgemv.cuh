// Quantized GEMV / skinny GEMM (decode path) — shared declarations.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "peer.cuh"

namespace wl {

// Epilogue kinds (applied once the full K sum of an output is known).
enum EpiKind : int {
  EPI_F32 = 0,     // segment s: y[s][b*ldy + col] = v
  EPI_ADD = 1,     // segment s: y[s][b*ldy + col] += v (residual)
  EPI_QKV = 2,     // seg0 -> q f32 (+rope), seg1 -> K pages f16 (+rope), seg2 -> V pages f16
  EPI_SWIGLU = 3,  // seg0 = gate, seg1 = up (paired in one cluster): y[0] gets silu(g)*u as
                   // f16 hi/lo planes (lo plane at y[0] + y_plane)
  EPI_PEER = 4,    // tensor-parallel partial sums pushed to every rank: peer[r][b*ldy + col] = v
                   // for r < nranks, then each CTA adds 1 to pflag[r] (release, system scope)
};


// Activation operand of the layout-B GEMV: f16 hi/lo planes, x = hi + lo with
// lo = f16(x - hi) (~22 significant bits).  Element (b, k) of the hi plane is
// x[b*ldx + k]; the lo plane starts x_plane elements later.  Layout A (the
// op-level matvec) takes plain f32 activations instead.
enum XKind : int {
  X_PLANES = 0,
  X_F32 = 1,
};


// Paged KV cache addressing for one layer: element (token j, kv head h, dim d)
// of a session lives at page = table[sess][j / page], slot = j % page, in
//   base[((page * kv_heads + h) * page_tokens + slot) * head_dim + d]
// so one (page, head) is a contiguous page_tokens x head_dim f16 chunk.
struct KvPages {
  __half* k = nullptr;
  __half* v = nullptr;
  const int* page_table = nullptr;  // [n_sessions_max][max_pages]
  int max_pages = 0;                // row stride of page_table
  int page = 16;                    // tokens per page
  int kv_heads = 0;
  int head_dim = 0;
};

__host__ __device__ inline size_t kv_offset(const KvPages& kv, int pg, int slot, int head, int d) {
  return (((size_t)pg * kv.kv_heads + head) * kv.page + slot) * kv.head_dim + d;
}

struct Epilogue {
  int kind = EPI_F32;
  void* y[3] = {nullptr, nullptr, nullptr};  // per-segment outputs
  int ldy[3] = {0, 0, 0};
  size_t y_plane = 0;  // EPI_SWIGLU: offset of the lo plane (elements)
  // QKV / rope
  int rope = 0;
  int head_dim = 0;
  float theta = 10000.f;
  const int* row_pos = nullptr;   // [B] absolute position of each row
  const int* row_sess = nullptr;  // [B] session slot of each row (page table row)
  KvPages kv{};
  // EPI_PEER: this rank's receive slot in every rank's buffer (own rank included,
  // peer pointers through CUDA IPC mappings) and its arrival counter there
  int nranks = 0;
  float* peer[kMaxPeers] = {};
  unsigned* pflag[kMaxPeers] = {};
};

struct GemvSeg {
  const uint8_t* W = nullptr;
  int N = 0;          // columns (layout B) or rows (layout A)
  int pitch = 0;      // bytes per matrix row
  int groups = 0;     // column groups (tiles) in this segment
  int group_base = 0;
};

struct GemvArgs {
  int type = 2;  // WL_Q4_0 / WL_Q4_1 / WL_Q8_0
  int nseg = 1;
  GemvSeg seg[3];
  int K = 0;     // reduction length
  int B = 0;     // rows of x (<= 32 per launch)
  int xkind = X_PLANES;
  const void* x = nullptr;  // __half planes (X_PLANES) or float (X_F32)
  size_t x_plane = 0;
  int ldx = 0;
  int csplit = 1;  // CTAs per cluster splitting K (1..16)
  int kchunk = 0;  // rows of K per CTA (multiple of 16; of 64 tiled; of 256 for layout A)
  int tiled = 0;   // layout B only: seg[s].W is the tiled decode copy (qtile_bytes)
  Epilogue epi;
  int* err = nullptr;  // optional: bit 2 set when the cluster reduction wait gave up
};

#ifdef __CUDACC__
// swiglu activation (tensor_utils.rs:512-532): silu(g) = g * (1 / (1 + exp(-g)))
__device__ __forceinline__ float silu(float g) { return g * (1.0f / (1.0f + expf(-g))); }

// One output element of segment `seg`, launch row b, segment column col:
// F32 store, residual ADD, or the QKV split (q as f32; k and v as f16 into the
// row's KV page).
__device__ __forceinline__ void store_out(const GemvArgs& a, int seg, int b, int col, float v) {
  const Epilogue& e = a.epi;
  switch (e.kind) {
    case EPI_F32:
      reinterpret_cast<float*>(e.y[seg])[(size_t)b * e.ldy[seg] + col] = v;
      break;
    case EPI_ADD:
      reinterpret_cast<float*>(e.y[seg])[(size_t)b * e.ldy[seg] + col] += v;
      break;
    case EPI_QKV:
      if (seg == 0) {
        reinterpret_cast<float*>(e.y[0])[(size_t)b * e.ldy[0] + col] = v;
      } else {
        const int p = e.row_pos[b];
        const int pg = e.kv.page_table[(size_t)e.row_sess[b] * e.kv.max_pages + p / e.kv.page];
        const size_t off =
            kv_offset(e.kv, pg, p % e.kv.page, col / e.kv.head_dim, col % e.kv.head_dim);
        (seg == 1 ? e.kv.k : e.kv.v)[off] = __float2half_rn(v);
      }
      break;
  }
}
#endif

// Prefill GEMM on tcgen05 tensor cores (qgemm.cu): all M rows of x (f16 hi/lo
// planes, a.ldx % 8 == 0) against layout-B weights given as their tiled decode
// copies (a.tiled = 1, seg[s].W from launch_repack_tiled) in one launch.  Needs
// K % 64 == 0 and every segment's N % 128 == 0 (SwiGLU: N % 64 == 0); rope off.
bool qgemm_b_ok(const GemvArgs& a, int M);
int launch_qgemm_b(const GemvArgs& a, int M, cudaStream_t st);

// Host launchers (stream-ordered).  Return a wl_status.
int launch_qgemv_b(const GemvArgs& a, cudaStream_t st);
int launch_qgemv_a(const GemvArgs& a, cudaStream_t st);
// generic (any alignment / F32 weights) fallback, f32 math; EPI_F32/EPI_ADD;
// x is f32 (x_plane == 0) or hi/lo f16 planes (x_plane = lo-plane offset)
int launch_qgemv_generic(int type, int layout, const uint8_t* W, int K, int N, int pitch,
                         const void* x, size_t x_plane, int ldx, int B, float* y, int ldy,
                         bool add, cudaStream_t st);
// f32 -> hi/lo f16 planes (lo plane `plane` elements after hi)
int launch_split_planes(const float* x, __half* y, size_t n, size_t plane, cudaStream_t st);
bool qgemv_b_fast_ok(int type, int K, int N, int pitch, const void* W);
// Q4_K / Q6_K: run from the tiled copy only (N % 256 == 0, K % 16 == 0)
bool kquant_type(int type);
int kquant_block_bytes(int type);  // GGUF bytes of one 256-value super-block
// layout A (ggml orientation) K-quants run from rows of super-blocks padded to
// kq_padded_bytes (Q4_K 144, Q6_K 224): launch_kq_pad writes them
int kq_padded_bytes(int type);
int launch_kq_pad(int type, const uint8_t* src, size_t src_pitch, int rows, int K, uint8_t* dst,
                  cudaStream_t st);
bool qgemv_a_fast_ok(int type, int K, int N, int pitch, const void* W);
// picks csplit / kchunk for a launch (fills the GPU)
void qgemv_plan(GemvArgs& a, int layout, int num_sms);

// Tiled decode copy of a layout-B matrix: for each 256-column group and each
// 64-row k stage, one contiguous block of 512 quant blocks' bytes (Q4_0 9216)
// arranged as the GEMV's MMA lanes read them: per (warp w, 16-row k step,
// block pair member) unit, each lane's A-fragment codes (8 bytes; Q8_0 16)
// for k rows 2t, 2t+1, 2t+8, 2t+9 and outputs g, g+8, 16+g, 24+g of its
// block, then the scales (Q4_1: and mins) as 8 bytes per (unit, t).  Rows
// past K and columns past N are zero weights.  Same size as the GGUF bytes
// when K % 64 == 0 and N % 256 == 0.
size_t qtile_bytes(int type, int K, int N);
int launch_repack_tiled(int type, const uint8_t* src, int K, int N, int pitch, uint8_t* dst,
                        cudaStream_t st);

int qgemv_group_cols(int layout);

}  // namespace wl
