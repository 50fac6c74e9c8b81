// Quantized GEMV / skinny GEMM for decode (B <= 32 rows per launch), sm_100a.
//
// Reference semantics:
//  - layout B (woolly-core projections, tensor_utils_simd.rs:1032-1081 and
//    tensor_utils.rs:118-157): y[b, o] = sum_k x[b, k] * W[k*N + o], where W
//    is the GGUF block stream of a [K][N] matrix (32-value blocks run along N);
//  - layout A (woolly-tensor quantized_matvec, quantization.rs:1100-1163):
//    y[b, r] = sum_k W[r*K + k] * x[b, k] (blocks run along K).
//
// Design (HBM-bound):
//  * A CTA streams a [rows x 8 blocks] byte tile of the weight matrix through
//    a 4-stage cp.async.cg (16-byte, L1-bypassing) pipeline: every global load
//    is a full, aligned 16-byte vector of the block stream, uploaded unchanged.
//  * Each warp dequantizes straight from the staged bytes into mma.sync
//    m16n8k16 A-fragments in registers (LOP3 nibble -> f16 exponent trick,
//    exact q and q-8 in f16, one f16 rounding of q*d or q*d+m); the rows of x
//    (f16) are the B operand, so one dequant feeds every row of the batch.
//    The dequantized weights never touch shared memory.
//  * The output index each A-fragment row maps to is permuted so that every
//    thread reads whole 16-bit words of the block payload.
//  * K is split across CTAs to fill all 148 SMs; partial sums go to a
//    workspace and the last-arriving CTA of each column group reduces them in
//    split order (deterministic) and runs the fused epilogue (residual add,
//    QKV split with RoPE and paged-KV append, SiLU(gate)*up, f16 cast).
#include <cuda_fp16.h>

#include <algorithm>
#include <string>

#include "common.h"
#include "qgemv.cuh"

namespace wl {
namespace {

template <int T>
struct QT;
template <>
struct QT<WL_Q4_0> {
  static constexpr int S = 18, QOFF = 2, SP = 144;
};
template <>
struct QT<WL_Q4_1> {
  static constexpr int S = 20, QOFF = 4, SP = 176;  // 160 + 16 bytes against bank conflicts
};
template <>
struct QT<WL_Q8_0> {
  static constexpr int S = 34, QOFF = 2, SP = 272;
};

constexpr int kThreads = 128;
constexpr int kRows = 64;  // matrix rows per pipeline stage
constexpr int kStages = 4;
constexpr int kGroupBlocks = 8;  // quant blocks per row in one stage tile
constexpr int kColsB = 256;      // output columns per CTA, layout B
constexpr int kColsA = 64;       // output rows per CTA, layout A

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem),
               "r"(src_bytes));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ __half2 as_h2(uint32_t u) {
  __half2 h;
  memcpy(&h, &u, 4);
  return h;
}
__device__ __forceinline__ uint32_t as_u(__half2 h) {
  uint32_t u;
  memcpy(&u, &h, 4);
  return u;
}
__device__ __forceinline__ uint32_t ld16(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}

// f16 magic: 0x6400 | q is the half 1024 + q (exact for q < 1024).
constexpr uint32_t kMagic = 0x64006400u;

// Two 4-bit codes in f16 lanes (1024+q) -> weights.  Q4_0: (q-8)*d, Q4_1: q*d+m.
template <int T>
__device__ __forceinline__ uint32_t q4w(uint32_t h, uint32_t d, uint32_t m) {
  if constexpr (T == WL_Q4_0) {
    return as_u(__hmul2(__hsub2(as_h2(h), as_h2(0x64086408u)), as_h2(d)));  // 1032 = 1024+8
  } else {
    return as_u(__hfma2(__hsub2(as_h2(h), as_h2(kMagic)), as_h2(d), as_h2(m)));
  }
}
// Two int8 codes (bytes 0 and 2 of v) -> weights q*d.
__device__ __forceinline__ uint32_t q8w(uint32_t v, uint32_t d) {
  uint32_t h = ((v & 0x00FF00FFu) ^ 0x00800080u) | kMagic;             // 1024 + q + 128
  return as_u(__hmul2(__hsub2(as_h2(h), as_h2(0x64806480u)), as_h2(d)));  // - 1152
}

__device__ __forceinline__ float silu(float g) { return g * (1.0f / (1.0f + expf(-g))); }

// ------------------------------------------------------------------ epilogue
// `tile` holds the final sums [b][c] (row pitch tp) for this CTA's columns:
// segment `seg`, segment-local first column col0, `nc` valid columns.
__device__ void apply_epilogue(const GemvArgs& a, int seg, int col0, int nc, float* tile, int tp) {
  const Epilogue& e = a.epi;
  const int B = a.B;
  const int tid = threadIdx.x;
  if (e.kind == EPI_QKV && e.rope && seg < 2) {
    // NeoX rotation of (i, i + hd/2) inside each head (RoPE::apply_f32,
    // woolly-tensor/src/ops/mod.rs:476-527); col0 is a multiple of head_dim.
    const int hd = e.head_dim, half = hd / 2;
    const int npairs = nc / 2;
    for (int i = tid; i < B * npairs; i += blockDim.x) {
      int b = i / npairs, j = i % npairs;
      int h = j / half, ii = j % half;
      int c1 = h * hd + ii, c2 = c1 + half;
      float freq = 1.0f / powf(e.theta, 2.0f * (float)ii / (float)hd);
      float ang = (float)e.row_pos[b] * freq;
      float sn, cs;
      sincosf(ang, &sn, &cs);
      float x1 = tile[b * tp + c1], x2 = tile[b * tp + c2];
      tile[b * tp + c1] = x1 * cs - x2 * sn;
      tile[b * tp + c2] = x1 * sn + x2 * cs;
    }
    __syncthreads();
  }
  for (int i = tid; i < B * nc; i += blockDim.x) {
    int b = i / nc, c = i % nc;
    float v = tile[b * tp + c];
    int col = col0 + c;
    switch (e.kind) {
      case EPI_F32:
        reinterpret_cast<float*>(e.y)[(size_t)b * e.ldy + col] = v;
        break;
      case EPI_ADD:
        reinterpret_cast<float*>(e.y)[(size_t)b * e.ldy + col] += v;
        break;
      case EPI_F16:
      case EPI_SWIGLU:
        reinterpret_cast<__half*>(e.y)[(size_t)b * e.ldy + col] = __float2half_rn(v);
        break;
      case EPI_QKV: {
        if (seg == 0) {
          reinterpret_cast<float*>(e.y)[(size_t)b * e.ldy + col] = v;
        } else {
          int p = e.row_pos[b];
          int pg = e.kv.page_table[(size_t)e.row_sess[b] * e.kv.max_pages + p / e.kv.page];
          size_t off = ((size_t)pg * e.kv.page + (p % e.kv.page)) * e.kv.kvd + col;
          (seg == 1 ? e.kv.k : e.kv.v)[off] = __float2half_rn(v);
        }
        break;
      }
    }
  }
}

// Split-K completion: returns true in the CTA that must run the epilogue; in
// that CTA `tile` then holds the reduced sums.  `unit` indexes counters.
template <int TC>
__device__ bool splitk_finish(const GemvArgs& a, int split, int gcol0, int unit, int ncols_valid,
                              float* tile, int tp, bool swiglu, int up_gcol0) {
  const int tid = threadIdx.x;
  const int B = a.B;
  float* wsp = a.ws + (size_t)split * B * a.total_cols;
  for (int i = tid; i < B * TC; i += blockDim.x) {
    int b = i / TC, c = i % TC;
    if (c < ncols_valid) wsp[(size_t)b * a.total_cols + gcol0 + c] = tile[b * tp + c];
  }
  __threadfence();
  __syncthreads();
  __shared__ unsigned s_last;
  if (tid == 0) {
    unsigned target = (unsigned)a.ksplit * (swiglu ? 2u : 1u);
    unsigned prev = atomicAdd(&a.counters[unit], 1u);
    s_last = prev == target - 1;
    if (s_last) a.counters[unit] = 0;  // ready for the next launch
  }
  __syncthreads();
  if (!s_last) return false;
  __threadfence();
  const size_t sstride = (size_t)B * a.total_cols;
  for (int i = tid; i < B * TC; i += blockDim.x) {
    int b = i / TC, c = i % TC;
    if (c >= ncols_valid) continue;
    if (swiglu) {
      // gate columns live at [unit*TC], up columns at [up_gcol0]
      const float* pg = a.ws + (size_t)b * a.total_cols + (size_t)unit * TC + c;
      const float* pu = a.ws + (size_t)b * a.total_cols + up_gcol0 + c;
      float g = 0.f, u = 0.f;
      for (int s = 0; s < a.ksplit; s++) g += __ldcg(pg + s * sstride), u += __ldcg(pu + s * sstride);
      tile[b * tp + c] = silu(g) * u;
    } else {
      const float* p = a.ws + (size_t)b * a.total_cols + gcol0 + c;
      float acc = 0.f;
      for (int s = 0; s < a.ksplit; s++) acc += __ldcg(p + s * sstride);
      tile[b * tp + c] = acc;
    }
  }
  __syncthreads();
  return true;
}

// ------------------------------------------------------------------ layout B
template <int T, int NT>
__global__ void __launch_bounds__(kThreads) k_qgemv_b(const GemvArgs a) {
  using Q = QT<T>;
  constexpr int BP = NT * 8;        // padded batch rows
  constexpr int XP = kRows + 8;     // halves per x row in a stage (bank-conflict pad)
  constexpr int RAW = kRows * Q::SP;
  constexpr int XST = BP * XP;      // halves per x stage
  constexpr int CH = kGroupBlocks * Q::S / 16;  // 16-byte chunks per tile row
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* raw = smem;
  __half* xs = reinterpret_cast<__half*>(smem + kStages * RAW);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int gx = blockIdx.x, split = blockIdx.y;
  int seg = 0;
#pragma unroll
  for (int s = 1; s < 3; s++)
    if (s < a.nseg && gx >= a.seg[s].group_base) seg = s;
  const GemvSeg& S = a.seg[seg];
  const int lg = gx - S.group_base;  // group index within segment
  const uint8_t* W = S.W + (size_t)lg * kGroupBlocks * Q::S;
  const int k0 = split * a.kchunk;
  const int k1 = min(a.K, k0 + a.kchunk);
  const int nstage = (k1 - k0 + kRows - 1) / kRows;

  // valid payload bytes of this group's tile row (the last group may be partial)
  const int vbytes = min(kGroupBlocks, S.N / 32 - lg * kGroupBlocks) * Q::S;
  auto load_stage = [&](int st, int buf) {
    const int r0 = k0 + st * kRows;
    uint8_t* dst = raw + buf * RAW;
    for (int i = tid; i < kRows * CH; i += kThreads) {
      int r = i / CH, c = i - r * CH;
      int row = r0 + r;
      bool ok = row < k1 && c * 16 < vbytes;
      const uint8_t* src = W + (size_t)(ok ? row : k0) * S.pitch + c * 16;
      cp_async16(dst + r * Q::SP + c * 16, src, ok ? 16 : 0);
    }
    __half* xd = xs + buf * XST;
    for (int i = tid; i < BP * (kRows / 8); i += kThreads) {
      int b = i / (kRows / 8), c = i % (kRows / 8);
      int row = r0 + c * 8;
      bool ok = b < a.B && row < k1;
      const __half* src = a.x + (size_t)(ok ? b : 0) * a.ldx + (ok ? row : k0);
      cp_async16(xd + b * XP + c * 8, src, ok ? 16 : 0);
    }
  };

  float acc[2][2][NT][4];
#pragma unroll
  for (int i = 0; i < 2; i++)
#pragma unroll
    for (int j = 0; j < 2; j++)
#pragma unroll
      for (int n = 0; n < NT; n++)
#pragma unroll
        for (int q = 0; q < 4; q++) acc[i][j][n][q] = 0.f;

#pragma unroll
  for (int s = 0; s < kStages - 1; s++) {
    if (s < nstage) load_stage(s, s);
    cp_commit();
  }
  for (int st = 0; st < nstage; st++) {
    cp_wait<kStages - 2>();
    __syncthreads();
    {
      int nx = st + kStages - 1;
      if (nx < nstage) load_stage(nx, nx % kStages);
      cp_commit();
    }
    const int buf = st % kStages;
    const uint8_t* rs = raw + buf * RAW;
    const __half* xb = xs + buf * XST;
    const int rows_here = min(kRows, k1 - (k0 + st * kRows));
    const int nks = rows_here >> 4;
    for (int ks = 0; ks < nks; ks++) {
      uint32_t bf[NT][2];
#pragma unroll
      for (int n = 0; n < NT; n++) {
        const __half* xp = xb + (n * 8 + g) * XP + ks * 16 + 2 * t;
        bf[n][0] = *reinterpret_cast<const uint32_t*>(xp);
        bf[n][1] = *reinterpret_cast<const uint32_t*>(xp + 8);
      }
      const int r0 = ks * 16 + 2 * t;
#pragma unroll
      for (int blk = 0; blk < 2; blk++) {
        const uint8_t* rb = rs + (warp * 2 + blk) * Q::S;
        const uint8_t* p0 = rb + r0 * Q::SP;
        const uint8_t* p1 = p0 + Q::SP;
        const uint8_t* p2 = p0 + 8 * Q::SP;
        const uint8_t* p3 = p2 + Q::SP;
        uint32_t d01 = ld16(p0) | (ld16(p1) << 16);
        uint32_t d23 = ld16(p2) | (ld16(p3) << 16);
        uint32_t af[2][4];
        if constexpr (T == WL_Q8_0) {
          const int o = Q::QOFF + 2 * g;
          uint32_t v01 = ld16(p0 + o) | (ld16(p1 + o) << 16);
          uint32_t v23 = ld16(p2 + o) | (ld16(p3 + o) << 16);
          uint32_t w01 = ld16(p0 + o + 16) | (ld16(p1 + o + 16) << 16);
          uint32_t w23 = ld16(p2 + o + 16) | (ld16(p3 + o + 16) << 16);
          af[0][0] = q8w(v01, d01);
          af[0][1] = q8w(v01 >> 8, d01);
          af[0][2] = q8w(v23, d23);
          af[0][3] = q8w(v23 >> 8, d23);
          af[1][0] = q8w(w01, d01);
          af[1][1] = q8w(w01 >> 8, d01);
          af[1][2] = q8w(w23, d23);
          af[1][3] = q8w(w23 >> 8, d23);
        } else {
          uint32_t m01 = 0, m23 = 0;
          if constexpr (T == WL_Q4_1) {
            m01 = ld16(p0 + 2) | (ld16(p1 + 2) << 16);
            m23 = ld16(p2 + 2) | (ld16(p3 + 2) << 16);
          }
          const int o = Q::QOFF + 2 * g;
          uint32_t v01 = ld16(p0 + o) | (ld16(p1 + o) << 16);
          uint32_t v23 = ld16(p2 + o) | (ld16(p3 + o) << 16);
          const uint32_t M = 0x000F000Fu;
          af[0][0] = q4w<T>((v01 & M) | kMagic, d01, m01);
          af[0][1] = q4w<T>(((v01 >> 8) & M) | kMagic, d01, m01);
          af[0][2] = q4w<T>((v23 & M) | kMagic, d23, m23);
          af[0][3] = q4w<T>(((v23 >> 8) & M) | kMagic, d23, m23);
          af[1][0] = q4w<T>(((v01 >> 4) & M) | kMagic, d01, m01);
          af[1][1] = q4w<T>(((v01 >> 12) & M) | kMagic, d01, m01);
          af[1][2] = q4w<T>(((v23 >> 4) & M) | kMagic, d23, m23);
          af[1][3] = q4w<T>(((v23 >> 12) & M) | kMagic, d23, m23);
        }
#pragma unroll
        for (int n = 0; n < NT; n++) {
          mma16816(acc[blk][0][n], af[0], bf[n][0], bf[n][1]);
          mma16816(acc[blk][1][n], af[1], bf[n][0], bf[n][1]);
        }
      }
    }
  }
  cp_wait<0>();
  __syncthreads();

  // accumulators -> tile[b][c]; A-row g <-> output 2g, row g+8 <-> 2g+1, +16 for m-tile 1
  constexpr int TP = kColsB + 4;
  float* tile = reinterpret_cast<float*>(smem);
#pragma unroll
  for (int blk = 0; blk < 2; blk++)
#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
      for (int n = 0; n < NT; n++)
#pragma unroll
        for (int q = 0; q < 4; q++) {
          int b = n * 8 + 2 * t + (q & 1);
          int c = (warp * 2 + blk) * 32 + 16 * mt + 2 * g + (q >> 1);
          tile[b * TP + c] = acc[blk][mt][n][q];
        }
  __syncthreads();
  const int ncv = min(kColsB, S.N - lg * kColsB);
  const bool swiglu = a.epi.kind == EPI_SWIGLU;
  if (a.ksplit > 1 || swiglu) {
    const int unit = swiglu ? lg : gx;
    const int up_g0 = swiglu ? (a.seg[1].group_base + lg) * kColsB : 0;
    if (!splitk_finish<kColsB>(a, split, gx * kColsB, unit, ncv, tile, TP, swiglu, up_g0)) return;
    if (swiglu) {
      apply_epilogue(a, 0, lg * kColsB, ncv, tile, TP);
      return;
    }
  }
  apply_epilogue(a, seg, lg * kColsB, ncv, tile, TP);
}

// ------------------------------------------------------------------ layout A
template <int T, int NT>
__global__ void __launch_bounds__(kThreads) k_qgemv_a(const GemvArgs a) {
  using Q = QT<T>;
  constexpr int BP = NT * 8;
  constexpr int KS = kGroupBlocks * 32;  // k values per stage (256)
  constexpr int XP = KS + 8;
  constexpr int RAW = kColsA * Q::SP;
  constexpr int XST = BP * XP;
  constexpr int CH = kGroupBlocks * Q::S / 16;
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* raw = smem;
  __half* xs = reinterpret_cast<__half*>(smem + kStages * RAW);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int gx = blockIdx.x, split = blockIdx.y;
  const GemvSeg& S = a.seg[0];
  const int n0 = gx * kColsA;
  const int k0 = split * a.kchunk;
  const int k1 = min(a.K, k0 + a.kchunk);
  const int nstage = (k1 - k0) / KS;

  auto load_stage = [&](int st, int buf) {
    const int kk = k0 + st * KS;
    const size_t byte0 = (size_t)(kk / 32) * Q::S;
    uint8_t* dst = raw + buf * RAW;
    for (int i = tid; i < kColsA * CH; i += kThreads) {
      int r = i / CH, c = i - r * CH;
      int row = n0 + r;
      bool ok = row < S.N;
      const uint8_t* src = S.W + (size_t)(ok ? row : 0) * S.pitch + byte0 + c * 16;
      cp_async16(dst + r * Q::SP + c * 16, src, ok ? 16 : 0);
    }
    __half* xd = xs + buf * XST;
    for (int i = tid; i < BP * (KS / 8); i += kThreads) {
      int b = i / (KS / 8), c = i % (KS / 8);
      bool ok = b < a.B;
      const __half* src = a.x + (size_t)(ok ? b : 0) * a.ldx + kk + c * 8;
      cp_async16(xd + b * XP + c * 8, src, ok ? 16 : 0);
    }
  };

  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; n++)
#pragma unroll
    for (int q = 0; q < 4; q++) acc[n][q] = 0.f;

#pragma unroll
  for (int s = 0; s < kStages - 1; s++) {
    if (s < nstage) load_stage(s, s);
    cp_commit();
  }
  for (int st = 0; st < nstage; st++) {
    cp_wait<kStages - 2>();
    __syncthreads();
    {
      int nx = st + kStages - 1;
      if (nx < nstage) load_stage(nx, nx % kStages);
      cp_commit();
    }
    const int buf = st % kStages;
    const uint8_t* rA0 = raw + buf * RAW + (warp * 16 + g) * Q::SP;
    const uint8_t* rB0 = rA0 + 8 * Q::SP;
    const __half* xb = xs + buf * XST;
#pragma unroll 2
    for (int bi = 0; bi < kGroupBlocks; bi++) {
      const uint8_t* rA = rA0 + bi * Q::S;
      const uint8_t* rB = rB0 + bi * Q::S;
      uint32_t dA = ld16(rA), dB = ld16(rB);
      dA |= dA << 16;
      dB |= dB << 16;
      uint32_t af[2][4];
      if constexpr (T == WL_Q8_0) {
        // byte j of the payload is k = j; k-step 0 covers k 0..15, k-step 1 k 16..31
#pragma unroll
        for (int s = 0; s < 2; s++) {
          const int o = Q::QOFF + 16 * s + 2 * t;
          af[s][0] = q8w(__byte_perm(ld16(rA + o), 0, 0x4140), dA);
          af[s][1] = q8w(__byte_perm(ld16(rB + o), 0, 0x4140), dB);
          af[s][2] = q8w(__byte_perm(ld16(rA + o + 8), 0, 0x4140), dA);
          af[s][3] = q8w(__byte_perm(ld16(rB + o + 8), 0, 0x4140), dB);
        }
      } else {
        uint32_t mA = 0, mB = 0;
        if constexpr (T == WL_Q4_1) {
          mA = ld16(rA + 2), mB = ld16(rB + 2);
          mA |= mA << 16;
          mB |= mB << 16;
        }
        const int o = Q::QOFF + 2 * t;
        // low nibble of byte j is k = j, high nibble is k = j + 16
        uint32_t xA0 = __byte_perm(ld16(rA + o), 0, 0x4140);
        uint32_t xA1 = __byte_perm(ld16(rA + o + 8), 0, 0x4140);
        uint32_t xB0 = __byte_perm(ld16(rB + o), 0, 0x4140);
        uint32_t xB1 = __byte_perm(ld16(rB + o + 8), 0, 0x4140);
        const uint32_t M = 0x000F000Fu;
        af[0][0] = q4w<T>((xA0 & M) | kMagic, dA, mA);
        af[0][1] = q4w<T>((xB0 & M) | kMagic, dB, mB);
        af[0][2] = q4w<T>((xA1 & M) | kMagic, dA, mA);
        af[0][3] = q4w<T>((xB1 & M) | kMagic, dB, mB);
        af[1][0] = q4w<T>(((xA0 >> 4) & M) | kMagic, dA, mA);
        af[1][1] = q4w<T>(((xB0 >> 4) & M) | kMagic, dB, mB);
        af[1][2] = q4w<T>(((xA1 >> 4) & M) | kMagic, dA, mA);
        af[1][3] = q4w<T>(((xB1 >> 4) & M) | kMagic, dB, mB);
      }
#pragma unroll
      for (int s = 0; s < 2; s++)
#pragma unroll
        for (int n = 0; n < NT; n++) {
          const __half* xp = xb + (n * 8 + g) * XP + bi * 32 + s * 16 + 2 * t;
          mma16816(acc[n], af[s], *reinterpret_cast<const uint32_t*>(xp),
                   *reinterpret_cast<const uint32_t*>(xp + 8));
        }
    }
  }
  cp_wait<0>();
  __syncthreads();
  constexpr int TP = kColsA + 4;
  float* tile = reinterpret_cast<float*>(smem);
#pragma unroll
  for (int n = 0; n < NT; n++)
#pragma unroll
    for (int q = 0; q < 4; q++) {
      int b = n * 8 + 2 * t + (q & 1);
      int c = warp * 16 + g + 8 * (q >> 1);
      tile[b * TP + c] = acc[n][q];
    }
  __syncthreads();
  const int ncv = min(kColsA, S.N - n0);
  if (a.ksplit > 1) {
    if (!splitk_finish<kColsA>(a, split, n0, gx, ncv, tile, TP, false, 0)) return;
  }
  apply_epilogue(a, 0, n0, ncv, tile, TP);
}

// ------------------------------------------------------------------ generic fallback
__device__ __forceinline__ float deq1(int type, const uint8_t* blk, int j) {
  float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(blk)));
  if (type == WL_Q4_0) {
    int q = j < 16 ? (blk[2 + j] & 15) - 8 : (blk[2 + j - 16] >> 4) - 8;
    return (float)q * d;
  }
  if (type == WL_Q4_1) {
    float m = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(blk + 2)));
    int q = j < 16 ? (blk[4 + j] & 15) : (blk[4 + j - 16] >> 4);
    return __fadd_rn(__fmul_rn((float)q, d), m);
  }
  return (float)(int8_t)blk[2 + j] * d;
}

__global__ void k_qgemv_generic(int type, int layout, const uint8_t* W, int K, int N, int pitch,
                                const __half* x, int ldx, int B, float* y, int ldy, int add) {
  int o = blockIdx.x * blockDim.x + threadIdx.x;
  int b = blockIdx.y;
  if (o >= N || b >= B) return;
  const int S = type == WL_Q4_0 ? 18 : type == WL_Q4_1 ? 20 : 34;
  float acc = 0.f;
  for (int k = 0; k < K; k++) {
    float w;
    if (type == WL_F32)
      w = layout == WL_LAYOUT_B ? reinterpret_cast<const float*>(W + (size_t)k * pitch)[o]
                                : reinterpret_cast<const float*>(W + (size_t)o * pitch)[k];
    else
      w = layout == WL_LAYOUT_B ? deq1(type, W + (size_t)k * pitch + (o / 32) * S, o % 32)
                                : deq1(type, W + (size_t)o * pitch + (k / 32) * S, k % 32);
    acc += __half2float(x[(size_t)b * ldx + k]) * w;
  }
  if (add)
    y[(size_t)b * ldy + o] += acc;
  else
    y[(size_t)b * ldy + o] = acc;
}

__global__ void k_f32_to_f16(const float* x, __half* y, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) y[i] = __float2half_rn(x[i]);
}

template <int T>
constexpr int raw_bytes_b() {
  return kStages * kRows * QT<T>::SP;
}

template <int T, int NT>
int launch_b_t(const GemvArgs& a, cudaStream_t st) {
  constexpr int BP = NT * 8;
  size_t pipe = (size_t)kStages * kRows * QT<T>::SP + (size_t)kStages * BP * (kRows + 8) * 2;
  size_t epi = (size_t)BP * (kColsB + 4) * 4;
  size_t smem = std::max(pipe, epi);
  static unsigned attr_done = 0;  // one bit per device, per instantiation
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_done >> (dev & 31) & 1u)) {
    WL_CUDA_TRY(cudaFuncSetAttribute(k_qgemv_b<T, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
    attr_done |= 1u << (dev & 31);
  }
  int groups = 0;
  for (int s = 0; s < a.nseg; s++) groups += a.seg[s].groups;
  dim3 grid(groups, a.ksplit);
  k_qgemv_b<T, NT><<<grid, kThreads, smem, st>>>(a);
  WL_CUDA_TRY(cudaGetLastError());
  return WL_OK;
}

template <int T, int NT>
int launch_a_t(const GemvArgs& a, cudaStream_t st) {
  constexpr int BP = NT * 8;
  size_t pipe = (size_t)kStages * kColsA * QT<T>::SP + (size_t)kStages * BP * (256 + 8) * 2;
  size_t epi = (size_t)BP * (kColsA + 4) * 4;
  size_t smem = std::max(pipe, epi);
  static unsigned attr_done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_done >> (dev & 31) & 1u)) {
    WL_CUDA_TRY(cudaFuncSetAttribute(k_qgemv_a<T, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
    attr_done |= 1u << (dev & 31);
  }
  dim3 grid(a.seg[0].groups, a.ksplit);
  k_qgemv_a<T, NT><<<grid, kThreads, smem, st>>>(a);
  WL_CUDA_TRY(cudaGetLastError());
  return WL_OK;
}

template <int T>
int dispatch_b(const GemvArgs& a, cudaStream_t st) {
  int nt = (a.B + 7) / 8;
  switch (nt) {
    case 1: return launch_b_t<T, 1>(a, st);
    case 2: return launch_b_t<T, 2>(a, st);
    case 3: return launch_b_t<T, 3>(a, st);
    case 4: return launch_b_t<T, 4>(a, st);
  }
  return fail(WL_ERR_INVALID_ARGUMENT, "qgemv: B must be 1..32 per launch");
}

template <int T>
int dispatch_a(const GemvArgs& a, cudaStream_t st) {
  int nt = (a.B + 7) / 8;
  switch (nt) {
    case 1: return launch_a_t<T, 1>(a, st);
    case 2: return launch_a_t<T, 2>(a, st);
    case 3: return launch_a_t<T, 3>(a, st);
    case 4: return launch_a_t<T, 4>(a, st);
  }
  return fail(WL_ERR_INVALID_ARGUMENT, "qgemv: B must be 1..32 per launch");
}

int block_bytes(int type) { return type == WL_Q4_0 ? 18 : type == WL_Q4_1 ? 20 : type == WL_Q8_0 ? 34 : 0; }

}  // namespace

int qgemv_group_cols(int layout) { return layout == WL_LAYOUT_B ? kColsB : kColsA; }

// Layout B needs 16-byte aligned rows (pitch % 16 == 0, padding allowed) and
// 16 readable bytes past the last row's payload (the tail chunk of a partial
// group may straddle the end of the payload).
bool qgemv_b_fast_ok(int type, int K, int N, int pitch, const void* W) {
  int S = block_bytes(type);
  if (!S) return false;
  return K % 16 == 0 && K > 0 && N % 32 == 0 && pitch % 16 == 0 && pitch >= N / 32 * S &&
         (reinterpret_cast<uintptr_t>(W) & 15) == 0;
}

bool qgemv_a_fast_ok(int type, int K, int N, int pitch, const void* W) {
  int S = block_bytes(type);
  if (!S) return false;
  (void)N;
  return K % 256 == 0 && pitch % 16 == 0 && pitch == K / 32 * S &&
         (reinterpret_cast<uintptr_t>(W) & 15) == 0;
}

void qgemv_plan(const GemvArgs& a, int layout, int num_sms, int* ksplit, int* kchunk) {
  int groups = 0;
  for (int s = 0; s < a.nseg; s++) groups += a.seg[s].groups;
  const int gran = layout == WL_LAYOUT_B ? 16 : 256;
  const int units = a.K / gran;
  const int target = 2 * num_sms;
  int ks = (target + groups - 1) / std::max(groups, 1);
  ks = std::max(1, std::min(ks, units));
  int chunk = (units + ks - 1) / ks * gran;
  ks = (a.K + chunk - 1) / chunk;
  *ksplit = ks;
  *kchunk = chunk;
}

size_t qgemv_ws_floats(int ksplit, int B, int total_cols) {
  return (size_t)ksplit * B * total_cols;
}

int launch_qgemv_b(const GemvArgs& a, cudaStream_t st) {
  switch (a.type) {
    case WL_Q4_0: return dispatch_b<WL_Q4_0>(a, st);
    case WL_Q4_1: return dispatch_b<WL_Q4_1>(a, st);
    case WL_Q8_0: return dispatch_b<WL_Q8_0>(a, st);
  }
  return fail(WL_ERR_UNSUPPORTED, "qgemv: unsupported type " + std::to_string(a.type));
}

int launch_qgemv_a(const GemvArgs& a, cudaStream_t st) {
  switch (a.type) {
    case WL_Q4_0: return dispatch_a<WL_Q4_0>(a, st);
    case WL_Q4_1: return dispatch_a<WL_Q4_1>(a, st);
    case WL_Q8_0: return dispatch_a<WL_Q8_0>(a, st);
  }
  return fail(WL_ERR_UNSUPPORTED, "qgemv: unsupported type " + std::to_string(a.type));
}

int launch_qgemv_generic(int type, int layout, const uint8_t* W, int K, int N, int pitch,
                         const __half* x, int ldx, int B, float* y, int ldy, bool add,
                         cudaStream_t st) {
  if (!block_bytes(type) && type != WL_F32) return fail(WL_ERR_UNSUPPORTED, "qgemv: unsupported type");
  dim3 grid((N + 127) / 128, B);
  k_qgemv_generic<<<grid, 128, 0, st>>>(type, layout, W, K, N, pitch, x, ldx, B, y, ldy, add);
  WL_CUDA_TRY(cudaGetLastError());
  return WL_OK;
}

int launch_f32_to_f16(const float* x, __half* y, size_t n, cudaStream_t st) {
  if (!n) return WL_OK;
  k_f32_to_f16<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, y, n);
  WL_CUDA_TRY(cudaGetLastError());
  return WL_OK;
}

}  // namespace wl
