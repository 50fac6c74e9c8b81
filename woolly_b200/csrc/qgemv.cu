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
//  * One CTA owns a tile of 8 quant blocks along a matrix row (256 columns in
//    layout B, 256 K-values in layout A) and streams its K-slice of rows
//    through a 4-stage cp.async.cg (16-byte, L1-bypassing) pipeline together
//    with the matching activation tile, so every global load is an aligned
//    16-byte vector of the block stream, uploaded unchanged.
//  * The MMA sees exact operands: A = the integer codes (q-8 for Q4_0, q for
//    Q4_1 / Q8_0, exact in f16; built with PRMT + LOP3 from the staged bytes
//    and the f16 exponent trick, never written back to shared memory), and
//    B = the activation times the block scale carried as an f16 hi/lo pair
//    ((x*d)_hi + (x*d)_lo, ~22 bits) built with HMUL2/HFMA2 from the hi/lo
//    activation planes.  Q4_1's min term sum_k x*m rides on an extra MMA with
//    an all-ones A.  m16n8k16 mma.sync with f32 accumulation.
//  * K is split across the CTAs of a thread-block cluster (up to 16); the
//    partial tiles are reduced through distributed shared memory in rank order
//    (deterministic), each CTA finishing a strided slice of the outputs and
//    applying the fused epilogue (residual add, QKV split with RoPE and
//    paged-KV append, SiLU(gate)*up with gate and up in one cluster).
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <climits>
#include <cstdint>
#include <map>
#include <mutex>
#include <tuple>
#include <cstdlib>
#include <string>

#include "common.h"
#include "qgemv.cuh"
#include "pdl.cuh"

namespace cg = cooperative_groups;

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
// K-quants run from the tiled copy only; S is the tiled bytes per 32-column
// unit of one k row: Q4_K 16 code bytes + the (hi, lo) f16 pair of d*sc + the
// f16 dmin; Q6_K 32 code bytes + two (hi, lo) pairs (one per 16 columns)
template <>
struct QT<WL_Q4_K> {
  static constexpr int S = 22, QOFF = 0, SP = 176;
};
template <>
struct QT<WL_Q6_K> {
  static constexpr int S = 40, QOFF = 0, SP = 320;
};
template <int T>
constexpr bool kB8 = T == WL_Q8_0 || T == WL_Q6_K;  // one code byte per weight
template <int T>
constexpr bool kMin = T == WL_Q4_1 || T == WL_Q4_K;  // a per-block additive term
template <int T>
constexpr bool kKq = T == WL_Q4_K || T == WL_Q6_K;  // scale given as an exact f16 pair

constexpr int kThreads = 128;  // layout A
constexpr int kThreadsB = 128;  // layout B: warps 4..7 take the second half of each stage's k-steps
constexpr int kKParts = kThreadsB / 128;
constexpr int kRows = 64;  // matrix rows per pipeline stage
constexpr int kStages = 4;  // layout A
// layout-B pipeline depth: batch tiles of up to 16 rows keep more stages in flight
__host__ __device__ constexpr int stages_b(int NT) { return 4; }
constexpr int kGroupBlocks = 8;  // quant blocks per tile row
constexpr int kColsB = 256;      // output columns per CTA, layout B
constexpr int kColsA = 64;       // output rows per CTA, layout A
constexpr int kMaxCluster = 16;
// Layout-B CTAs per SM the K-split planner aims for, when their shared memory
// fits (measured on the 7B decode step: 3 beats 2 by 5%; 4 no longer fits and
// spills into a second wave)
constexpr int kPlanCtasPerSm = 3;
constexpr int kSmemPerSm = 228 * 1024;  // B200 shared memory per SM (1 KB of it reserved per CTA)

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
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// four 8x8 b16 matrices; lane l supplies the row address of matrix l/8, row l%8
__device__ __forceinline__ void ldsm_x4(const void* row_addr, uint32_t& r0, uint32_t& r1,
                                        uint32_t& r2, uint32_t& r3) {
  const unsigned a = (unsigned)__cvta_generic_to_shared(row_addr);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
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
__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b) {
  return as_u(__hsub2(as_h2(a), as_h2(b)));
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  return __byte_perm(a, b, sel);
}

// 0x6400 | c is the f16 value 1024 + c (exact for c < 1024).
constexpr uint32_t kMagic = 0x64006400u;
constexpr uint32_t kOnes = 0x3C003C00u;  // half2(1, 1)

// low-nibble codes in f16 lanes (1024+q) -> exact q-8 (Q4_0) or q (Q4_1)
template <int T>
__device__ __forceinline__ uint32_t q4a(uint32_t h) {
  return hsub2u(h, T == WL_Q4_0 ? 0x64086408u : kMagic);
}
// high-nibble codes in f16 lanes (1024+16q) -> exact 16(q-8) (Q4_0) or 16q (Q4_1)
template <int T>
__device__ __forceinline__ uint32_t q4a_hi(uint32_t h) {
  return hsub2u(h, T == WL_Q4_0 ? 0x64806480u : kMagic);
}
// int8 codes in bytes 0 and 2 of v (bytes 1 and 3 zero) -> exact q in f16 lanes
__device__ __forceinline__ uint32_t q8a(uint32_t v) {
  return hsub2u((v ^ 0x00800080u) | kMagic, 0x64806480u);  // 1024 + q + 128 - 1152
}

// (d*x) as an f16 pair hi + lo: hi = f16(d*xh), lo = f16(d*xl + (d*xh - hi));
// the residual d*xh - hi is exact in f16, so hi + lo carries ~22 bits.
__device__ __forceinline__ void scale_split(uint32_t d, uint32_t xh, uint32_t xl, uint32_t& hi,
                                            uint32_t& lo) {
  __half2 hh = __hmul2(as_h2(d), as_h2(xh));
  __half2 r = __hfma2(as_h2(d), as_h2(xh), __hneg2(hh));
  hi = as_u(hh);
  lo = as_u(__hfma2(as_h2(d), as_h2(xl), r));
}
// The same for a scale s = sh + sl that needs more than 11 bits (the K-quant
// sub-block scale d*sc, up to 19 bits, split exactly into two f16 at repack):
// hi = f16(sh*xh), lo = f16(sh*xl + sl*xh + (sh*xh - hi)).
__device__ __forceinline__ void scale_split2(uint32_t sh, uint32_t sl, uint32_t xh, uint32_t xl,
                                             uint32_t& hi, uint32_t& lo) {
  __half2 hh = __hmul2(as_h2(sh), as_h2(xh));
  __half2 r = __hfma2(as_h2(sh), as_h2(xh), __hneg2(hh));
  r = __hfma2(as_h2(sl), as_h2(xh), r);
  hi = as_u(hh);
  lo = as_u(__hfma2(as_h2(sh), as_h2(xl), r));
}


// Layout A: cp.async copies of one stage's f32 activation tile [BP][KC]; rows
// >= B and columns >= k1 are zero-filled.
__device__ __forceinline__ void load_x_f32(const GemvArgs& a, float* dst, int BP, int KC, int kk0,
                                           int k1) {
  const int nch = KC / 4;
  const float* x = reinterpret_cast<const float*>(a.x);
  for (int i = threadIdx.x; i < BP * nch; i += blockDim.x) {
    const int b = i / nch, c = i - b * nch;
    const int k = kk0 + c * 4;
    const bool ok = b < a.B && k < k1;
    cp_async16(dst + b * KC + c * 4, x + (ok ? (size_t)b * a.ldx + k : 0), ok ? 16 : 0);
  }
}

// f32 tile [BP][KC] -> hi/lo planes [2][BP][XP]
__device__ __forceinline__ void split_tile(const float* src, __half* xs, int BP, int KC, int XP) {
  for (int i = threadIdx.x; i < BP * KC; i += blockDim.x) {
    const int b = i / KC, k = i - b * KC;
    const float v = src[i];
    const __half hi = __float2half_rn(v);
    xs[b * XP + k] = hi;
    xs[BP * XP + b * XP + k] = __float2half_rn(v - __half2float(hi));
  }
}

// ------------------------------------------------------------------ epilogue
// store_out (qgemv.cuh) applies F32 / ADD / QKV outputs per element.

// Cluster split-K reduction by push.  The output tile of a CTA (B rows x
// `cols` columns, ncv valid) is cut into float4 groups; group q of every CTA
// is owned by rank item(q) % C.  Each CTA sends its partial of every group to
// the owner's receive area with st.async (remote shared-memory stores that
// count bytes on the owner's mbarrier), then waits until the C partials of its
// own groups have arrived and sums them in rank order (deterministic).  One
// cluster barrier, split into arrive (kernel start, after the mbarrier init)
// and wait (before the first send), orders the init before any remote store;
// no barrier is needed at the end because an owner only exits after its bytes
// have landed.  RoPE items hold the pair of groups (i, i + hd/2); for
// EPI_SWIGLU gate tiles sit at even ranks and the matching up tiles at odd
// ranks.
__device__ __forceinline__ float4 f4add(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

struct ClusterRed {
  uint32_t bar = 0;  // shared address of the mbarrier
  float4* recv = nullptr;
  int C = 1, r = 0, nitems = 0, parts = 1, ipr = 0;
};

// receive area bytes for BP padded rows of `cols` columns
__host__ __device__ constexpr size_t recv_bytes(int BP, int cols) {
  return ((size_t)BP * cols / 4 + 2 * kMaxCluster) * 16;
}

__device__ __forceinline__ bool red_rope(const GemvArgs& a, int seg) {
  return a.epi.kind == EPI_QKV && a.epi.rope && seg < 2;
}

__device__ __forceinline__ void red_begin(ClusterRed& R, const GemvArgs& a, int seg, int ncv,
                                          uint64_t* bar, void* recv) {
  cg::cluster_group cl = cg::this_cluster();
  R.C = (int)cl.num_blocks();
  R.r = (int)cl.block_rank();
  R.parts = red_rope(a, seg) ? 2 : 1;
  R.nitems = a.B * (ncv / (4 * R.parts));
  R.ipr = (R.nitems + R.C - 1) / R.C;
  R.recv = reinterpret_cast<float4*>(recv);
  R.bar = (uint32_t)__cvta_generic_to_shared(bar);
  if (threadIdx.x == 0) {
    const int mine = R.r < R.nitems ? (R.nitems - 1 - R.r) / R.C + 1 : 0;
    const uint32_t bytes = (uint32_t)(mine * R.C * R.parts * 16);
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(R.bar) : "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(R.bar), "r"(bytes)
                 : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
}

__device__ __forceinline__ void st_async4(uint32_t dst, float4 v, uint32_t bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];\n" ::"r"(dst),
      "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(bar)
      : "memory");
}
__device__ __forceinline__ uint32_t mapa(uint32_t addr, int rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(out) : "r"(addr), "r"(rank));
  return out;
}

// bounded wait for phase 0 of the receive barrier; false when it gave up
__device__ __forceinline__ bool red_wait(uint32_t bar) {
  for (int it = 0; it < (1 << 22); it++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], 0;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar)
        : "memory");
    if (ok) return true;
  }
  return false;
}

__device__ void cluster_finish(const GemvArgs& a, const ClusterRed& R, float* tile, int tp,
                               int ncv, int seg, int col0) {
  const int C = R.C, r = R.r, P = R.parts;
  const int B = a.B;
  const Epilogue& e = a.epi;
  const int g4 = ncv / 4;
  const int hd = e.head_dim, half = hd / 2;
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");  // every mbarrier is set up
  // send: group q = (b, c) of this CTA's tile to its owner
  const uint32_t recv0 = (uint32_t)__cvta_generic_to_shared(R.recv);
  if (P == 1) {
    // item = q: owner q % C, slot q / C, row q / g4 -- stepped incrementally
    // (q advances by blockDim.x), no integer division per item
    const int step = (int)blockDim.x;
    const int so = step % C, sj = step / C, sb = step / g4, sc = step % g4;
    int q = threadIdx.x, owner = q % C, j = q / C, b = q / g4, c4 = q % g4;
    for (; q < B * g4; q += step) {
      const float4 v = *reinterpret_cast<const float4*>(tile + b * tp + c4 * 4);
      st_async4(mapa(recv0 + (uint32_t)((r * R.ipr + j) * 16), owner), v, mapa(R.bar, owner));
      owner += so, j += sj, b += sb, c4 += sc;
      if (owner >= C) owner -= C, j++;
      if (c4 >= g4) c4 -= g4, b++;
    }
  } else {
    for (int q = threadIdx.x; q < B * g4; q += blockDim.x) {
      const int b = q / g4, c = (q - b * g4) * 4;
      const int h = c / hd, w = c - h * hd;
      const int part = w >= half;
      const int item = b * (g4 / 2) + h * (half / 4) + (w - part * half) / 4;
      const int owner = item % C, j = item / C;
      const float4 v = *reinterpret_cast<const float4*>(tile + b * tp + c);
      st_async4(mapa(recv0 + (uint32_t)(((r * R.ipr + j) * P + part) * 16), owner), v,
                mapa(R.bar, owner));
    }
  }
  const bool got = red_wait(R.bar);
  if (!got && a.err && threadIdx.x == 0) atomicOr(a.err, 4);
  // finish the owned items, partials summed in rank order
  for (int j = threadIdx.x; got && r + C * j < R.nitems; j += blockDim.x) {
    const int item = r + C * j;
    if (e.kind == EPI_SWIGLU) {
      const int b = item / g4, c = (item - b * g4) * 4;
      float4 gs = make_float4(0.f, 0.f, 0.f, 0.f), us = gs;
      for (int src = 0; src < C; src += 2) gs = f4add(gs, R.recv[src * R.ipr + j]);
      for (int src = 1; src < C; src += 2) us = f4add(us, R.recv[src * R.ipr + j]);
      const float gv[4] = {gs.x, gs.y, gs.z, gs.w}, uv[4] = {us.x, us.y, us.z, us.w};
      __half* out = reinterpret_cast<__half*>(e.y[0]);
      const size_t o = (size_t)b * e.ldy[0] + col0 + c;
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float v = silu(gv[u]) * uv[u];  // swiglu, tensor_utils.rs:512-532
        const __half hi = __float2half_rn(v);
        out[o + u] = hi;
        out[o + u + e.y_plane] = __float2half_rn(v - __half2float(hi));
      }
    } else if (P == 2) {
      // NeoX rotation inside each head (RoPE::apply_f32, woolly-tensor/src/ops/mod.rs:476-527);
      // col0 is a multiple of head_dim.
      const int np4 = g4 / 2;
      const int b = item / np4, p = item - b * np4;
      const int h = p / (half / 4), ii = (p - h * (half / 4)) * 4;
      const int c1 = h * hd + ii, c2 = c1 + half;
      float4 s1 = make_float4(0.f, 0.f, 0.f, 0.f), s2 = s1;
      for (int src = 0; src < C; src++) {
        s1 = f4add(s1, R.recv[(src * R.ipr + j) * 2]);
        s2 = f4add(s2, R.recv[(src * R.ipr + j) * 2 + 1]);
      }
      const float x1[4] = {s1.x, s1.y, s1.z, s1.w}, x2[4] = {s2.x, s2.y, s2.z, s2.w};
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float freq = 1.0f / powf(e.theta, 2.0f * (float)(ii + u) / (float)hd);
        float sn, cs;
        sincosf((float)e.row_pos[b] * freq, &sn, &cs);
        store_out(a, seg, b, col0 + c1 + u, x1[u] * cs - x2[u] * sn);
        store_out(a, seg, b, col0 + c2 + u, x1[u] * sn + x2[u] * cs);
      }
    } else {
      const int b = item / g4, c = (item - b * g4) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int src = 0; src < C; src++) v = f4add(v, R.recv[src * R.ipr + j]);
      if (e.kind == EPI_PEER) {  // NVLink stores into every rank's receive slot
        const size_t o = (size_t)b * e.ldy[0] + col0 + c;
        for (int pr = 0; pr < e.nranks; pr++) *reinterpret_cast<float4*>(e.peer[pr] + o) = v;
      } else {
        store_out(a, seg, b, col0 + c, v.x);
        store_out(a, seg, b, col0 + c + 1, v.y);
        store_out(a, seg, b, col0 + c + 2, v.z);
        store_out(a, seg, b, col0 + c + 3, v.w);
      }
    }
  }
  if (e.kind == EPI_PEER) {
    // every CTA signals once its stores are out (also after a failed cluster
    // wait, with the error flag set, so that no rank waits for it in vain)
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      for (int pr = 0; pr < e.nranks; pr++)
        asm volatile("red.release.sys.global.add.u32 [%0], 1;\n" ::"l"(e.pflag[pr]) : "memory");
    }
  }
}

// ------------------------------------------------------------------ layout B
// LOC (lo in columns, B <= 4 only): the MMA's 8 columns carry the hi part of
// (x*d) for rows 0-3 in columns 0-3 and the lo part in columns 4-7, so one MMA
// pair per tile replaces the hi and lo pairs; the epilogue adds column c + 4
// to column c.
// TLD: weights in the tiled decode layout (qtile_bytes): a stage is one
// contiguous copy and each lane reads its A-fragment codes and scales with two
// 8-byte loads (outputs g, g+8, 16+g, 24+g of its block).
template <int T, int NT, bool LOC, bool TLD>
__global__ void __launch_bounds__(kThreadsB) k_qgemv_b(const GemvArgs a) {
  using Q = QT<T>;
  constexpr int BP = NT * 8;  // padded batch rows
  constexpr int RAW = kRows * Q::SP;
  constexpr int XP = kRows + 8;               // halves per staged x row (bank-conflict pad)
  constexpr int SST = RAW + 2 * BP * XP * 2;  // stage: weight tile + hi/lo x planes
  constexpr int SB = stages_b(NT);
  constexpr int CH = kGroupBlocks * Q::S / 16;  // 16-byte chunks per tile row
  constexpr int XCH = 2 * BP * (kRows / 8);     // 16-byte chunks of x per stage
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* raw = smem;

  // Tiled codes enter the MMA as f16 subnormals (q * 2^-24: one LOP3 per pair,
  // no HSUB2).  Q4_1 has no offset; Q4_0's -8 and Q8_0's -128 (codes stored
  // as q + 128) then cost a ones-MMA per B fragment, which pays only when LOC
  // halves the MMAs (Q4_0 decode: B = 1 +7%, B = 16 -2%).
  // K-quants: Q4_K is Q4_1 with the two-term scale; Q6_K is Q8_0-like codes
  // (q - 32) with one scale per 16 columns, i.e. per m-tile
  constexpr bool SUBN = TLD && (kMin<T> || (LOC && !kKq<T>));
  constexpr float kOff = T == WL_Q4_0 ? -8.0f : -128.0f;  // SUBN offset of Q4_0 / Q8_0
  const int tid = threadIdx.x, lane = tid & 31;
  const int warp = (tid >> 5) & 3, kpart = tid >> 7;  // block pair, k-step part
  const int g = lane >> 2, t = lane & 3;
  const int gx = blockIdx.x, split = blockIdx.y;
  int seg = 0, lg;
  if (a.epi.kind == EPI_SWIGLU) {  // x = 2*group + (0 gate | 1 up)
    seg = gx & 1;
    lg = gx >> 1;
  } else {
#pragma unroll
    for (int s = 1; s < 3; s++)
      if (s < a.nseg && gx >= a.seg[s].group_base) seg = s;
    lg = gx - a.seg[seg].group_base;
  }
  const int Nseg = a.seg[seg].N, pitch = a.seg[seg].pitch;
  constexpr int STB = 512 * Q::S;                  // tiled: bytes of one (group, stage) block
  constexpr int CODEB = 1024 * (kB8<T> ? 16 : 8);  // tiled: code bytes of a stage block
  const uint8_t* W = TLD ? a.seg[seg].W + ((size_t)lg * ((a.K + kRows - 1) / kRows) + split * (a.kchunk / kRows)) * STB
                         : a.seg[seg].W + (size_t)lg * kGroupBlocks * Q::S;
  const int k0 = split * a.kchunk;
  const int k1 = min(a.K, k0 + a.kchunk);
  const int nstage = k1 > k0 ? (k1 - k0 + kRows - 1) / kRows : 0;
  // valid payload bytes of this group's tile row (the last group may be partial)
  const int vbytes = min(kGroupBlocks, Nseg / 32 - lg * kGroupBlocks) * Q::S;
  const int ncv = min(kColsB, Nseg - lg * kColsB);
  constexpr int PIPE = SB * SST > BP * (kColsB + 4) * 4 ? SB * SST : BP * (kColsB + 4) * 4;
  __shared__ uint64_t red_bar;
  ClusterRed R;
  red_begin(R, a, seg, ncv, &red_bar, smem + PIPE);

  // this thread's 16-byte chunks of a stage (fixed across stages)
  constexpr int NWC = (kRows * CH + kThreadsB - 1) / kThreadsB;
  constexpr int NXC = (XCH + kThreadsB - 1) / kThreadsB;
  int wr[NWC], wc[NWC];
#pragma unroll
  for (int j = 0; j < NWC; j++) {
    const int i = tid + j * kThreadsB;
    wr[j] = i < kRows * CH ? i / CH : -1;
    wc[j] = i - (i / CH) * CH;
  }
  const __half* xg = reinterpret_cast<const __half*>(a.x);
  int xc[NXC], xo[NXC];
  size_t xsrc[NXC];
#pragma unroll
  for (int j = 0; j < NXC; j++) {
    const int i = tid + j * kThreadsB;
    const int p = i / (BP * (kRows / 8)), rem = i - p * BP * (kRows / 8);
    const int b = rem / (kRows / 8), c = rem - b * (kRows / 8);
    const bool live = i < XCH && b < a.B;
    xc[j] = live ? c * 8 : -1;
    xo[j] = (p * BP * XP + b * XP + c * 8) * 2;
    xsrc[j] = live ? p * a.x_plane + (size_t)b * a.ldx + c * 8 : 0;
  }
  auto load_w = [&](int st, int buf) {  // immutable weights
    if constexpr (TLD) {  // one contiguous block per stage
      uint8_t* dst = raw + buf * SST;
      const uint8_t* src = W + (size_t)st * STB;
#pragma unroll
      for (int j = 0; j < (STB / 16 + kThreadsB - 1) / kThreadsB; j++) {
        const int c = tid + j * kThreadsB;
        if (c < STB / 16) cp_async16(dst + c * 16, src + c * 16, 16);
      }
      return;
    }
    const int r0 = k0 + st * kRows;
    uint8_t* dst = raw + buf * SST;
#pragma unroll
    for (int j = 0; j < NWC; j++) {
      if (wr[j] < 0) continue;
      const int row = r0 + wr[j];
      const bool ok = row < k1 && wc[j] * 16 < vbytes;
      cp_async16(dst + wr[j] * Q::SP + wc[j] * 16,
                 W + (ok ? (size_t)row * pitch + wc[j] * 16 : 0), ok ? 16 : 0);
    }
  };
  auto load_x = [&](int st, int buf) {  // activations written by the previous kernel
    const int r0 = k0 + st * kRows;
    uint8_t* dst = raw + buf * SST;
#pragma unroll
    for (int j = 0; j < NXC; j++) {
      if (tid + j * kThreadsB >= XCH) continue;
      const bool ok = xc[j] >= 0 && r0 + xc[j] < k1;
      cp_async16(dst + RAW + xo[j], xg + (ok ? xsrc[j] + r0 : 0), ok ? 16 : 0);
    }
  };
  auto load_stage = [&](int st, int buf) {
    load_w(st, buf);
    load_x(st, buf);
  };

  // weight prefetch of the first stages may overlap the previous kernel (PDL)
#pragma unroll
  for (int s = 0; s < SB - 1; s++)
    if (s < nstage) load_w(s, s);
  pdl_wait();
  pdl_trigger();
#pragma unroll
  for (int s = 0; s < SB - 1; s++) {
    if (s < nstage) load_x(s, s);
    cp_commit();
  }

  float acc[2][2][NT][4];
  float accm[2][NT][4];  // Q4_1: sum_k x*m per block (same for all rows of the block)
#pragma unroll
  for (int i = 0; i < 2; i++)
#pragma unroll
    for (int n = 0; n < NT; n++)
#pragma unroll
      for (int q = 0; q < 4; q++) acc[i][0][n][q] = acc[i][1][n][q] = accm[i][n][q] = 0.f;

  for (int st = 0; st < nstage; st++) {
    cp_wait<SB - 2>();
    __syncthreads();
    {
      const int nx = st + SB - 1;
      if (nx < nstage) load_stage(nx, nx % SB);
      cp_commit();
    }
    const uint8_t* rs = raw + (st % SB) * SST;
    const __half* xs = reinterpret_cast<const __half*>(rs + RAW);
    // rows past the end of this split are zero-filled and contribute exactly 0
#pragma unroll
    for (int kk = 0; kk < kRows / 16 / kKParts; kk++) {
      const int ks = kpart * (kRows / 16 / kKParts) + kk;
      // B fragments (session = n*8 + g, k = 2t..2t+1 | +8) of the hi and lo planes:
      // matrices {hi k0-7, hi k8-15, lo k0-7, lo k8-15} of rows n*8..n*8+7
      uint32_t xh[NT][2], xl[NT][2];
#pragma unroll
      for (int n = 0; n < NT; n++) {
        const int mi = lane >> 3;
        const int xrow = LOC ? (lane & 3) : (lane & 7);  // LOC: rows 4-7 read rows 0-3 again
        const __half* ra = xs + (mi >> 1) * BP * XP + (n * 8 + xrow) * XP + ks * 16 + (mi & 1) * 8;
        ldsm_x4(ra, xh[n][0], xh[n][1], xl[n][0], xl[n][1]);
      }
      const uint8_t* p0b = rs + (ks * 16 + 2 * t) * Q::SP + warp * 2 * Q::S;
#pragma unroll
      for (int blk = 0; blk < 2; blk++) {
        uint32_t af[2][4];
        uint32_t d01, d23, m01 = 0, m23 = 0;
        uint32_t e01 = 0, e23 = 0;                        // K-quants: lo halves of the scales
        uint32_t d01b = 0, d23b = 0, e01b = 0, e23b = 0;  // Q6_K: scales of m-tile 1
        if constexpr (TLD) {
          const int u = (warp * 4 + ks) * 2 + blk;
          if constexpr (T == WL_Q6_K) {
            const uint4 s0 = *reinterpret_cast<const uint4*>(rs + CODEB + (u * 8 + t) * 16);
            const uint4 s1 = *reinterpret_cast<const uint4*>(rs + CODEB + (u * 8 + 4 + t) * 16);
            d01 = s0.x, d23 = s0.y, e01 = s0.z, e23 = s0.w;
            d01b = s1.x, d23b = s1.y, e01b = s1.z, e23b = s1.w;
          } else if constexpr (T == WL_Q4_K) {
            const uint4 sw = *reinterpret_cast<const uint4*>(rs + CODEB + (u * 4 + t) * 16);
            d01 = sw.x, d23 = sw.y, e01 = sw.z, e23 = sw.w;
            const uint2 mw = *reinterpret_cast<const uint2*>(rs + CODEB + 2048 + (u * 4 + t) * 8);
            m01 = mw.x;
            m23 = mw.y;
          } else {
            const uint2 sw = *reinterpret_cast<const uint2*>(rs + CODEB + (u * 4 + t) * 8);
            d01 = sw.x;
            d23 = sw.y;
          }
          if constexpr (T == WL_Q4_1) {
            const uint2 mw = *reinterpret_cast<const uint2*>(rs + CODEB + 1024 + (u * 4 + t) * 8);
            m01 = mw.x;
            m23 = mw.y;
          }
          if constexpr (kB8<T>) {
            const uint4 cw = *reinterpret_cast<const uint4*>(rs + u * 512 + lane * 16);
            const uint32_t w[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
            for (int q = 0; q < 4; q++) {
              if constexpr (SUBN) {  // q + 128 as subnormal f16
                af[q >> 1][(q & 1) * 2] = prmt(w[q], 0u, 0x4140) ^ 0x00800080u;
                af[q >> 1][(q & 1) * 2 + 1] = prmt(w[q], 0u, 0x4342) ^ 0x00800080u;
              } else {
                af[q >> 1][(q & 1) * 2] = q8a(prmt(w[q], 0u, 0x4140));
                af[q >> 1][(q & 1) * 2 + 1] = q8a(prmt(w[q], 0u, 0x4342));
              }
            }
          } else {
            const uint2 cw = *reinterpret_cast<const uint2*>(rs + u * 256 + lane * 8);
            const uint32_t w0 = cw.x, w1 = cw.y, v0 = w0 >> 8, v1 = w1 >> 8;
            const uint32_t ML = 0x000F000Fu, MH = 0x00F000F0u;
            if constexpr (SUBN) {
              // f16 subnormals: q * 2^-24 (low nibbles), 16q * 2^-24 (high); the
              // epilogue scales by 2^24 / 2^20 and Q4_0's -8 offset comes from accm
              af[0][0] = w0 & ML;
              af[0][1] = v0 & ML;
              af[0][2] = w1 & ML;
              af[0][3] = v1 & ML;
              af[1][0] = w0 & MH;
              af[1][1] = v0 & MH;
              af[1][2] = w1 & MH;
              af[1][3] = v1 & MH;
            } else {
              af[0][0] = q4a<T>((w0 & ML) | kMagic);
              af[0][1] = q4a<T>((v0 & ML) | kMagic);
              af[0][2] = q4a<T>((w1 & ML) | kMagic);
              af[0][3] = q4a<T>((v1 & ML) | kMagic);
              af[1][0] = q4a_hi<T>((w0 & MH) | kMagic);
              af[1][1] = q4a_hi<T>((v0 & MH) | kMagic);
              af[1][2] = q4a_hi<T>((w1 & MH) | kMagic);
              af[1][3] = q4a_hi<T>((v1 & MH) | kMagic);
            }
          }
        } else {
        const uint8_t* p0 = p0b + blk * Q::S;
        const uint8_t* p1 = p0 + Q::SP;
        const uint8_t* p2 = p0 + 8 * Q::SP;
        const uint8_t* p3 = p2 + Q::SP;
        d01 = prmt(ld16(p0), ld16(p1), 0x5410);
        d23 = prmt(ld16(p2), ld16(p3), 0x5410);
        const int o = Q::QOFF + 2 * g;
        // byte 0 (sel 0x6420) or byte 1 (sel 0x6521) of the 16-bit payload words of
        // rows (r0, r0+1) and (r0+8, r0+9), one per f16 lane
        const uint32_t q0 = ld16(p0 + o), q1 = ld16(p1 + o), q2 = ld16(p2 + o), q3 = ld16(p3 + o);
        const uint32_t x00 = prmt(q0, q1, 0x6420), x01 = prmt(q0, q1, 0x6521);
        const uint32_t x20 = prmt(q2, q3, 0x6420), x21 = prmt(q2, q3, 0x6521);
        if constexpr (T == WL_Q8_0) {
          // A-row g <-> output 2g, row g+8 <-> 2g+1; m-tile 1 = outputs +16
          const uint32_t s0 = ld16(p0 + o + 16), s1 = ld16(p1 + o + 16);
          const uint32_t s2 = ld16(p2 + o + 16), s3 = ld16(p3 + o + 16);
          af[0][0] = q8a(x00);
          af[0][1] = q8a(x01);
          af[0][2] = q8a(x20);
          af[0][3] = q8a(x21);
          af[1][0] = q8a(prmt(s0, s1, 0x6420));
          af[1][1] = q8a(prmt(s0, s1, 0x6521));
          af[1][2] = q8a(prmt(s2, s3, 0x6420));
          af[1][3] = q8a(prmt(s2, s3, 0x6521));
        } else {
          // A-row g <-> output 2g, row g+8 <-> 2g+1 (m-tile 0: low nibbles); m-tile 1
          // (outputs +16, high nibbles) holds 16x the codes and is rescaled at the end
          const uint32_t ML = 0x000F000Fu, MH = 0x00F000F0u;
          af[0][0] = q4a<T>((x00 & ML) | kMagic);
          af[0][1] = q4a<T>((x01 & ML) | kMagic);
          af[0][2] = q4a<T>((x20 & ML) | kMagic);
          af[0][3] = q4a<T>((x21 & ML) | kMagic);
          af[1][0] = q4a_hi<T>((x00 & MH) | kMagic);
          af[1][1] = q4a_hi<T>((x01 & MH) | kMagic);
          af[1][2] = q4a_hi<T>((x20 & MH) | kMagic);
          af[1][3] = q4a_hi<T>((x21 & MH) | kMagic);
        }
        if constexpr (T == WL_Q4_1) {
          m01 = prmt(ld16(p0 + 2), ld16(p1 + 2), 0x5410);
          m23 = prmt(ld16(p2 + 2), ld16(p3 + 2), 0x5410);
        }
        }
#pragma unroll
        for (int n = 0; n < NT; n++) {
          uint32_t bh0, bl0, bh1, bl1;
          if constexpr (kKq<T>) {
            scale_split2(d01, e01, xh[n][0], xl[n][0], bh0, bl0);
            scale_split2(d23, e23, xh[n][1], xl[n][1], bh1, bl1);
          } else {
            scale_split(d01, xh[n][0], xl[n][0], bh0, bl0);
            scale_split(d23, xh[n][1], xl[n][1], bh1, bl1);
          }
          if constexpr (T == WL_Q6_K) {  // m-tile 1 has its own scales
            uint32_t ch0, cl0, ch1, cl1;
            scale_split2(d01b, e01b, xh[n][0], xl[n][0], ch0, cl0);
            scale_split2(d23b, e23b, xh[n][1], xl[n][1], ch1, cl1);
            if constexpr (LOC) {
              const bool loc = g >= 4;
              mma16816(acc[blk][0][n], af[0], loc ? bl0 : bh0, loc ? bl1 : bh1);
              mma16816(acc[blk][1][n], af[1], loc ? cl0 : ch0, loc ? cl1 : ch1);
            } else {
              mma16816(acc[blk][0][n], af[0], bh0, bh1);
              mma16816(acc[blk][1][n], af[1], ch0, ch1);
              mma16816(acc[blk][0][n], af[0], bl0, bl1);
              mma16816(acc[blk][1][n], af[1], cl0, cl1);
            }
          } else if constexpr (LOC) {
            const bool loc = g >= 4;  // this lane's B column carries a lo part
            const uint32_t b0 = loc ? bl0 : bh0, b1 = loc ? bl1 : bh1;
            mma16816(acc[blk][0][n], af[0], b0, b1);
            mma16816(acc[blk][1][n], af[1], b0, b1);
          } else {
            mma16816(acc[blk][0][n], af[0], bh0, bh1);
            mma16816(acc[blk][1][n], af[1], bh0, bh1);
            mma16816(acc[blk][0][n], af[0], bl0, bl1);
            mma16816(acc[blk][1][n], af[1], bl0, bl1);
          }
          if constexpr (SUBN && !kMin<T>) {  // sum_k x*d of the block, for the offset
            const uint32_t ones[4] = {kOnes, kOnes, kOnes, kOnes};
            if constexpr (LOC) {
              const bool loc = g >= 4;
              mma16816(accm[blk][n], ones, loc ? bl0 : bh0, loc ? bl1 : bh1);
            } else {
              mma16816(accm[blk][n], ones, bh0, bh1);
              mma16816(accm[blk][n], ones, bl0, bl1);
            }
          }
          if constexpr (kMin<T>) {
            const uint32_t ones[4] = {kOnes, kOnes, kOnes, kOnes};
            uint32_t mh0, ml0, mh1, ml1;
            scale_split(m01, xh[n][0], xl[n][0], mh0, ml0);
            scale_split(m23, xh[n][1], xl[n][1], mh1, ml1);
            if constexpr (LOC) {
              const bool loc = g >= 4;
              mma16816(accm[blk][n], ones, loc ? ml0 : mh0, loc ? ml1 : mh1);
            } else {
              mma16816(accm[blk][n], ones, mh0, mh1);
              mma16816(accm[blk][n], ones, ml0, ml1);
            }
          }
        }
      }
    }
  }
  cp_wait<0>();
  __syncthreads();

  // accumulators -> tile[b][c] (reuses the pipeline buffers); the k-step parts
  // add up in the tile
  constexpr int TP = kColsB + 4;
  float* tile = reinterpret_cast<float*>(smem);
#pragma unroll
  for (int pass = 0; pass < kKParts; pass++) {
    if (kpart == pass) {
#pragma unroll
      for (int blk = 0; blk < 2; blk++)
#pragma unroll
        for (int mt = 0; mt < 2; mt++)
#pragma unroll
          for (int n = 0; n < NT; n++)
#pragma unroll
            for (int q = 0; q < 4; q++) {
              const int b = n * 8 + 2 * t + (q & 1);
              // A-row r of m-tile mt: output 2r / 2r+1 (GGUF byte order) or r (tiled)
              const int c = (warp * 2 + blk) * 32 + 16 * mt + (TLD ? g + 8 * (q >> 1) : 2 * g + (q >> 1));
              // m-tile 1 of the 4-bit types accumulated 16x the codes; the
              // subnormal codes of the tiled path carry 2^-24 (exact powers of two)
              // (Q6_K: the scale pair is d*sc, the reference's /64 is applied here)
              const float sc = SUBN ? ((!kB8<T> && mt == 1) ? 1048576.0f : 16777216.0f)
                               : T == WL_Q6_K ? 0.015625f
                                              : (!kB8<T> && mt == 1) ? 0.0625f : 1.0f;
              // accm: sum x*m (Q4_1 / Q4_K) or, subnormal Q4_0 / Q8_0, sum x*d times the offset
              const float cm = (SUBN && !kMin<T>) ? kOff : 1.0f;
              float v = acc[blk][mt][n][q] * sc + cm * accm[blk][n][q];
              if constexpr (LOC) {  // column b + 4 (lane t + 2) holds row b's lo part
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                if (t >= 2) continue;
              }
              if (pass == 0)
                tile[b * TP + c] = v;
              else
                tile[b * TP + c] += v;
            }
    }
    __syncthreads();
  }
  cluster_finish(a, R, tile, TP, ncv, seg, lg * kColsB);
}

// ------------------------------------------------------------------ layout A
template <int T, int NT>
__global__ void __launch_bounds__(kThreads) k_qgemv_a(const GemvArgs a) {
  using Q = QT<T>;
  constexpr int BP = NT * 8;
  constexpr int KS = kGroupBlocks * 32;  // k values per stage (256)
  constexpr int RAW = kColsA * Q::SP;
  constexpr int CH = kGroupBlocks * Q::S / 16;
  constexpr int STG = NT <= 2 ? kStages : 2;  // pipeline depth (large batch tiles use 2)
  constexpr int SST = RAW + BP * KS * 4;      // weight tile + f32 activation tile per stage
  constexpr int XP = KS + 8;
  constexpr int PIPE = STG * SST > BP * (kColsA + 4) * 4 ? STG * SST : BP * (kColsA + 4) * 4;
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* raw = smem;
  pdl_wait();
  pdl_trigger();
  __half* xs = reinterpret_cast<__half*>(smem + PIPE);
  const __half* xl_base = xs + BP * XP;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int gx = blockIdx.x, split = blockIdx.y;
  const GemvSeg& S = a.seg[0];
  const int n0 = gx * kColsA;
  const int k0 = split * a.kchunk;
  const int k1 = min(a.K, k0 + a.kchunk);
  const int nstage = k1 > k0 ? (k1 - k0) / KS : 0;
  const int ncv = min(kColsA, S.N - n0);
  __shared__ uint64_t red_bar;
  ClusterRed R;
  red_begin(R, a, 0, ncv, &red_bar, smem + PIPE + 2 * BP * XP * 2);

  auto load_stage = [&](int st, int buf) {
    const size_t byte0 = (size_t)((k0 + st * KS) / 32) * Q::S;
    uint8_t* dst = raw + buf * SST;
    for (int i = tid; i < kColsA * CH; i += kThreads) {
      const int r = i / CH, c = i - r * CH;
      const int row = n0 + r;
      const bool ok = row < S.N;
      cp_async16(dst + r * Q::SP + c * 16, S.W + (size_t)(ok ? row : 0) * S.pitch + byte0 + c * 16,
                 ok ? 16 : 0);
    }
    load_x_f32(a, reinterpret_cast<float*>(dst + RAW), BP, KS, k0 + st * KS, k1);
  };

#pragma unroll
  for (int s = 0; s < STG - 1; s++) {
    if (s < nstage) load_stage(s, s);
    cp_commit();
  }

  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; n++)
#pragma unroll
    for (int q = 0; q < 4; q++) acc[n][q] = 0.f;

  for (int st = 0; st < nstage; st++) {
    cp_wait<STG - 2>();
    __syncthreads();
    {
      const int nx = st + STG - 1;
      if (nx < nstage) load_stage(nx, nx % STG);
      cp_commit();
    }
    split_tile(reinterpret_cast<const float*>(raw + (st % STG) * SST + RAW), xs, BP, KS, XP);
    __syncthreads();
    const uint8_t* rA0 = raw + (st % STG) * SST + (warp * 16 + g) * Q::SP;
    const uint8_t* rB0 = rA0 + 8 * Q::SP;
#pragma unroll 2
    for (int bi = 0; bi < kGroupBlocks; bi++) {
      const uint8_t* rA = rA0 + bi * Q::S;
      const uint8_t* rB = rB0 + bi * Q::S;
      const float dA = __half2float(__ushort_as_half((unsigned short)ld16(rA)));
      const float dB = __half2float(__ushort_as_half((unsigned short)ld16(rB)));
      uint32_t af[2][4];
      if constexpr (T == WL_Q8_0) {
        // payload byte j is k = j: k-step 0 covers k 0..15, k-step 1 k 16..31
#pragma unroll
        for (int s = 0; s < 2; s++) {
          const int o = Q::QOFF + 16 * s + 2 * t;
          af[s][0] = q8a(__byte_perm(ld16(rA + o), 0, 0x4140));
          af[s][1] = q8a(__byte_perm(ld16(rB + o), 0, 0x4140));
          af[s][2] = q8a(__byte_perm(ld16(rA + o + 8), 0, 0x4140));
          af[s][3] = q8a(__byte_perm(ld16(rB + o + 8), 0, 0x4140));
        }
      } else {
        const int o = Q::QOFF + 2 * t;
        // low nibble of byte j is k = j, high nibble is k = j + 16
        const uint32_t xA0 = __byte_perm(ld16(rA + o), 0, 0x4140);
        const uint32_t xA1 = __byte_perm(ld16(rA + o + 8), 0, 0x4140);
        const uint32_t xB0 = __byte_perm(ld16(rB + o), 0, 0x4140);
        const uint32_t xB1 = __byte_perm(ld16(rB + o + 8), 0, 0x4140);
        const uint32_t M = 0x000F000Fu;
        af[0][0] = q4a<T>((xA0 & M) | kMagic);
        af[0][1] = q4a<T>((xB0 & M) | kMagic);
        af[0][2] = q4a<T>((xA1 & M) | kMagic);
        af[0][3] = q4a<T>((xB1 & M) | kMagic);
        af[1][0] = q4a<T>(((xA0 >> 4) & M) | kMagic);
        af[1][1] = q4a<T>(((xB0 >> 4) & M) | kMagic);
        af[1][2] = q4a<T>(((xA1 >> 4) & M) | kMagic);
        af[1][3] = q4a<T>(((xB1 >> 4) & M) | kMagic);
      }
      const uint32_t ones[4] = {kOnes, kOnes, kOnes, kOnes};
#pragma unroll
      for (int n = 0; n < NT; n++) {
        float c[4] = {0.f, 0.f, 0.f, 0.f}, cm[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 2; s++) {
          const int kk = bi * 32 + s * 16 + 2 * t;
          const __half* xp = xs + (n * 8 + g) * XP + kk;
          const __half* lp = xl_base + (n * 8 + g) * XP + kk;
          const uint32_t h0 = *reinterpret_cast<const uint32_t*>(xp);
          const uint32_t h1 = *reinterpret_cast<const uint32_t*>(xp + 8);
          const uint32_t l0 = *reinterpret_cast<const uint32_t*>(lp);
          const uint32_t l1 = *reinterpret_cast<const uint32_t*>(lp + 8);
          mma16816(c, af[s], h0, h1);
          mma16816(c, af[s], l0, l1);
          if constexpr (T == WL_Q4_1) {
            mma16816(cm, ones, h0, h1);
            mma16816(cm, ones, l0, l1);
          }
        }
        // block scale per A row: c0,c1 belong to row g, c2,c3 to row g+8
        acc[n][0] += dA * c[0];
        acc[n][1] += dA * c[1];
        acc[n][2] += dB * c[2];
        acc[n][3] += dB * c[3];
        if constexpr (T == WL_Q4_1) {
          const float mA = __half2float(__ushort_as_half((unsigned short)ld16(rA + 2)));
          const float mB = __half2float(__ushort_as_half((unsigned short)ld16(rB + 2)));
          acc[n][0] += mA * cm[0];
          acc[n][1] += mA * cm[1];
          acc[n][2] += mB * cm[2];
          acc[n][3] += mB * cm[3];
        }
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
      const int b = n * 8 + 2 * t + (q & 1);
      const int c = warp * 16 + g + 8 * (q >> 1);
      tile[b * TP + c] = acc[n][q];
    }
  __syncthreads();
  cluster_finish(a, R, tile, TP, ncv, 0, n0);
}

// ------------------------------------------------------------------ generic fallback
__device__ __forceinline__ float deq1(int type, const uint8_t* blk, int j) {
  const float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(blk)));
  if (type == WL_Q4_0) {
    const int q = j < 16 ? (blk[2 + j] & 15) - 8 : (blk[2 + j - 16] >> 4) - 8;
    return (float)q * d;
  }
  if (type == WL_Q4_1) {
    const float m = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(blk + 2)));
    const int q = j < 16 ? (blk[4 + j] & 15) : (blk[4 + j - 16] >> 4);
    return __fadd_rn(__fmul_rn((float)q, d), m);
  }
  return (float)(int8_t)blk[2 + j] * d;
}

__global__ void k_qgemv_generic(int type, int layout, const uint8_t* W, int K, int N, int pitch,
                                const void* xv, size_t x_plane, int ldx, int B, float* y, int ldy,
                                int add) {
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (o >= N || b >= B) return;
  const int S = type == WL_Q4_0 ? 18 : type == WL_Q4_1 ? 20 : 34;
  const float* xf = reinterpret_cast<const float*>(xv);
  const __half* xh = reinterpret_cast<const __half*>(xv);
  float acc = 0.f;
  for (int k = 0; k < K; k++) {
    float w;
    if (type == WL_F32)
      w = layout == WL_LAYOUT_B ? reinterpret_cast<const float*>(W + (size_t)k * pitch)[o]
                                : reinterpret_cast<const float*>(W + (size_t)o * pitch)[k];
    else
      w = layout == WL_LAYOUT_B ? deq1(type, W + (size_t)k * pitch + (o / 32) * S, o % 32)
                                : deq1(type, W + (size_t)o * pitch + (k / 32) * S, k % 32);
    const size_t xi = (size_t)b * ldx + k;
    const float xk = x_plane ? __half2float(xh[xi]) + __half2float(xh[xi + x_plane]) : xf[xi];
    acc += xk * w;
  }
  if (add)
    y[(size_t)b * ldy + o] += acc;
  else
    y[(size_t)b * ldy + o] = acc;
}

__global__ void k_split_planes(const float* x, __half* y, size_t n, size_t plane) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = x[i];
  const __half hi = __float2half_rn(v);
  y[i] = hi;
  y[i + plane] = __float2half_rn(v - __half2float(hi));
}

// ------------------------------------------------------------------ launch
template <int T>
size_t smem_b(int NT) {
  const size_t BP = (size_t)NT * 8;
  const size_t pipe = (size_t)stages_b(NT) * (kRows * QT<T>::SP + 2 * BP * (kRows + 8) * 2);
  const size_t tile = BP * (kColsB + 4) * 4;
  return std::max(pipe, tile) + recv_bytes((int)BP, kColsB);
}
template <int T>
size_t smem_a(int NT) {
  const size_t BP = (size_t)NT * 8;
  const int stg = NT <= 2 ? kStages : 2;
  const size_t pipe = (size_t)stg * (kColsA * QT<T>::SP + BP * 256 * 4);
  const size_t tile = BP * (kColsA + 4) * 4;
  const size_t xs = 2 * BP * (256 + 8) * 2;
  return std::max(pipe, tile) + xs + recv_bytes((int)BP, kColsA);
}

template <class Kern>
int launch_cluster(Kern kern, dim3 grid, int threads, size_t smem, int cx, int cy,
                   const GemvArgs& a, cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (first_use_on_device((const void*)kern)) {
    WL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    WL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = cx;
  at[0].val.clusterDim.y = cy;
  at[0].val.clusterDim.z = 1;
  cfg.numAttrs = 1;
  if (pdl_enabled()) {
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  cfg.attrs = at;
  WL_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
  return WL_OK;
}

// ------------------------------------------------------------------ tiled decode copy
// One thread per (group, stage, unit, lane): writes the lane's code bytes of
// one unit (warp w, k step ks, block pair member blk) and, for lanes 0-3, the
// unit's scales (and mins) for t = lane.  Source: GGUF blocks [K][N/32].
template <int T>
__global__ void k_repack_tiled(const uint8_t* src, int K, int N, int pitch, uint8_t* dst, int stages,
                               size_t total) {
  using Q = QT<T>;
  constexpr int STB = 512 * Q::S;
  constexpr int CB = T == WL_Q8_0 ? 16 : 8;  // code bytes per lane per unit
  constexpr int CODEB = 1024 * CB;  // 32 units x 32 lanes
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int lane = (int)(i & 31), u = (int)((i >> 5) & 31);
  const size_t gs = i >> 10;  // group * stages + stage
  const int stage = (int)(gs % stages);
  const int group = (int)(gs / stages);
  const int w = u >> 3, ks = (u >> 1) & 3, blk = u & 1;
  const int cb = group * kGroupBlocks + w * 2 + blk;
  const bool colok = cb < N / 32;
  const int g = lane >> 2, t = lane & 3;
  const int kb = stage * kRows + ks * 16;
  uint8_t* D = dst + gs * STB;
  auto code = [&](int o, int k) -> uint32_t {  // output o (0..31) of block cb at k row k
    if (!colok || k >= K) return T == WL_Q4_0 ? 8u : 0u;
    const uint8_t* b = src + (size_t)k * pitch + (size_t)cb * Q::S;
    if (T == WL_Q8_0) return b[2 + o];
    return o < 16 ? (b[Q::QOFF + o] & 15u) : (b[Q::QOFF + o - 16] >> 4);
  };
  auto scale = [&](int k, int which) -> uint32_t {  // which 0: d, 1: m (Q4_1)
    if (!colok || k >= K) return 0u;
    const uint8_t* b = src + (size_t)k * pitch + (size_t)cb * Q::S + 2 * which;
    return (uint32_t)(b[0] | (b[1] << 8));
  };
  uint8_t* C = D + u * (32 * CB) + lane * CB;
  if (T == WL_Q8_0) {
    // registers m-tile 0 a0..a3, m-tile 1 a0..a3, 2 codes each (k even, k odd)
    for (int mt = 0; mt < 2; mt++)
      for (int r = 0; r < 4; r++) {
        const int o = mt * 16 + g + 8 * (r & 1), k = kb + 2 * t + 8 * (r >> 1);
        C[(mt * 4 + r) * 2] = (uint8_t)code(o, k);
        C[(mt * 4 + r) * 2 + 1] = (uint8_t)code(o, k + 1);
      }
  } else {
    // word w (k rows 2t, 2t+1 | 2t+8, 2t+9): nibbles 0..7 =
    // (g,k) (16+g,k) (g+8,k) (24+g,k) (g,k+1) (16+g,k+1) (g+8,k+1) (24+g,k+1)
    for (int wd = 0; wd < 2; wd++) {
      const int k = kb + 2 * t + 8 * wd;
      const int os[4] = {g, 16 + g, g + 8, 24 + g};
      uint32_t word = 0;
      for (int j = 0; j < 8; j++) word |= code(os[j & 3], k + (j >> 2)) << (4 * j);
      for (int j = 0; j < 4; j++) C[wd * 4 + j] = (uint8_t)(word >> (8 * j));
    }
  }
  if (g == 0) {  // scales: d(2t) d(2t+1) d(2t+8) d(2t+9) (then the mins) of unit u
    for (int which = 0; which < (T == WL_Q4_1 ? 2 : 1); which++) {
      uint16_t* sp = reinterpret_cast<uint16_t*>(D + CODEB + which * 1024 + (u * 4 + t) * 8);
      sp[0] = (uint16_t)scale(kb + 2 * t, which);
      sp[1] = (uint16_t)scale(kb + 2 * t + 1, which);
      sp[2] = (uint16_t)scale(kb + 2 * t + 8, which);
      sp[3] = (uint16_t)scale(kb + 2 * t + 9, which);
    }
  }
}

// K-quant super-blocks (256 columns of one k row, one GEMV group) into the
// same tile geometry.  Codes and scales follow woolly_gguf::dequantize's own
// reading of the blocks (dequantize.rs:381-537), so the tiled product equals
// the dequantized matrix times x:
//   Q4_K (144 bytes): w(i) = d*sc[i/32]*q(i) + dmin, q(i) nibble i%2 of byte
//     16 + i/2, sc the six-bit field of byte 3j/2 (low six bits for even j,
//     top two bits plus the next byte's low nibble for odd j), d and dmin f16
//     at bytes 12 and 14.  Tiled: q as the Q4_1 nibbles, d*sc (exact in f32,
//     <= 17 significant bits) as the f16 pair (hi, lo = d*sc - hi), dmin as
//     the Q4_1 min.
//   Q6_K (210 bytes): w(i) = d*sc[i/16]*(q(i) - 32)/64, q(i) from ql (bytes
//     0-127) and qh (128-191) by the reference's index arithmetic, sc bytes
//     192-207 (unsigned), d f16 at 208.  Tiled: (q - 32) as Q8_0 code bytes,
//     d*sc (<= 19 bits) as an f16 pair per 16 columns; the 1/64 is applied
//     to the f32 accumulator.
// Both splits are exact: d*sc is a multiple of d's f16 quantum (>= 2^-24)
// and has at most 19 significant bits, so lo holds the remaining <= 8 bits.
__device__ __forceinline__ int kq_code(int T, const uint8_t* b, int i) {
  if (T == WL_Q4_K) return (i % 2 == 0) ? (b[16 + i / 2] & 15) : (b[16 + i / 2] >> 4);
  const uint8_t *ql = b, *qh = b + 128;
  const int ql_idx = 64 * (i / 128) + 32 * ((i % 128) / 64) + 16 * ((i % 64) / 32) + (i % 16);
  const int qh_idx = 32 * (i / 128) + 16 * ((i % 128) / 64) + 8 * ((i % 64) / 32) + (i % 32) / 4;
  const int sh = 2 * ((i % 32) % 4);
  const int qv = qh[qh_idx];
  if (i < 128) return (ql[ql_idx] & 15) | (((qv >> sh) & 3) << 4);
  const int ext = sh < 6 ? ((qv >> (sh + 2)) & 3) : (qh_idx + 1 < 64 ? (qh[qh_idx + 1] & 3) : 0);
  return (ql[ql_idx] >> 4) | (ext << 4);
}
__device__ __forceinline__ float kq_scale(int T, const uint8_t* b, int j) {
  if (T == WL_Q4_K) {
    const int src = (j * 3) / 2;
    const int sc = (j % 2 == 0) ? (b[src] & 63) : (((b[src] >> 6) | ((b[src + 1] & 15) << 2)) & 63);
    return __fmul_rn(__half2float(__ushort_as_half((uint16_t)(b[12] | (b[13] << 8)))), (float)sc);
  }
  return __fmul_rn(__half2float(__ushort_as_half((uint16_t)(b[208] | (b[209] << 8)))), (float)b[192 + j]);
}

template <int T>
__global__ void k_repack_tiled_k(const uint8_t* src, int K, int pitch, uint8_t* dst, int stages,
                                 size_t total) {
  constexpr int STB = 512 * QT<T>::S;
  constexpr int CB = T == WL_Q6_K ? 16 : 8;
  constexpr int CODEB = 1024 * CB;
  constexpr int SBB = T == WL_Q4_K ? 144 : 210;
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int lane = (int)(i & 31), u = (int)((i >> 5) & 31);
  const size_t gs = i >> 10;
  const int stage = (int)(gs % stages);
  const int group = (int)(gs / stages);  // = super-block column index
  const int w = u >> 3, ks = (u >> 1) & 3, blk = u & 1;
  const int j32 = w * 2 + blk;  // 32-column unit within the super-block
  const int g = lane >> 2, t = lane & 3;
  const int kb = stage * kRows + ks * 16;
  uint8_t* D = dst + gs * STB;
  auto sb = [&](int k) { return src + (size_t)k * pitch + (size_t)group * SBB; };
  auto code = [&](int o, int k) -> uint32_t {  // output o (0..31) of the unit at k row k
    if (k >= K) return 0u;
    const int q = kq_code(T, sb(k), j32 * 32 + o);
    return T == WL_Q6_K ? (uint32_t)(uint8_t)(int8_t)(q - 32) : (uint32_t)q;
  };
  uint8_t* C = D + u * (32 * CB) + lane * CB;
  if (T == WL_Q6_K) {
    for (int mt = 0; mt < 2; mt++)
      for (int r = 0; r < 4; r++) {
        const int o = mt * 16 + g + 8 * (r & 1), k = kb + 2 * t + 8 * (r >> 1);
        C[(mt * 4 + r) * 2] = (uint8_t)code(o, k);
        C[(mt * 4 + r) * 2 + 1] = (uint8_t)code(o, k + 1);
      }
  } else {
    for (int wd = 0; wd < 2; wd++) {
      const int k = kb + 2 * t + 8 * wd;
      const int os[4] = {g, 16 + g, g + 8, 24 + g};
      uint32_t word = 0;
      for (int jj = 0; jj < 8; jj++) word |= code(os[jj & 3], k + (jj >> 2)) << (4 * jj);
      for (int jj = 0; jj < 4; jj++) C[wd * 4 + jj] = (uint8_t)(word >> (8 * jj));
    }
  }
  if (g != 0) return;
  const int rows[4] = {kb + 2 * t, kb + 2 * t + 1, kb + 2 * t + 8, kb + 2 * t + 9};
  for (int mt = 0; mt < (T == WL_Q6_K ? 2 : 1); mt++) {
    uint16_t* sp = reinterpret_cast<uint16_t*>(D + CODEB + ((T == WL_Q6_K ? u * 8 + mt * 4 : u * 4) + t) * 16);
    for (int r = 0; r < 4; r++) {
      const float sv = rows[r] < K ? kq_scale(T, sb(rows[r]), T == WL_Q6_K ? j32 * 2 + mt : j32) : 0.f;
      const __half hi = __float2half_rn(sv);
      const __half lo = __float2half_rn(sv - __half2float(hi));
      sp[r] = __half_as_ushort(hi);
      sp[4 + r] = __half_as_ushort(lo);
    }
  }
  if (T == WL_Q4_K) {
    uint16_t* mp = reinterpret_cast<uint16_t*>(D + CODEB + 2048 + (u * 4 + t) * 8);
    for (int r = 0; r < 4; r++) {
      const uint8_t* b = rows[r] < K ? sb(rows[r]) : nullptr;
      mp[r] = b ? (uint16_t)(b[14] | (b[15] << 8)) : (uint16_t)0;
    }
  }
}

template <int T>
int repack_tiled_t(const uint8_t* src, int K, int N, int pitch, uint8_t* dst, cudaStream_t st) {
  const int groups = (N + kColsB - 1) / kColsB, stages = (K + kRows - 1) / kRows;
  const size_t total = (size_t)groups * stages * 1024;
  if (!total) return WL_OK;
  if constexpr (kKq<T>)
    k_repack_tiled_k<T><<<(unsigned)((total + 255) / 256), 256, 0, st>>>(src, K, pitch, dst, stages, total);
  else
    k_repack_tiled<T><<<(unsigned)((total + 255) / 256), 256, 0, st>>>(src, K, N, pitch, dst, stages, total);
  WL_CUDA_TRY(cudaGetLastError());
  return WL_OK;
}

// ------------------------------------------------------------------ layout A, K-quants
// ggml orientation (rows of K values, 256-value super-blocks along K), the
// values woolly_gguf::dequantize reads (dequantize.rs:381-537).  The loader
// keeps each row's super-blocks padded to 16-byte multiples (Q4_K 144 bytes,
// Q6_K 210 -> 224: launch_kq_pad) so that a stage (256 k = one super-block
// per row) is 9 or 14 aligned cp.async chunks.  Per 32-value (Q4_K) or
// 16-value (Q6_K) sub-block: the integer codes enter the MMA as exact f16
// (q, or q - 32), the activations as hi/lo planes, and each row's partial
// sum is scaled in f32 by d*sc (Q6_K: /64); Q4_K's dmin is added once per
// value as dmin * sum(x) through a ones-matrix MMA.
template <int T>
constexpr int kSBP = T == WL_Q4_K ? 144 : 224;  // padded super-block bytes

__global__ void k_kq_pad(const uint8_t* src, size_t src_pitch, int rows, int nsb, int sb, int sbp,
                         uint8_t* dst) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t row_bytes = (size_t)nsb * sbp;
  if (i >= row_bytes * rows) return;
  const size_t r = i / row_bytes, o = i % row_bytes;
  const int j = (int)(o / sbp), b = (int)(o % sbp);
  dst[i] = b < sb ? src[r * src_pitch + (size_t)j * sb + b] : 0;
}

__device__ __forceinline__ uint32_t nib_pair(uint32_t b) {  // byte -> exact f16 (low, high nibble)
  return hsub2u(((b & 0xFu) | ((b & 0xF0u) << 12)) | kMagic, kMagic);
}
__device__ __forceinline__ uint32_t q6_pair(const uint8_t* sb, int i) {  // exact f16 (q(i)-32, q(i+1)-32)
  const uint32_t v = (uint32_t)kq_code(WL_Q6_K, sb, i) | ((uint32_t)kq_code(WL_Q6_K, sb, i + 1) << 16);
  return hsub2u(v | kMagic, 0x64206420u);
}
__device__ __forceinline__ float q4k_scale(const uint8_t* sb, int j) {
  const int src = (j * 3) / 2;
  const int sc = (j % 2 == 0) ? (sb[src] & 63) : (((sb[src] >> 6) | ((sb[src + 1] & 15) << 2)) & 63);
  return __fmul_rn(__half2float(__ushort_as_half((uint16_t)(sb[12] | (sb[13] << 8)))), (float)sc);
}

template <int T, int NT>
__global__ void __launch_bounds__(kThreads) k_qgemv_ak(const GemvArgs a) {
  constexpr int BP = NT * 8;
  constexpr int KS = 256;
  constexpr int SBP = kSBP<T>;
  constexpr int SP = SBP + 16;  // shared row pitch (rows of a warp start in different banks)
  constexpr int RAW = kColsA * SP;
  constexpr int CH = SBP / 16;
  constexpr int STG = NT <= 2 ? kStages : 2;
  constexpr int SST = RAW + BP * KS * 4;
  constexpr int XP = KS + 8;
  constexpr int PIPE = STG * SST > BP * (kColsA + 4) * 4 ? STG * SST : BP * (kColsA + 4) * 4;
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* raw = smem;
  pdl_wait();
  pdl_trigger();
  __half* xs = reinterpret_cast<__half*>(smem + PIPE);
  const __half* xl_base = xs + BP * XP;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int gx = blockIdx.x, split = blockIdx.y;
  const GemvSeg& S = a.seg[0];
  const int n0 = gx * kColsA;
  const int k0 = split * a.kchunk;
  const int k1 = min(a.K, k0 + a.kchunk);
  const int nstage = k1 > k0 ? (k1 - k0) / KS : 0;
  const int ncv = min(kColsA, S.N - n0);
  __shared__ uint64_t red_bar;
  ClusterRed R;
  red_begin(R, a, 0, ncv, &red_bar, smem + PIPE + 2 * BP * XP * 2);

  auto load_stage = [&](int st, int buf) {
    const size_t byte0 = (size_t)((k0 + st * KS) / KS) * SBP;
    uint8_t* dst = raw + buf * SST;
    for (int i = tid; i < kColsA * CH; i += kThreads) {
      const int r = i / CH, c = i - r * CH;
      const int row = n0 + r;
      const bool ok = row < S.N;
      cp_async16(dst + r * SP + c * 16, S.W + (size_t)(ok ? row : 0) * S.pitch + byte0 + c * 16,
                 ok ? 16 : 0);
    }
    load_x_f32(a, reinterpret_cast<float*>(dst + RAW), BP, KS, k0 + st * KS, k1);
  };
#pragma unroll
  for (int s = 0; s < STG - 1; s++) {
    if (s < nstage) load_stage(s, s);
    cp_commit();
  }
  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; n++)
#pragma unroll
    for (int q = 0; q < 4; q++) acc[n][q] = 0.f;
  const uint32_t ones[4] = {kOnes, kOnes, kOnes, kOnes};

  for (int st = 0; st < nstage; st++) {
    cp_wait<STG - 2>();
    __syncthreads();
    {
      const int nx = st + STG - 1;
      if (nx < nstage) load_stage(nx, nx % STG);
      cp_commit();
    }
    split_tile(reinterpret_cast<const float*>(raw + (st % STG) * SST + RAW), xs, BP, KS, XP);
    __syncthreads();
    const uint8_t* rA = raw + (st % STG) * SST + (warp * 16 + g) * SP;  // rows g and g + 8 of the warp
    const uint8_t* rB = rA + 8 * SP;
    // the activation B fragments of k step [kk, kk + 16) for batch tile n
    auto xfrag = [&](int n, int kk, uint32_t& h0, uint32_t& h1, uint32_t& l0, uint32_t& l1) {
      const __half* xp = xs + (n * 8 + g) * XP + kk + 2 * t;
      const __half* lp = xl_base + (n * 8 + g) * XP + kk + 2 * t;
      h0 = *reinterpret_cast<const uint32_t*>(xp);
      h1 = *reinterpret_cast<const uint32_t*>(xp + 8);
      l0 = *reinterpret_cast<const uint32_t*>(lp);
      l1 = *reinterpret_cast<const uint32_t*>(lp + 8);
    };
    if constexpr (T == WL_Q4_K) {
      const float mA = __half2float(__ushort_as_half((uint16_t)(rA[14] | (rA[15] << 8))));
      const float mB = __half2float(__ushort_as_half((uint16_t)(rB[14] | (rB[15] << 8))));
#pragma unroll 2
      for (int j = 0; j < 8; j++) {
        const float sA = q4k_scale(rA, j), sB = q4k_scale(rB, j);
        uint32_t af[2][4];
#pragma unroll
        for (int s2 = 0; s2 < 2; s2++) {  // byte of k = j*32 + s2*16 + 2t (low nibble) and + 1 (high)
          const int o = 16 + j * 16 + s2 * 8 + t;
          af[s2][0] = nib_pair(rA[o]);
          af[s2][1] = nib_pair(rB[o]);
          af[s2][2] = nib_pair(rA[o + 4]);
          af[s2][3] = nib_pair(rB[o + 4]);
        }
#pragma unroll
        for (int n = 0; n < NT; n++) {
          float c[4] = {0.f, 0.f, 0.f, 0.f}, cm[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int s2 = 0; s2 < 2; s2++) {
            uint32_t h0, h1, l0, l1;
            xfrag(n, j * 32 + s2 * 16, h0, h1, l0, l1);
            mma16816(c, af[s2], h0, h1);
            mma16816(c, af[s2], l0, l1);
            mma16816(cm, ones, h0, h1);
            mma16816(cm, ones, l0, l1);
          }
          acc[n][0] += sA * c[0] + mA * cm[0];
          acc[n][1] += sA * c[1] + mA * cm[1];
          acc[n][2] += sB * c[2] + mB * cm[2];
          acc[n][3] += sB * c[3] + mB * cm[3];
        }
      }
    } else {
      const float dA = __half2float(__ushort_as_half((uint16_t)(rA[208] | (rA[209] << 8)))) * 0.015625f;
      const float dB = __half2float(__ushort_as_half((uint16_t)(rB[208] | (rB[209] << 8)))) * 0.015625f;
#pragma unroll 2
      for (int j = 0; j < 16; j++) {  // 16-value sub-blocks: one k step each
        const float sA = dA * (float)rA[192 + j], sB = dB * (float)rB[192 + j];
        const int kk = j * 16;
        uint32_t af[4];
        af[0] = q6_pair(rA, kk + 2 * t);
        af[1] = q6_pair(rB, kk + 2 * t);
        af[2] = q6_pair(rA, kk + 8 + 2 * t);
        af[3] = q6_pair(rB, kk + 8 + 2 * t);
#pragma unroll
        for (int n = 0; n < NT; n++) {
          float c[4] = {0.f, 0.f, 0.f, 0.f};
          uint32_t h0, h1, l0, l1;
          xfrag(n, kk, h0, h1, l0, l1);
          mma16816(c, af, h0, h1);
          mma16816(c, af, l0, l1);
          acc[n][0] += sA * c[0];
          acc[n][1] += sA * c[1];
          acc[n][2] += sB * c[2];
          acc[n][3] += sB * c[3];
        }
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
      const int b = n * 8 + 2 * t + (q & 1);
      const int c = warp * 16 + g + 8 * (q >> 1);
      tile[b * TP + c] = acc[n][q];
    }
  __syncthreads();
  cluster_finish(a, R, tile, TP, ncv, 0, n0);
}

template <int T>
size_t smem_ak(int NT) {
  const size_t BP = (size_t)NT * 8;
  const int stg = NT <= 2 ? kStages : 2;
  const size_t pipe = (size_t)stg * (kColsA * (kSBP<T> + 16) + BP * 256 * 4);
  const size_t tile = BP * (kColsA + 4) * 4;
  const size_t xs = 2 * BP * (256 + 8) * 2;
  return std::max(pipe, tile) + xs + recv_bytes((int)BP, kColsA);
}

template <int T, int NT>
int launch_ak_t(const GemvArgs& a, cudaStream_t st) {
  return launch_cluster(k_qgemv_ak<T, NT>, dim3(a.seg[0].groups, a.csplit), kThreads, smem_ak<T>(NT), 1,
                        a.csplit, a, st);
}

template <int T>
int dispatch_ak(const GemvArgs& a, cudaStream_t st) {
  switch ((a.B + 7) / 8) {
    case 1: return launch_ak_t<T, 1>(a, st);
    case 2: return launch_ak_t<T, 2>(a, st);
    case 3: return launch_ak_t<T, 3>(a, st);
    case 4: return launch_ak_t<T, 4>(a, st);
  }
  return fail(WL_ERR_INVALID_ARGUMENT, "qgemv: B must be 1..32 per launch");
}

template <int T, int NT, bool LOC = false, bool TLD = false>
int launch_b_t(const GemvArgs& a, cudaStream_t st) {
  int groups = 0;
  for (int s = 0; s < a.nseg; s++) groups += a.seg[s].groups;
  const bool sw = a.epi.kind == EPI_SWIGLU;
  return launch_cluster(k_qgemv_b<T, NT, LOC, TLD>, dim3(groups, a.csplit), kThreadsB, smem_b<T>(NT),
                        sw ? 2 : 1,
                        a.csplit, a, st);
}

template <int T, int NT>
int launch_a_t(const GemvArgs& a, cudaStream_t st) {
  return launch_cluster(k_qgemv_a<T, NT>, dim3(a.seg[0].groups, a.csplit), kThreads,
                        smem_a<T>(NT), 1,
                        a.csplit, a, st);
}

template <int T, bool TLD>
int dispatch_b(const GemvArgs& a, cudaStream_t st) {
  switch ((a.B + 7) / 8) {
    case 1: return a.B <= 4 ? launch_b_t<T, 1, true, TLD>(a, st) : launch_b_t<T, 1, false, TLD>(a, st);
    case 2: return launch_b_t<T, 2, false, TLD>(a, st);
    case 3: return launch_b_t<T, 3, false, TLD>(a, st);
    case 4: return launch_b_t<T, 4, false, TLD>(a, st);
  }
  return fail(WL_ERR_INVALID_ARGUMENT, "qgemv: B must be 1..32 per launch");
}

template <int T, bool LB>
int dispatch(const GemvArgs& a, cudaStream_t st) {
  if constexpr (kKq<T>) {
    if (!LB || !a.tiled) return fail(WL_ERR_UNSUPPORTED, "qgemv: K-quant weights run from their tiled copy only");
    return dispatch_b<T, true>(a, st);
  } else {
    if (LB) return a.tiled ? dispatch_b<T, true>(a, st) : dispatch_b<T, false>(a, st);
    switch ((a.B + 7) / 8) {
      case 1: return launch_a_t<T, 1>(a, st);
      case 2: return launch_a_t<T, 2>(a, st);
      case 3: return launch_a_t<T, 3>(a, st);
      case 4: return launch_a_t<T, 4>(a, st);
    }
    return fail(WL_ERR_INVALID_ARGUMENT, "qgemv: B must be 1..32 per launch");
  }
}

int block_bytes(int type) { return type == WL_Q4_0 ? 18 : type == WL_Q4_1 ? 20 : type == WL_Q8_0 ? 34 : 0; }
// bytes of one 32-column unit of one k row in the tiled copy
int unit_bytes(int type) {
  switch (type) {
    case WL_Q4_0: return QT<WL_Q4_0>::S;
    case WL_Q4_1: return QT<WL_Q4_1>::S;
    case WL_Q8_0: return QT<WL_Q8_0>::S;
    case WL_Q4_K: return QT<WL_Q4_K>::S;
    case WL_Q6_K: return QT<WL_Q6_K>::S;
  }
  return 0;
}
size_t smem_b_type(int type, int NT) {
  switch (type) {
    case WL_Q4_1: return smem_b<WL_Q4_1>(NT);
    case WL_Q8_0: return smem_b<WL_Q8_0>(NT);
    case WL_Q4_K: return smem_b<WL_Q4_K>(NT);
    case WL_Q6_K: return smem_b<WL_Q6_K>(NT);
  }
  return smem_b<WL_Q4_0>(NT);
}

}  // namespace

bool kquant_type(int type) { return type == WL_Q4_K || type == WL_Q6_K; }
int kquant_block_bytes(int type) { return type == WL_Q4_K ? 144 : type == WL_Q6_K ? 210 : 0; }
int kq_padded_bytes(int type) { return type == WL_Q4_K ? kSBP<WL_Q4_K> : type == WL_Q6_K ? kSBP<WL_Q6_K> : 0; }

int launch_kq_pad(int type, const uint8_t* src, size_t src_pitch, int rows, int K, uint8_t* dst,
                  cudaStream_t st) {
  if (!kquant_type(type) || K % 256 || rows <= 0) return fail(WL_ERR_INVALID_ARGUMENT, "kq_pad: bad shape");
  const int nsb = K / 256, sb = kquant_block_bytes(type), sbp = kq_padded_bytes(type);
  const size_t total = (size_t)rows * nsb * sbp;
  k_kq_pad<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(src, src_pitch, rows, nsb, sb, sbp, dst);
  WL_CUDA_TRY(cudaGetLastError());
  return WL_OK;
}

int qgemv_group_cols(int layout) { return layout == WL_LAYOUT_B ? kColsB : kColsA; }

// Layout B needs 16-byte aligned rows (pitch % 16 == 0, padding allowed) and
// 16 readable bytes past the last row's payload (the tail chunk of a partial
// group may straddle the end of the payload); K a multiple of 16.
bool qgemv_b_fast_ok(int type, int K, int N, int pitch, const void* W) {
  if (kquant_type(type))  // the repack reads any pitch; the GEMV reads the tiled copy
    return K % 16 == 0 && K > 0 && N % 256 == 0 && N > 0 && pitch >= N / 256 * kquant_block_bytes(type);
  const int S = block_bytes(type);
  if (!S) return false;
  return K % 16 == 0 && K > 0 && N % 32 == 0 && pitch % 16 == 0 && pitch >= N / 32 * S &&
         (reinterpret_cast<uintptr_t>(W) & 15) == 0;
}

bool qgemv_a_fast_ok(int type, int K, int N, int pitch, const void* W) {
  if (kquant_type(type))  // padded super-blocks (launch_kq_pad)
    return K % 256 == 0 && K > 0 && pitch == K / 256 * kq_padded_bytes(type) &&
           (reinterpret_cast<uintptr_t>(W) & 15) == 0;
  const int S = block_bytes(type);
  if (!S) return false;
  (void)N;
  return K % 256 == 0 && pitch % 16 == 0 && pitch == K / 32 * S &&
         (reinterpret_cast<uintptr_t>(W) & 15) == 0;
}

namespace {
// Layout-B kernel instance a launch of `a` uses (as dispatch_b picks it).
using KernB = void (*)(const GemvArgs);
template <int T, bool TLD>
KernB kernel_b_t(int B) {
  switch ((B + 7) / 8) {
    case 1: return B <= 4 ? k_qgemv_b<T, 1, true, TLD> : k_qgemv_b<T, 1, false, TLD>;
    case 2: return k_qgemv_b<T, 2, false, TLD>;
    case 3: return k_qgemv_b<T, 3, false, TLD>;
    default: return k_qgemv_b<T, 4, false, TLD>;
  }
}
KernB kernel_b(const GemvArgs& a) {
  if (a.type == WL_Q4_0) return a.tiled ? kernel_b_t<WL_Q4_0, true>(a.B) : kernel_b_t<WL_Q4_0, false>(a.B);
  if (a.type == WL_Q4_1) return a.tiled ? kernel_b_t<WL_Q4_1, true>(a.B) : kernel_b_t<WL_Q4_1, false>(a.B);
  if (a.type == WL_Q4_K) return kernel_b_t<WL_Q4_K, true>(a.B);
  if (a.type == WL_Q6_K) return kernel_b_t<WL_Q6_K, true>(a.B);
  return a.tiled ? kernel_b_t<WL_Q8_0, true>(a.B) : kernel_b_t<WL_Q8_0, false>(a.B);
}

std::mutex g_cap_mu;
std::map<std::tuple<int, const void*, int, int, size_t>, int> g_cap;

// CTAs of (cx, cy) clusters of the kernel that can be resident at once on
// this device (registers, shared memory and cluster placement together),
// from the occupancy calculator; cached per (device, kernel, cluster shape).
// A grid larger than this runs in two waves.
int cluster_capacity(KernB k, int cx, int cy, size_t smem) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const auto key = std::make_tuple(dev, (const void*)k, cx, cy, smem);
  {
    std::lock_guard<std::mutex> lk(g_cap_mu);
    auto it = g_cap.find(key);
    if (it != g_cap.end()) return it->second;
  }
  // the launch path sets these too; the occupancy query needs them first
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cx, cy);
  cfg.blockDim = dim3(kThreadsB);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeClusterDimension;
  at.val.clusterDim.x = cx;
  at.val.clusterDim.y = cy;
  at.val.clusterDim.z = 1;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = -1;  // unknown: do not constrain the plan
  }
  const int cap = n < 0 ? INT32_MAX : n * cx * cy;
  std::lock_guard<std::mutex> lk(g_cap_mu);
  g_cap[key] = cap;
  return cap;
}
}  // namespace

void qgemv_plan(GemvArgs& a, int layout, int num_sms) {
  int groups = 0;
  for (int s = 0; s < a.nseg; s++) groups += a.seg[s].groups;
  const int gran = layout == WL_LAYOUT_B ? (a.tiled ? kRows : 16) : 256;
  const int units = (a.K + gran - 1) / gran;
  int per_sm = 2;
  if (layout == WL_LAYOUT_B) {
    const int NT = (std::min(a.B, 32) + 7) / 8;
    const size_t sm = smem_b_type(a.type, NT);
    per_sm = std::max(1, std::min(kPlanCtasPerSm, (int)(kSmemPerSm / (sm + 2048))));
  }
  const int target = per_sm * num_sms;
  const int cmax = a.epi.kind == EPI_SWIGLU ? kMaxCluster / 2 : kMaxCluster;
  // round down: every CTA resident in one wave
  int c = target / std::max(groups, 1);
  c = std::max(1, std::min({c, cmax, units}));
  a.kchunk = (units + c - 1) / c * gran;
  a.csplit = (a.K + a.kchunk - 1) / a.kchunk;
  if (layout != WL_LAYOUT_B) return;
  // clusters must also fit one wave: a GPC holds whole clusters only, so a
  // split that fits by CTA count can still leave CTAs for a second wave
  const int NT = (std::min(a.B, 32) + 7) / 8;
  const size_t sm = smem_b_type(a.type, NT);
  const int cx = a.epi.kind == EPI_SWIGLU ? 2 : 1;
  const KernB k = kernel_b(a);
  while (a.csplit > 1 && groups * a.csplit > cluster_capacity(k, cx, a.csplit, sm)) {
    c = a.csplit - 1;
    a.kchunk = (units + c - 1) / c * gran;
    a.csplit = (a.K + a.kchunk - 1) / a.kchunk;
  }
}

size_t qtile_bytes(int type, int K, int N) {
  if (kquant_type(type) && N % 256) return 0;
  const int S = unit_bytes(type);
  return (size_t)((N + kColsB - 1) / kColsB) * ((K + kRows - 1) / kRows) * 512 * S;
}

int launch_repack_tiled(int type, const uint8_t* src, int K, int N, int pitch, uint8_t* dst,
                        cudaStream_t st) {
  if (N % 32 || K <= 0) return fail(WL_ERR_INVALID_ARGUMENT, "repack: N % 32 != 0 or K <= 0");
  switch (type) {
    case WL_Q4_0: return repack_tiled_t<WL_Q4_0>(src, K, N, pitch, dst, st);
    case WL_Q4_1: return repack_tiled_t<WL_Q4_1>(src, K, N, pitch, dst, st);
    case WL_Q8_0: return repack_tiled_t<WL_Q8_0>(src, K, N, pitch, dst, st);
    case WL_Q4_K:
    case WL_Q6_K:
      if (N % 256) return fail(WL_ERR_INVALID_ARGUMENT, "repack: K-quant N % 256 != 0");
      return type == WL_Q4_K ? repack_tiled_t<WL_Q4_K>(src, K, N, pitch, dst, st)
                             : repack_tiled_t<WL_Q6_K>(src, K, N, pitch, dst, st);
  }
  return fail(WL_ERR_UNSUPPORTED, "repack: unsupported type " + std::to_string(type));
}

int launch_qgemv_b(const GemvArgs& a, cudaStream_t st) {
  switch (a.type) {
    case WL_Q4_0: return dispatch<WL_Q4_0, true>(a, st);
    case WL_Q4_1: return dispatch<WL_Q4_1, true>(a, st);
    case WL_Q8_0: return dispatch<WL_Q8_0, true>(a, st);
    case WL_Q4_K: return dispatch<WL_Q4_K, true>(a, st);
    case WL_Q6_K: return dispatch<WL_Q6_K, true>(a, st);
  }
  return fail(WL_ERR_UNSUPPORTED, "qgemv: unsupported type " + std::to_string(a.type));
}

int launch_qgemv_a(const GemvArgs& a, cudaStream_t st) {
  switch (a.type) {
    case WL_Q4_K: return dispatch_ak<WL_Q4_K>(a, st);
    case WL_Q6_K: return dispatch_ak<WL_Q6_K>(a, st);
    case WL_Q4_0: return dispatch<WL_Q4_0, false>(a, st);
    case WL_Q4_1: return dispatch<WL_Q4_1, false>(a, st);
    case WL_Q8_0: return dispatch<WL_Q8_0, false>(a, st);
  }
  return fail(WL_ERR_UNSUPPORTED, "qgemv: unsupported type " + std::to_string(a.type));
}

int launch_qgemv_generic(int type, int layout, const uint8_t* W, int K, int N, int pitch,
                         const void* x, size_t x_plane, int ldx, int B, float* y, int ldy,
                         bool add, cudaStream_t st) {
  if (!block_bytes(type) && type != WL_F32) return fail(WL_ERR_UNSUPPORTED, "qgemv: unsupported type");
  dim3 grid((N + 127) / 128, B);
  k_qgemv_generic<<<grid, 128, 0, st>>>(type, layout, W, K, N, pitch, x, x_plane, ldx, B, y, ldy,
                                        add);
  WL_CUDA_TRY(cudaGetLastError());
  return WL_OK;
}

int launch_split_planes(const float* x, __half* y, size_t n, size_t plane, cudaStream_t st) {
  if (!n) return WL_OK;
  k_split_planes<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, y, n, plane);
  WL_CUDA_TRY(cudaGetLastError());
  return WL_OK;
}

}  // namespace wl
