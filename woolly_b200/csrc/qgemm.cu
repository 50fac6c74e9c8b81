// Prefill GEMM on the 5th-generation tensor cores (tcgen05 MMA, TMEM
// accumulators) for layout-B quantized weights.
//
// Y[m][n] = sum_k X[m][k] * W[k][n] for M token rows at once (woolly's
// layout-B matmul, tensor_utils.rs:118-157, applied to a whole prompt).  One
// CTA computes 128 weight columns x 128 token rows.  Per 64-row k stage:
//   * the 8 warps dequantize the stage's Q4_0 / Q4_1 / Q8_0 blocks straight
//     into shared memory as f16 hi/lo pairs with W = Whi + Wlo exactly
//     (Q4_0 / Q8_0: Whi = f16(q*d) by HMUL2, Wlo = fma(q, d, -Whi) by HFMA2,
//     the residual being exact in f16; Q4_1 in f32), laid out N-major with
//     the 128-byte swizzle (a layout-B row already runs along N, so no
//     transpose);
//   * the activation hi/lo planes are copied in K-major with the same swizzle;
//   * one thread issues 3 MMAs per 16-k step into the TMEM accumulator:
//     Xhi*Whi + Xhi*Wlo + Xlo*Whi (the dropped Xlo*Wlo term is ~2^-22 of the
//     product), then commits the stage to an mbarrier that gates its reuse.
// A 3-slot ring software-pipelines the stages: while stage i is dequantized
// and multiplied, stage i+1's activation copies and raw weight loads are in
// flight.  The epilogue reads the accumulator with tcgen05.ld (warp w owns
// TMEM lanes 32w..32w+31 = weight columns) and applies the same F32 / ADD /
// QKV / SwiGLU outputs as the decode GEMV.  Every mbarrier wait is bounded; on
// expiry the kernel raises an error bit, waits (bounded) for its issued MMAs
// and frees its TMEM before returning.
#include <cuda_fp16.h>

#include <cstdint>
#include <cstring>
#include <string>

#include "common.h"
#include "pdl.cuh"
#include "qgemv.cuh"

namespace wl {
namespace {

constexpr int kGN = 128;  // weight columns per CTA (MMA M)
constexpr int kGM = 128;  // token rows per CTA (MMA N)
constexpr int kGK = 64;   // k rows per stage (one 128-byte swizzle row of f16)
constexpr int kGStages = 3;
constexpr int kGThreads = 512;  // 16 warps: two per quant block of each k row
constexpr int kGTile = 128 * kGK * 2;  // bytes of one f16 operand tile (16 KB)
constexpr int kGStage = 4 * kGTile;    // W hi, W lo, X hi, X lo
constexpr int kGSmem = kGStages * kGStage + 1024 + 64;  // + alignment slack + barriers
constexpr int kTmemCols = kGM;                          // f32 accumulator columns (token rows)

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// tcgen05 shared-memory matrix descriptor: start, leading and stride byte
// offsets (16-byte units), descriptor version 1, 128-byte swizzle (layout 2).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// instruction descriptor, kind::f16: D f32, A and B f16, A N-major (bit 15),
// B K-major, N = kGM (bits 17-22, /8), M = kGN (bits 24-28, /16)
constexpr uint32_t kIdesc = (1u << 4) | (1u << 15) | ((uint32_t)(kGM >> 3) << 17) |
                            ((uint32_t)(kGN >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t da, uint64_t db, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
      "l"(da), "l"(db), "r"(kIdesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ bool gbar_wait(uint32_t bar, uint32_t phase) {
  for (int it = 0; it < (1 << 22); it++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(phase)
        : "memory");
    if (ok) return true;
  }
  return false;
}

__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0)
               : "memory");
}

__device__ __forceinline__ uint32_t h2u(__half2 h) {
  uint32_t u;
  memcpy(&u, &h, 4);
  return u;
}
__device__ __forceinline__ __half2 u2h(uint32_t u) {
  __half2 h;
  memcpy(&h, &u, 4);
  return h;
}

// q pair (exact f16 codes) x d -> hi, lo with hi + lo = q*d exactly
__device__ __forceinline__ void split_pair(uint32_t q, __half2 d2, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __hmul2(u2h(q), d2);
  hi = h2u(h);
  lo = h2u(__hfma2(u2h(q), d2, __hneg2(h)));
}

// Half a quant block's bytes held in registers as 16-bit words (blocks are only
// 2-byte aligned in a layout-B row): the scale (Q4_1: and min) plus the code
// words of the half.  Q4_0 / Q4_1 half p holds code bytes 8p..8p+7 (columns
// 8p..8p+7 and 16+8p..23+8p); Q8_0 half p holds codes 16p..16p+15.
template <int T>
struct RawBlock {
  static constexpr int HDR = T == WL_Q4_1 ? 2 : 1;  // words before the codes
  static constexpr int CW = T == WL_Q8_0 ? 8 : 4;   // code words per half
  uint16_t w[HDR + CW];
};
template <int T>
__device__ __forceinline__ void raw_load(RawBlock<T>& r, const uint8_t* blk, int part, bool live) {
  using R = RawBlock<T>;
  const unsigned short* p = reinterpret_cast<const unsigned short*>(blk);
#pragma unroll
  for (int i = 0; i < R::HDR; i++) r.w[i] = live ? __ldg(p + i) : (unsigned short)0;
#pragma unroll
  for (int i = 0; i < R::CW; i++) r.w[R::HDR + i] = live ? __ldg(p + R::HDR + part * R::CW + i) : (unsigned short)0;
}

// Dequantizes half (`part`) of one quant block (16 of its 32 columns) of k row
// `kk` of the stage into the hi and lo tiles; the block is columns b*32.. of
// the tile.
template <int T>
__device__ __forceinline__ void dequant_half(const RawBlock<T>& raw, uint8_t* whi, uint8_t* wlo,
                                             int kk, int b, int part, bool live) {
  constexpr int H = RawBlock<T>::HDR;
  uint32_t hi[8], lo[8];  // two 8-column chunks: pairs 0-3 -> chunk A, 4-7 -> chunk B
  int chA, chB;           // chunk indices (8 columns each) within the block
  if constexpr (T == WL_Q8_0) {
    chA = 2 * part;
    chB = 2 * part + 1;
  } else {
    chA = part;      // low nibbles: columns 8p..8p+7
    chB = 2 + part;  // high nibbles: columns 16+8p..
  }
  if (!live) {
#pragma unroll
    for (int j = 0; j < 8; j++) hi[j] = lo[j] = 0u;
  } else if constexpr (T == WL_Q4_1) {
    const float d = __half2float(__ushort_as_half(raw.w[0]));
    const float m = __half2float(__ushort_as_half(raw.w[1]));
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint32_t w = raw.w[H + j];
      const float q[4] = {(float)(w & 15u), (float)((w >> 8) & 15u), (float)((w >> 4) & 15u),
                          (float)((w >> 12) & 15u)};
      __half hh[4], hl[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float v = q[u] * d + m;  // q*d + m (dequantize_q4_1, dequantize.rs:372)
        hh[u] = __float2half_rn(v);
        hl[u] = __float2half_rn(v - __half2float(hh[u]));
      }
      hi[j] = h2u(__halves2half2(hh[0], hh[1]));
      lo[j] = h2u(__halves2half2(hl[0], hl[1]));
      hi[4 + j] = h2u(__halves2half2(hh[2], hh[3]));
      lo[4 + j] = h2u(__halves2half2(hl[2], hl[3]));
    }
  } else if constexpr (T == WL_Q8_0) {
    const __half dh = __ushort_as_half(raw.w[0]);
    const __half2 d2 = __halves2half2(dh, dh);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const uint32_t w = raw.w[H + j];  // codes of columns 16p+2j, 16p+2j+1
      const uint32_t v = ((w & 0xFFu) | ((w & 0xFF00u) << 8)) ^ 0x00800080u;
      const uint32_t q = h2u(__hsub2(u2h(v | 0x64006400u), u2h(0x64806480u)));  // exact int8
      split_pair(q, d2, hi[j], lo[j]);
    }
  } else {  // Q4_0: (q - 8) * d (dequantize_q4_0, dequantize.rs:315-321)
    const __half dh = __ushort_as_half(raw.w[0]);
    const __half2 d2 = __halves2half2(dh, dh);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint32_t w = raw.w[H + j];                                     // bytes 8p+2j, +1
      const uint32_t lo_n = (w & 0x000Fu) | ((w & 0x0F00u) << 8);         // low nibbles
      const uint32_t hi_n = ((w & 0x00F0u) >> 4) | ((w & 0xF000u) << 4);  // high nibbles
      const uint32_t qa = h2u(__hsub2(u2h(lo_n | 0x64006400u), u2h(0x64086408u)));
      const uint32_t qb = h2u(__hsub2(u2h(hi_n | 0x64006400u), u2h(0x64086408u)));
      split_pair(qa, d2, hi[j], lo[j]);
      split_pair(qb, d2, hi[4 + j], lo[4 + j]);
    }
  }
  // column c of the tile: 64-column block jb = c / 64, 16-byte chunk c8 = (c % 64) / 8;
  // N-major 128B-swizzled atom (k group g = kk / 8, jb) holds 8 k rows of 128 bytes
  const int g = kk >> 3, r = kk & 7;
#pragma unroll
  for (int q = 0; q < 2; q++) {
    const int c = b * 32 + (q ? chB : chA) * 8;
    const int jb = c >> 6, c8 = (c & 63) >> 3;
    const uint32_t off = (uint32_t)(((g * 2 + jb) << 10) + (r << 7) + ((c8 ^ r) << 4));
    *reinterpret_cast<uint4*>(whi + off) = make_uint4(hi[q * 4], hi[q * 4 + 1], hi[q * 4 + 2], hi[q * 4 + 3]);
    *reinterpret_cast<uint4*>(wlo + off) = make_uint4(lo[q * 4], lo[q * 4 + 1], lo[q * 4 + 2], lo[q * 4 + 3]);
  }
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

template <int T>
__global__ void __launch_bounds__(kGThreads, 1) k_qgemm_b(const GemvArgs a, int M) {
  constexpr int S = T == WL_Q4_0 ? 18 : T == WL_Q4_1 ? 20 : 34;
  extern __shared__ uint8_t gsm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kGStages * kGStage);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kGStages);
  __shared__ int s_fail, s_issued;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool sw = a.epi.kind == EPI_SWIGLU;
  // column tile -> segment and first column (SwiGLU tiles: 64 gate + 64 up columns)
  const int nt = blockIdx.x, m0 = blockIdx.y * kGM;
  int seg = 0, n0;
  if (sw) {
    n0 = nt * 64;
  } else {
    n0 = nt * kGN;  // walk the segments in order
    while (seg + 1 < a.nseg && n0 >= a.seg[seg].N) {
      n0 -= a.seg[seg].N;
      seg++;
    }
  }

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < kGStages; s++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_addr(bars + s)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    s_fail = 0;
    s_issued = 0;
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  pdl_trigger();

  const int nk = a.K / kGK;
  const __half* x = reinterpret_cast<const __half*>(a.x);
  // dequant task of this thread: half `part` of quant block b of the tile, k row kk
  const int kk = tid >> 3, b = (tid >> 1) & 3, part = tid & 1;
  const GemvSeg& ws = a.seg[sw ? (b >> 1) : seg];
  const int col0 = sw ? n0 + (b & 1) * 32 : n0 + b * 32;  // first column of the block in its segment
  const bool wlive = col0 < ws.N;
  const uint8_t* wsrc = ws.W + (size_t)(col0 / 32) * S;

  // activations of stage `it` into ring slot it % kGStages (K-major, 128B swizzle):
  // this thread copies chunk c of rows rr0 + 32q (q < 4) of both planes; the
  // swizzled destination and the source row offsets do not change per stage
  const int xc = tid & 7, xr0 = tid >> 3;  // rows xr0, xr0 + 64
  uint32_t xdst[4];
  const __half* xsrc[4];
  bool xok[4];
#pragma unroll
  for (int q = 0; q < 4; q++) {
    const int pl = q >> 1, rr = xr0 + (q & 1) * 64;
    xok[q] = m0 + rr < M;
    xdst[q] = (uint32_t)((2 + pl) * kGTile + (rr << 7) + ((xc ^ (rr & 7)) << 4));
    xsrc[q] = x + (size_t)pl * a.x_plane + (size_t)(xok[q] ? m0 + rr : 0) * a.ldx + xc * 8;
  }
  const uint32_t smb = smem_addr(sm);
  auto load_x = [&](int it) {
    const uint32_t st = smb + (uint32_t)((it % kGStages) * kGStage);
    const int k0 = it * kGK;
#pragma unroll
    for (int q = 0; q < 4; q++) cp16(st + xdst[q], xsrc[q] + k0, xok[q]);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };
  // waits until the MMAs that last read ring slot (it % kGStages) are done (uniform result)
  auto slot_free = [&](int it) -> bool {
    if (it < kGStages) return true;
    const bool w = gbar_wait(smem_addr(bars + it % kGStages), (uint32_t)((it / kGStages - 1) & 1));
    const bool bad = __syncthreads_or(!w);
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    return !bad;
  };

  // raw weight words run two stages ahead of the dequantization
  RawBlock<T> r0, r1, r2;
  load_x(0);
  raw_load<T>(r0, wsrc + (size_t)kk * ws.pitch, part, wlive);
  if (nk > 1) raw_load<T>(r1, wsrc + (size_t)(kGK + kk) * ws.pitch, part, wlive);
  for (int it = 0; it < nk; it++) {
    const int s = it % kGStages;
    uint8_t* st = sm + s * kGStage;
    const bool more = it + 1 < nk;
    if (more) {
      if (!slot_free(it + 1)) {  // uniform: every thread leaves together
        if (tid == 0) s_fail = 1;
        break;
      }
      load_x(it + 1);
    }
    if (it + 2 < nk) raw_load<T>(r2, wsrc + (size_t)((it + 2) * kGK + kk) * ws.pitch, part, wlive);
    dequant_half<T>(r0, st, st + kGTile, kk, b, part, wlive);
    if (more)
      asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    else
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      const uint32_t wa = smem_addr(st), xa = smem_addr(st + 2 * kGTile);
#pragma unroll
      for (int ks = 0; ks < kGK / 16; ks++) {
        // A (weights, N-major): a k step spans 2 k-groups of 2 KB; LBO = 1 KB (64-column
        // block), SBO = 2 KB (8-row k group)
        const uint64_t ah = desc_sw128(wa + ks * 4096, 1024, 2048);
        const uint64_t al = desc_sw128(wa + kGTile + ks * 4096, 1024, 2048);
        // B (activations, K-major): 32 bytes per k step inside the swizzle row; SBO = 1 KB
        const uint64_t bh = desc_sw128(xa + ks * 32, 16, 1024);
        const uint64_t bl = desc_sw128(xa + kGTile + ks * 32, 16, 1024);
        umma_f16(tmem, ah, bh, (it > 0 || ks > 0) ? 1u : 0u);
        umma_f16(tmem, al, bh, 1u);
        umma_f16(tmem, ah, bl, 1u);
      }
      umma_commit(smem_addr(bars + s));
      s_issued = it + 1;
    }
    r0 = r1;
    r1 = r2;
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  // wait for the last issued commit (it covers every MMA issued before it); after
  // a failed wait this still drains the issued MMAs before TMEM is freed
  __syncthreads();
  const int n_issued = s_issued;
  bool ok = !s_fail;
  {
    const int lastc = n_issued - 1;
    const bool w = lastc < 0 ||
                   gbar_wait(smem_addr(bars + (lastc % kGStages)), (uint32_t)((lastc / kGStages) & 1));
    ok = __syncthreads_and(ok && w && n_issued == nk);
  }
  if (!ok && a.err && tid == 0) atomicOr(a.err, 16);
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");

  if (ok && warp < 4) {
    // warp w reads TMEM lanes 32w..32w+31 = tile columns; TMEM columns = token rows
    const int c = warp * 32 + lane;
    float* upbuf = reinterpret_cast<float*>(sm);  // SwiGLU: up values [row][64]
    for (int r0 = 0; r0 < kGM; r0 += 16) {
      uint32_t v[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)r0, v);
      if (sw) {
        if (warp >= 2) {
#pragma unroll
          for (int i = 0; i < 16; i++) upbuf[(r0 + i) * 64 + (c - 64)] = __uint_as_float(v[i]);
        }
      } else {
        const int col = n0 + c;
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int row = m0 + r0 + i;
          if (row < M && col < a.seg[seg].N) store_out(a, seg, row, col, __uint_as_float(v[i]));
        }
      }
    }
  }
  __syncthreads();
  if (ok && sw && warp < 2) {
    const Epilogue& e = a.epi;
    __half* out = reinterpret_cast<__half*>(e.y[0]);
    const int c = warp * 32 + lane;
    const int col = n0 + c;
    const float* upbuf = reinterpret_cast<const float*>(sm);
    for (int r0 = 0; r0 < kGM; r0 += 16) {
      uint32_t v[16];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)r0, v);
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const int row = m0 + r0 + i;
        if (row >= M || col >= a.seg[0].N) continue;
        const float val = silu(__uint_as_float(v[i])) * upbuf[(r0 + i) * 64 + c];
        const size_t o = (size_t)row * e.ldy[0] + col;
        const __half hi = __float2half_rn(val);
        out[o] = hi;
        out[o + e.y_plane] = __float2half_rn(val - __half2float(hi));
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols)
                 : "memory");
}

template <int T>
int launch_t(const GemvArgs& a, int M, int ntiles, cudaStream_t st) {
  if (first_use_on_device((const void*)k_qgemm_b<T>))
    WL_CUDA_TRY(cudaFuncSetAttribute(k_qgemm_b<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGSmem));
  return launch_k(k_qgemm_b<T>, dim3(ntiles, (M + kGM - 1) / kGM), dim3(kGThreads), (size_t)kGSmem,
                  st, a, M);
}

}  // namespace

bool qgemm_b_ok(const GemvArgs& a, int M) {
  if (M < 1 || a.K <= 0 || a.K % kGK) return false;
  if (!(a.type == WL_Q4_0 || a.type == WL_Q4_1 || a.type == WL_Q8_0)) return false;
  if (a.xkind != X_PLANES || a.ldx % 8 || a.x_plane % 8 || (reinterpret_cast<uintptr_t>(a.x) & 15))
    return false;
  if (a.epi.kind == EPI_QKV && a.epi.rope) return false;
  if (a.epi.kind == EPI_SWIGLU) return a.nseg == 2 && a.seg[0].N == a.seg[1].N && a.seg[0].N % 64 == 0;
  for (int s = 0; s < a.nseg; s++)
    if (a.seg[s].N % kGN) return false;
  return true;
}

int launch_qgemm_b(const GemvArgs& a, int M, cudaStream_t st) {
  if (!qgemm_b_ok(a, M)) return fail(WL_ERR_INVALID_ARGUMENT, "qgemm: unsupported shape, layout or epilogue");
  int ntiles = 0;
  if (a.epi.kind == EPI_SWIGLU) {
    ntiles = a.seg[0].N / 64;
  } else {
    for (int s = 0; s < a.nseg; s++) ntiles += a.seg[s].N / kGN;
  }
  switch (a.type) {
    case WL_Q4_0: return launch_t<WL_Q4_0>(a, M, ntiles, st);
    case WL_Q4_1: return launch_t<WL_Q4_1>(a, M, ntiles, st);
    case WL_Q8_0: return launch_t<WL_Q8_0>(a, M, ntiles, st);
  }
  return fail(WL_ERR_UNSUPPORTED, "qgemm: unsupported type");
}

}  // namespace wl
