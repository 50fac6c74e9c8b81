// Prefill GEMM on the 5th-generation tensor cores (tcgen05 MMA, TMEM
// accumulators) for layout-B quantized weights.
//
// Y[m][n] = sum_k X[m][k] * W[k][n] for M token rows at once (woolly's
// layout-B matmul, tensor_utils.rs:118-157, applied to a whole prompt).  One
// CTA computes 128 weight columns x 128 token rows.  The weights are read from
// the tiled decode copy (qtile_bytes): a 64-row stage of a 128-column tile is
// four or six contiguous byte ranges (codes, scales, mins of two 64-column
// quarters).  Warp-specialised, no CTA-wide barrier inside the K loop:
//   * a control warp keeps bulk copies (cp.async.bulk, the TMA engine) of
//     those ranges three stages ahead, completing on per-slot mbarriers; it
//     waits until the dequantizing warps have filled a stage slot, issues 3
//     MMAs per 16-k step into the TMEM accumulator, Xhi*Whi + Xhi*Wlo +
//     Xlo*Whi (the dropped Xlo*Wlo term is ~2^-22 of the product), and
//     commits them to the slot's mbarrier;
//   * 16 dequantizing warps (512 threads) each turn one (quarter, unit, lane)
//     record of 16 weights into f16 hi/lo pairs with W = Whi + Wlo exactly
//     (Q4_0 / Q8_0: Whi = f16(q*d) by HMUL2, Wlo = fma(q, d, -Whi) by HFMA2,
//     the residual being exact in f16; Q4_1 and the K-quants in f32), stored
//     K-major with the 128-byte swizzle (4-byte k-pair stores, bank-conflict
//     free), copy their share of the activation hi/lo planes K-major with the
//     same swizzle, and hand the slot over on a 16-arrival mbarrier; they wait
//     on the slot's MMA commit only before reusing it.
// The epilogue reads the accumulator with tcgen05.ld (all 16 dequantizing
// warps: lane quarter w % 4 = 32 weight columns, token rows 32 * (w / 4)..)
// and applies the same F32 / ADD / QKV / SwiGLU outputs as the decode GEMV.  Every mbarrier wait is bounded; on expiry the
// kernel raises an error bit, waits (bounded) for its issued MMAs and bulk
// copies and frees its TMEM before returning.
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
constexpr int kGDeq = 512;                // dequantizing threads: 16 warps, two per quant block of each k row
constexpr int kGThreads = kGDeq + 32;     // + one control warp (bulk copies, MMA issue)
constexpr int kGCtl = kGDeq / 32;         // the control warp
constexpr int kGTile = 128 * kGK * 2;  // bytes of one f16 operand tile (16 KB)
constexpr int kGStage = 4 * kGTile;    // W hi, W lo, X hi, X lo
constexpr int kGRaw = 10240;  // per-stage raw weight bytes (largest: Q8_0 9216)
constexpr int kGSmem = kGStages * (kGStage + kGRaw) + 1024 + 128;  // + alignment slack + barriers
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

// instruction descriptor, kind::f16: D f32, A and B f16, both K-major,
// N = kGM (bits 17-22, /8), M = kGN (bits 24-28, /16)
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kGM >> 3) << 17) | ((uint32_t)(kGN >> 4) << 24);

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

// Bytes of one 64-column quarter of a tiled-copy stage block (see
// qtile_bytes): the codes of its 8 (k step, block) units in the lanes'
// fragment order, then its f16 scales (4 per lane quad and unit), then Q4_1's
// mins in the same order.
// K-quants (the tiled copy of k_repack_tiled_k): Q4_K scales are (hi, lo)
// f16 pairs of d*sc (16 bytes per lane quad and unit) followed by dmin as
// Q4_1's mins; Q6_K codes are (q - 32) bytes as Q8_0's, with one (hi, lo)
// scale pair per 16 columns (32 bytes per lane quad and unit).
template <int T>
struct Quarter {
  static constexpr bool B8 = T == WL_Q8_0 || T == WL_Q6_K;
  static constexpr int CB = B8 ? 16 : 8;     // code bytes per lane per unit
  static constexpr int CODES = 8 * 32 * CB;  // 2048 (8-bit codes: 4096)
  static constexpr int SCALES = 8 * 4 * (T == WL_Q6_K ? 32 : T == WL_Q4_K ? 16 : 8);
  static constexpr int MINS = (T == WL_Q4_1 || T == WL_Q4_K) ? 256 : 0;
  static constexpr int UNIT = T == WL_Q4_0 ? 18 : T == WL_Q4_1 ? 20 : T == WL_Q8_0 ? 34 : T == WL_Q4_K ? 22 : 40;
};
// one stage's raw bytes for a 128-column tile: [codes q0][codes q1][scales q0][scales q1][mins q0][mins q1]
template <int T>
__host__ __device__ constexpr int raw_stage_bytes() {
  return 2 * (Quarter<T>::CODES + Quarter<T>::SCALES + Quarter<T>::MINS);
}

// Thread tid dequantizes the 16 weights of one (quarter, unit, lane) of the
// stage's raw bytes: output columns g, g+8, 16+g, 24+g of block `blk` and k
// rows 2t, 2t+1, 2t+8, 2t+9 of k step ks, as f16 hi/lo pairs (hi + lo = w
// exactly) into the K-major 128-byte-swizzled A tiles (one 128-byte row per
// tile column, k contiguous): every store is one k pair (4 bytes), and the 32
// lanes of a warp hit 32 different banks.
template <int T>
__device__ __forceinline__ void dequant_frag(const uint8_t* raw, uint8_t* whi, uint8_t* wlo, int tid) {
  using Qt = Quarter<T>;
  const int qd = tid >> 8, rem = tid & 255, ul = rem >> 5, lane = rem & 31;
  const int g = lane >> 2, t = lane & 3, ks = ul >> 1, blk = ul & 1;
  const uint8_t* codes = raw + qd * Qt::CODES + ul * 32 * Qt::CB + lane * Qt::CB;
  // (d(2t), d(2t+1)), (d(2t+8), d(2t+9)); K-quants also the lo halves, Q6_K per m-tile
  uint32_t dpair[2][2], epair[2][2] = {{0u, 0u}, {0u, 0u}};
  if constexpr (T == WL_Q6_K) {
#pragma unroll
    for (int mt = 0; mt < 2; mt++) {
      const uint4 sw = *reinterpret_cast<const uint4*>(raw + 2 * Qt::CODES + qd * Qt::SCALES +
                                                       ((ul * 2 + mt) * 4 + t) * 16);
      dpair[mt][0] = sw.x, dpair[mt][1] = sw.y, epair[mt][0] = sw.z, epair[mt][1] = sw.w;
    }
  } else if constexpr (T == WL_Q4_K) {
    const uint4 sw = *reinterpret_cast<const uint4*>(raw + 2 * Qt::CODES + qd * Qt::SCALES + (ul * 4 + t) * 16);
    dpair[0][0] = dpair[1][0] = sw.x, dpair[0][1] = dpair[1][1] = sw.y;
    epair[0][0] = epair[1][0] = sw.z, epair[0][1] = epair[1][1] = sw.w;
  } else {
    const uint2 sw = *reinterpret_cast<const uint2*>(raw + 2 * Qt::CODES + qd * Qt::SCALES + (ul * 4 + t) * 8);
    dpair[0][0] = dpair[1][0] = sw.x, dpair[0][1] = dpair[1][1] = sw.y;
  }
  uint32_t mpair[2] = {0u, 0u};
  if constexpr (Qt::MINS) {
    const uint2 mw = *reinterpret_cast<const uint2*>(raw + 2 * (Qt::CODES + Qt::SCALES) + qd * Qt::MINS +
                                                     (ul * 4 + t) * 8);
    mpair[0] = mw.x, mpair[1] = mw.y;
  }
  // q pairs: qp[h][j] = codes of column os[j] at k rows (2t + 8h, +1)
  const int os[4] = {g, 16 + g, g + 8, 24 + g};
  uint32_t qp[2][4];
  if constexpr (Qt::B8) {
    const uint4 c = *reinterpret_cast<const uint4*>(codes);
    const uint32_t w[4] = {c.x, c.y, c.z, c.w};
    // byte (mt*4 + r)*2 + e: column mt*16 + g + 8(r&1), k rows 2t + 8(r>>1) + e
#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
      for (int r = 0; r < 4; r++) {
        const int idx = mt * 4 + r;  // 16-bit word index
        const uint32_t wd = w[idx >> 1] >> (16 * (idx & 1));
        const uint32_t v = ((wd & 0xFFu) | ((wd & 0xFF00u) << 8)) ^ 0x00800080u;
        const uint32_t q = h2u(__hsub2(u2h(v | 0x64006400u), u2h(0x64806480u)));  // exact int8
        const int j = mt == 0 ? ((r & 1) ? 2 : 0) : ((r & 1) ? 3 : 1);   // os index of the column
        qp[r >> 1][j] = q;
      }
  } else {
    const uint2 c = *reinterpret_cast<const uint2*>(codes);
    const uint32_t w[2] = {c.x, c.y};
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const uint32_t n = ((w[h] >> (4 * j)) & 0x000F000Fu) | 0x64006400u;  // 1024 + q per lane
        qp[h][j] = h2u(__hsub2(u2h(n), u2h(T == WL_Q4_0 ? 0x64086408u : 0x64006400u)));
      }
  }
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int c8 = 2 * ks + h;  // 16-byte chunk of k rows ks*16 + 8h .. +7
#pragma unroll
    for (int j = 0; j < 4; j++) {
      uint32_t hi, lo;
      const int mt = j & 1;  // os[j] = g, 16+g, g+8, 24+g: m-tile 0, 1, 0, 1
      if constexpr (T == WL_Q4_1 || T == WL_Q4_K || T == WL_Q6_K) {
        // in f32, rounded once to hi: Q4_1 q*d + m (dequantize_q4_1, dequantize.rs:372);
        // Q4_K q*(d*sc) + dmin (:404-462); Q6_K (q-32)*(d*sc)/64 (:465-537)
        const float2 qf = __half22float2(u2h(qp[h][j]));
        float2 df = __half22float2(u2h(dpair[mt][h]));
        if constexpr (T != WL_Q4_1) {
          const float2 ef = __half22float2(u2h(epair[mt][h]));
          df.x += ef.x, df.y += ef.y;  // exact: the pair splits d*sc
        }
        const float2 mf = __half22float2(u2h(mpair[h]));
        float v0 = qf.x * df.x + mf.x, v1 = qf.y * df.y + mf.y;
        if constexpr (T == WL_Q6_K) v0 *= 0.015625f, v1 *= 0.015625f;
        const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
        hi = h2u(__halves2half2(h0, h1));
        lo = h2u(__halves2half2(__float2half_rn(v0 - __half2float(h0)), __float2half_rn(v1 - __half2float(h1))));
      } else {
        split_pair(qp[h][j], u2h(dpair[0][h]), hi, lo);
      }
      const int row = qd * 64 + blk * 32 + os[j];
      const uint32_t off = (uint32_t)((row << 7) + ((c8 ^ (row & 7)) << 4) + 4 * t);
      *reinterpret_cast<uint32_t*>(whi + off) = hi;
      *reinterpret_cast<uint32_t*>(wlo + off) = lo;
    }
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
  using Qt = Quarter<T>;
  static_assert(raw_stage_bytes<T>() <= kGRaw, "raw stage slot too small");
  constexpr int STB = 512 * Qt::UNIT;  // bytes of one (256-column group, 64-row stage) block of the tiled copy
  extern __shared__ uint8_t gsm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* rawb = sm + kGStages * kGStage;  // [kGStages][kGRaw] bulk-copied weight bytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(rawb + kGStages * kGRaw);  // MMA done, per slot
  uint64_t* wbars = bars + kGStages;                                       // raw bytes landed, per slot
  uint64_t* fbars = wbars + kGStages;  // slot dequantized and its activations landed (16 warp arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fbars + kGStages);
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
  // the two 64-column quarters of this tile in the tiled copies: (source, group, quarter)
  const int nk = a.K / kGK;
  const uint8_t* qsrc[2];
  for (int q = 0; q < 2; q++) {
    const GemvSeg& gs = a.seg[sw ? q : seg];
    const int c = sw ? n0 : n0 + 64 * q;  // first column of the quarter in its segment
    qsrc[q] = gs.W + (size_t)(c / 256) * nk * STB;  // the quarter within the group: qw0 / qw1
  }
  const int qw0 = (n0 % 256) / 64, qw1 = sw ? qw0 : qw0 + 1;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < 2 * kGStages; s++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(smem_addr(bars + s)) : "memory");
    for (int s = 0; s < kGStages; s++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(fbars + s)), "r"(kGDeq / 32)
                   : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    s_fail = 0;
    s_issued = 0;
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  // stage `it`'s weight bytes of both quarters into raw slot it % kGStages with
  // bulk copies (TMA engine), completing on wbars[slot] (thread 0 only)
  auto issue_w = [&](int it) {
    const int slot = it % kGStages;
    const uint32_t dst = smem_addr(rawb + slot * kGRaw), bar = smem_addr(wbars + slot);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar),
                 "r"((uint32_t)raw_stage_bytes<T>())
                 : "memory");
    for (int q = 0; q < 2; q++) {
      const int qw = q ? qw1 : qw0;
      const uint8_t* blk = qsrc[q] + (size_t)it * STB;
      const uint8_t* parts[3] = {blk + qw * Qt::CODES, blk + 32 * 32 * Qt::CB + qw * Qt::SCALES,
                                 blk + 32 * 32 * Qt::CB + 4 * Qt::SCALES + qw * 256};
      const uint32_t dsts[3] = {dst + q * Qt::CODES, dst + 2 * Qt::CODES + q * Qt::SCALES,
                                dst + 2 * (Qt::CODES + Qt::SCALES) + q * Qt::MINS};
      const uint32_t sizes[3] = {(uint32_t)Qt::CODES, (uint32_t)Qt::SCALES, (uint32_t)Qt::MINS};
      for (int k = 0; k < 3; k++)
        if (sizes[k])
          asm volatile(
              "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                  dsts[k]),
              "l"(parts[k]), "r"(sizes[k]), "r"(bar)
              : "memory");
    }
  };
  // Warp-specialised pipeline.  The control warp (lane 0) keeps the bulk
  // weight copies three stages ahead, waits until the 16 dequantizing warps
  // have filled a ring slot (fbars), issues its MMAs and commits them to the
  // slot's `bars` barrier; the dequantizing warps wait on that barrier only
  // before reusing the slot.  No CTA-wide barrier inside the K loop.
  const bool ctl = warp == kGCtl;
  if (ctl && lane == 0)  // the weights do not depend on earlier kernels: start them before the PDL wait
    for (int it = 0; it < kGStages && it < nk; it++) issue_w(it);
  pdl_wait();
  pdl_trigger();

  if (ctl) {
    if (lane == 0) {
      int issued = 0;
      for (int it = 0; it < nk; it++) {
        const int s = it % kGStages;
        if (!gbar_wait(smem_addr(fbars + s), (uint32_t)((it / kGStages) & 1))) {
          s_fail = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        const uint32_t wa = smem_addr(sm + s * kGStage), xa = wa + 2 * kGTile;
#pragma unroll
        for (int ks = 0; ks < kGK / 16; ks++) {
          // A (weights) and B (activations) both K-major: 32 bytes per k step
          // inside the 128-byte swizzle row; SBO = 1 KB (8 rows)
          const uint64_t ah = desc_sw128(wa + ks * 32, 16, 1024);
          const uint64_t al = desc_sw128(wa + kGTile + ks * 32, 16, 1024);
          const uint64_t bh = desc_sw128(xa + ks * 32, 16, 1024);
          const uint64_t bl = desc_sw128(xa + kGTile + ks * 32, 16, 1024);
          umma_f16(tmem, ah, bh, (it > 0 || ks > 0) ? 1u : 0u);
          umma_f16(tmem, al, bh, 1u);
          umma_f16(tmem, ah, bl, 1u);
        }
        umma_commit(smem_addr(bars + s));
        issued = it + 1;
        // fbars[s] also says the raw slot s (stage it) has been read: refill it
        if (it + kGStages < nk) {
          asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
          issue_w(it + kGStages);
        }
      }
      s_issued = issued;
    }
    __syncwarp();
  } else {
    const __half* x = reinterpret_cast<const __half*>(a.x);
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
    load_x(0);
    for (int it = 0; it < nk; it++) {
      const int s = it % kGStages;
      uint8_t* st = sm + s * kGStage;
      const bool more = it + 1 < nk;
      if (more) {
        // slot (it + 1) % kGStages last fed the MMAs of stage it + 1 - kGStages
        const int nx = it + 1;
        if (nx >= kGStages &&
            !gbar_wait(smem_addr(bars + nx % kGStages), (uint32_t)((nx / kGStages - 1) & 1))) {
          s_fail = 1;
          break;
        }
        load_x(nx);
      }
      if (!gbar_wait(smem_addr(wbars + s), (uint32_t)((it / kGStages) & 1))) {
        s_fail = 1;
        break;
      }
      dequant_frag<T>(rawb + s * kGRaw, st, st + kGTile, tid);
      if (more)
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");
      else
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(fbars + s)) : "memory");
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  }
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
  // bulk copies still in flight (after a failure) must land before the CTA exits
  if (tid == 0)
    for (int it = n_issued; it < nk && it < n_issued + kGStages; it++)
      gbar_wait(smem_addr(wbars + it % kGStages), (uint32_t)((it / kGStages) & 1));
  if (!ok && a.err && tid == 0) atomicOr(a.err, 16);
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");

  // all 16 dequantizing warps drain the accumulator: warp w reads TMEM lanes
  // 32*(w%4).. (tile columns; a warp may only address its lane quarter) for
  // token rows [32*(w/4), +32) (TMEM columns)
  const int lw = warp & 3, rq = warp >> 2;
  if (ok && warp < kGDeq / 32) {
    const int c = lw * 32 + lane;
    float* upbuf = reinterpret_cast<float*>(sm);  // SwiGLU: up values [row][64]
    for (int r0 = rq * 32; r0 < rq * 32 + 32; r0 += 16) {
      uint32_t v[16];
      tmem_ld16(tmem + ((uint32_t)(lw * 32) << 16) + (uint32_t)r0, v);
      if (sw) {
        if (lw >= 2) {
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
  if (ok && sw && warp < kGDeq / 32 && lw < 2) {
    const Epilogue& e = a.epi;
    __half* out = reinterpret_cast<__half*>(e.y[0]);
    const int c = lw * 32 + lane;
    const int col = n0 + c;
    const float* upbuf = reinterpret_cast<const float*>(sm);
    for (int r0 = rq * 32; r0 < rq * 32 + 32; r0 += 16) {
      uint32_t v[16];
      tmem_ld16(tmem + ((uint32_t)(lw * 32) << 16) + (uint32_t)r0, v);
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
  if (M < 1 || a.K <= 0 || a.K % kGK || !a.tiled) return false;
  if (!(a.type == WL_Q4_0 || a.type == WL_Q4_1 || a.type == WL_Q8_0 || a.type == WL_Q4_K || a.type == WL_Q6_K))
    return false;
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
    case WL_Q4_K: return launch_t<WL_Q4_K>(a, M, ntiles, st);
    case WL_Q6_K: return launch_t<WL_Q6_K>(a, M, ntiles, st);
  }
  return fail(WL_ERR_UNSUPPORTED, "qgemm: unsupported type");
}

}  // namespace wl
