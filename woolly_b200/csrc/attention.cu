// GQA attention for decode and prefill rows (sm_100a).
//
// Reference: LazyTransformer::compute_optimized_gqa_attention
// (woolly-core/src/model/lazy_transformer.rs:360-434): for query head h the
// KV head is h / (H / KVH); scores q.k * hd^-1/2 over keys 0..=pos (causal,
// the KV cache holds past ++ new); max-subtracted softmax; output sum p_j v_j.
// The optional window W keeps keys j in (pos - W, pos] (Mistral shape; no
// reference counterpart).
//
// Paged path (flash-decoding): one CTA per (KV head, query row, context
// split).  The KV cache is paged as [page][kv_head][16 tokens][head_dim] f16,
// so a (page, head) pair is one contiguous 2-8 KB chunk; the CTA streams the K
// and V chunks of its pages with 1-D bulk copies (cp.async.bulk, completion
// on an mbarrier) through a 4-stage shared-memory ring, scores all G = H/KVH
// query heads of the group from shared memory (GQA reuse), keeps an online
// softmax per head and writes either the final row (one split) or an
// unnormalised partial (o, m, l) that k_attn_combine merges with the
// log-sum-exp rule.  Every mbarrier wait is bounded; on expiry the kernel
// raises an error flag instead of spinning.
//
// Prompt chunks of one session take k_attn_prefill instead (tensor cores,
// see below); decode rows and short chunks the paged kernel.
#include <cuda_fp16.h>

#include <cmath>
#include <cstring>
#include <string>

#include "common.h"
#include "kernels.cuh"
#include "pdl.cuh"

namespace wl {
namespace {

constexpr int kAttnThreads = 128;
constexpr int kPage = 16;    // tokens per KV page
constexpr int kRingA = 3;            // tiles in flight per CTA
constexpr int kTile = 64;    // tokens per softmax tile (f32 path)

// ---------------------------------------------------------------- mbarrier / bulk copy
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  const unsigned a = (unsigned)__cvta_generic_to_shared(bar);
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(a), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  const unsigned a = (unsigned)__cvta_generic_to_shared(bar);
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(a), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  const unsigned b = (unsigned)__cvta_generic_to_shared(bar);
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(d),
      "l"(src), "r"(bytes), "r"(b)
      : "memory");
}
// bounded wait for the given phase parity; false if the bound expired
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  const unsigned a = (unsigned)__cvta_generic_to_shared(bar);
  for (int it = 0; it < (1 << 22); it++) {
    unsigned done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// f32 output, or f16 hi/lo planes (lo plane `plane` elements after hi) when plane != 0
__device__ __forceinline__ void put_out(void* out, size_t plane, size_t i, float v) {
  if (!plane) {
    reinterpret_cast<float*>(out)[i] = v;
  } else {
    const __half hi = __float2half_rn(v);
    reinterpret_cast<__half*>(out)[i] = hi;
    reinterpret_cast<__half*>(out)[i + plane] = __float2half_rn(v - __half2float(hi));
  }
}

// ---------------------------------------------------------------- paged kernel
// TPG pages per softmax round: 2 when the launch has fewer (KV head, row)
// pairs than SMs, 1 (shorter rounds, more resident CTAs, more context splits)
// when it has at least one per SM.
template <int HD, int G, int TPG>
__global__ void __launch_bounds__(kAttnThreads) k_attn_paged(const AttnArgs a, float scale) {
  constexpr int kTilePages = TPG;
  constexpr int CHUNK = kPage * HD;        // halves per (page, head) chunk
  constexpr int LPT = HD / 8;              // lanes per token in the score phase
  constexpr int TPP = kAttnThreads / LPT;  // tokens per pass
  constexpr int NW = kAttnThreads / 32;
  constexpr int DP = HD / 2;
  constexpr int NS = kAttnThreads / DP;  // token streams in the V phase
  constexpr int TT = kTilePages * kPage;     // tokens per round
  extern __shared__ __align__(128) __half kvs[];  // [kRingA][kTilePages][2][CHUNK]
  __shared__ __align__(8) uint64_t bars[kRingA];
  __shared__ float s_p[G][TT];
  __shared__ float s_m[G], s_l[G], s_alpha[G];
  __shared__ float s_red[NS][G][HD];
  __shared__ int s_fail;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kvh = blockIdx.x, r = blockIdx.y, sp = blockIdx.z;
  pdl_wait();
  pdl_trigger();
  const int pos = a.row_pos[r];
  const int sess = a.row_sess[r];
  const int j0 = (a.window > 0 && pos - a.window + 1 > 0) ? pos - a.window + 1 : 0;
  const int P0 = j0 / kPage, P1 = pos / kPage;
  const int npg = P1 - P0 + 1;
  const int pc = (npg + a.nsplit - 1) / a.nsplit;
  const int pa = P0 + sp * pc;
  const int pb = min(P1 + 1, pa + pc);
  const int mine = pb > pa ? pb - pa : 0;
  const int ntile = (mine + kTilePages - 1) / kTilePages;
  const int* table = a.kv.page_table + (size_t)sess * a.kv.max_pages;

  auto issue = [&](int i) {  // tile i (pages pa + 4i ...) into ring slot i % kRingA (thread 0 only)
    const int st = i % kRingA;
    const int q0 = i * kTilePages;
    const int n = min(kTilePages, mine - q0);
    mbar_expect_tx(&bars[st], (unsigned)(n * 2 * CHUNK * 2));
    for (int q = 0; q < n; q++) {
      const int pg = table[pa + q0 + q];
      const size_t off = ((size_t)pg * a.kv.kv_heads + kvh) * CHUNK;
      __half* dst = kvs + ((size_t)st * kTilePages + q) * 2 * CHUNK;
      bulk_g2s(dst, a.kv.k + off, CHUNK * 2, &bars[st]);
      bulk_g2s(dst + CHUNK, a.kv.v + off, CHUNK * 2, &bars[st]);
    }
  };
  if (tid == 0) {
    for (int s = 0; s < kRingA; s++) mbar_init(&bars[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    s_fail = 0;
  }
  __syncthreads();
  if (tid == 0)
    for (int i = 0; i < kRingA && i < ntile; i++) issue(i);

  const int sub = tid / LPT, li = tid % LPT;
  float qr[G][8];
#pragma unroll
  for (int h = 0; h < G; h++) {
    const float* qp = a.q + (size_t)r * a.ldq + (size_t)(kvh * G + h) * HD + li * 8;
#pragma unroll
    for (int i = 0; i < 8; i++) qr[h][i] = qp[i];
  }
  if (tid < G) s_m[tid] = -INFINITY, s_l[tid] = 0.f;
  const int stream = tid / DP, dp = tid % DP;
  float o[G][2];
#pragma unroll
  for (int h = 0; h < G; h++) o[h][0] = o[h][1] = 0.f;
  __syncthreads();

  for (int i = 0; i < ntile; i++) {
    const int st = i % kRingA;
    if (!mbar_wait(&bars[st], (unsigned)((i / kRingA) & 1))) {
      if (a.err) atomicOr(a.err, 2);
      s_fail = 1;
    }
    __syncthreads();
    if (s_fail) break;
    const __half* T = kvs + (size_t)st * kTilePages * 2 * CHUNK;  // page q: K at q*2*CHUNK, V after
    const int tok0 = (pa + i * kTilePages) * kPage;
    const int tvalid = min(TT, (mine - i * kTilePages) * kPage);  // tokens of loaded pages
#pragma unroll 4
    for (int pass = 0; pass < TT / TPP; pass++) {
      const int tk = pass * TPP + sub;
      const int j = tok0 + tk;
      const bool ok = tk < tvalid && j >= j0 && j <= pos;
      float kf[8];
      if (tk < tvalid) {
        const uint4 u = *reinterpret_cast<const uint4*>(T + (size_t)(tk / kPage) * 2 * CHUNK +
                                                        (tk % kPage) * HD + li * 8);
        const __half2* hh = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float2 f = __half22float2(hh[q]);
          kf[2 * q] = f.x, kf[2 * q + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int q = 0; q < 8; q++) kf[q] = 0.f;
      }
#pragma unroll
      for (int h = 0; h < G; h++) {
        float s = 0.f;
#pragma unroll
        for (int q = 0; q < 8; q++) s += qr[h][q] * kf[q];
#pragma unroll
        for (int off = LPT / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (li == 0) s_p[h][tk] = ok ? s * scale : -INFINITY;
      }
    }
    __syncthreads();
    for (int h = warp; h < G; h += NW) {
      constexpr int SV = (TT + 31) / 32;
      float sv[SV];
      float mx = -INFINITY;
#pragma unroll
      for (int q = 0; q < SV; q++) {
        sv[q] = lane + 32 * q < TT ? s_p[h][lane + 32 * q] : -INFINITY;
        mx = fmaxf(mx, sv[q]);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = s_m[h];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.f;
#pragma unroll
      for (int q = 0; q < SV; q++) {
        const float p = sv[q] == -INFINITY ? 0.f : expf(sv[q] - m_new);
        if (lane + 32 * q < TT) s_p[h][lane + 32 * q] = p;
        sum += p;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      if (lane == 0) {
        const float alpha = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
        s_alpha[h] = alpha;
        s_l[h] = s_l[h] * alpha + sum;
        s_m[h] = m_new;
      }
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < G; h++) {
      const float al = s_alpha[h];
      o[h][0] *= al, o[h][1] *= al;
    }
    // V rows of loaded pages only (tokens past tvalid were never copied)
#pragma unroll 4
    for (int tk = stream; tk < tvalid; tk += NS) {
      const float2 vv = __half22float2(*reinterpret_cast<const __half2*>(
          T + (size_t)(tk / kPage) * 2 * CHUNK + CHUNK + (tk % kPage) * HD + 2 * dp));
#pragma unroll
      for (int h = 0; h < G; h++) {
        const float p = s_p[h][tk];
        o[h][0] += p * vv.x;
        o[h][1] += p * vv.y;
      }
    }
    __syncthreads();  // ring slot st fully consumed
    if (tid == 0 && i + kRingA < ntile) issue(i + kRingA);
  }
#pragma unroll
  for (int h = 0; h < G; h++) {
    s_red[stream][h][2 * dp] = o[h][0];
    s_red[stream][h][2 * dp + 1] = o[h][1];
  }
  __syncthreads();
  for (int i = tid; i < G * HD; i += kAttnThreads) {
    const int h = i / HD, d = i % HD;
    float acc = 0.f;
#pragma unroll
    for (int s = 0; s < NS; s++) acc += s_red[s][h][d];
    const int qh = kvh * G + h;
    if (a.nsplit == 1) {
      const float l = s_l[h];
      put_out(a.out, a.out_plane, (size_t)r * a.ldo + (size_t)qh * HD + d,
              l > 0.f ? acc * (1.0f / l) : 0.f);
    } else {
      const size_t pi = ((size_t)r * a.heads + qh) * a.nsplit + sp;
      a.part_o[pi * HD + d] = acc;
      if (d == 0) {
        a.part_ml[pi * 2] = s_m[h];
        a.part_ml[pi * 2 + 1] = s_l[h];
      }
    }
  }
}

template <int HD>
__global__ void k_attn_combine(const float* part_o, const float* part_ml, int heads, int nsplit,
                               void* out, int ldo, size_t out_plane) {
  const int r = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  pdl_wait();
  pdl_trigger();
  const size_t base = ((size_t)r * heads + h) * nsplit;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; s++) M = fmaxf(M, part_ml[(base + s) * 2]);
  float L = 0.f, acc = 0.f;
  for (int s = 0; s < nsplit; s++) {
    const float m = part_ml[(base + s) * 2];
    if (m == -INFINITY) continue;
    const float w = expf(m - M);
    L += part_ml[(base + s) * 2 + 1] * w;
    acc += part_o[(base + s) * HD + d] * w;
  }
  put_out(out, out_plane, (size_t)r * ldo + (size_t)h * HD + d, L > 0.f ? acc * (1.0f / L) : 0.f);
}

template <int HD, int G, int TPG>
int launch_paged_t(const AttnArgs& a, float scale, cudaStream_t st) {
  const size_t smem = (size_t)kRingA * TPG * 2 * kPage * HD * sizeof(__half);
  if (first_use_on_device((const void*)k_attn_paged<HD, G, TPG>))
    WL_CUDA_TRY(cudaFuncSetAttribute(k_attn_paged<HD, G, TPG>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  return launch_k(k_attn_paged<HD, G, TPG>, dim3(a.kv_heads, a.rows, a.nsplit), dim3(kAttnThreads),
                  smem, st, a, scale);
}

int device_sms() {
  static int cache[32] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int& n = cache[dev & 31];
  if (!n && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 148;
  return n;
}

template <int HD, int G>
int launch_paged_g(const AttnArgs& a, float scale, cudaStream_t st) {
  return a.rows * a.kv_heads >= device_sms() ? launch_paged_t<HD, G, 1>(a, scale, st)
                                             : launch_paged_t<HD, G, 2>(a, scale, st);
}

template <int HD>
int launch_paged_hd(const AttnArgs& a, int G, float scale, cudaStream_t st) {
  int s;
  switch (G) {
    case 1: s = launch_paged_g<HD, 1>(a, scale, st); break;
    case 2: s = launch_paged_g<HD, 2>(a, scale, st); break;
    case 4: s = launch_paged_g<HD, 4>(a, scale, st); break;
    case 8: s = launch_paged_g<HD, 8>(a, scale, st); break;
    default:
      return fail(WL_ERR_UNSUPPORTED,
                  "attention: heads per KV head must be 1, 2, 4 or 8 (got " + std::to_string(G) + ")");
  }
  if (s) return s;
  if (a.nsplit > 1) {
    WL_TRY(launch_k(k_attn_combine<HD>, dim3(a.rows, a.heads), dim3(HD), 0, st,
                    (const float*)a.part_o, (const float*)a.part_ml, a.heads, a.nsplit, a.out, a.ldo,
                    a.out_plane));
  }
  return WL_OK;
}

// ---------------------------------------------------------------- prefill on tensor cores
// Prompt rows of one session (consecutive positions; the model's prefill
// chunks) on mma.sync m16n8k16, flash-attention style.  One CTA per (64
// MMA rows, KV head): an MMA row is a (query row, head of the group) pair,
// 16 per warp (16 / G query rows x G heads), so the CTA shares every K / V
// block among its four warps and the G heads.  Keys stream in blocks of 64
// (four pages) through a two-stage cp.async ring, stored with the 16-byte
// chunks of each key row XOR-swizzled so that the ldmatrix reads of K (and the
// transposed reads of V) are bank-conflict free; chunks of pages past the
// last query position are zero-filled.  Exactness as elsewhere: q = qhi + qlo
// and p = phi + plo as f16 pairs (~22 bits) against the f16 K / V cache, two
// MMAs per product, f32 accumulation; the online softmax (max subtraction,
// expf, rescale) runs in f32 on the accumulator fragments.  Scores are
// (q.k) * hd^-1/2 with the causal bound and the optional window, as the
// paged kernel applies them.
constexpr int kPfThreads = 128;
constexpr int kPfKeys = 64;

__device__ __forceinline__ void pf_cp16(uint32_t dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void pf_mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void pf_ldsm4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                         uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void pf_ldsm4t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// (x0, x1) -> f16 pairs hi = f16(x), lo = f16(x - hi)
__device__ __forceinline__ void pf_split(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  const __half2 h = __halves2half2(h0, h1);
  const __half2 l = __halves2half2(__float2half_rn(x0 - __half2float(h0)), __float2half_rn(x1 - __half2float(h1)));
  memcpy(&hi, &h, 4);
  memcpy(&lo, &l, 4);
}

template <int HD, int G>
__global__ void __launch_bounds__(kPfThreads) k_attn_prefill(const AttnArgs a, float scale) {
  constexpr int QR = 16 / G;  // query rows per warp
  constexpr int CR = 4 * QR;  // query rows per CTA
  constexpr int KS = HD / 16;
  constexpr int NT = HD / 8;
  constexpr int CH = HD / 8;  // 16-byte chunks per key row
  constexpr int BLK = kPfKeys * HD;  // halves of one K (or V) block
  extern __shared__ __align__(128) __half pf_s[];  // [2 stages][K, V][64 keys][HD] swizzled
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int kvh = blockIdx.y, row0 = blockIdx.x * CR;
  pdl_wait();
  pdl_trigger();
  if (row0 >= a.rows) return;
  const int nrows = min(CR, a.rows - row0);
  const int sess = a.row_sess[row0];
  const int* table = a.kv.page_table + (size_t)sess * a.kv.max_pages;
  const int pos_first = a.row_pos[row0], pos_last = a.row_pos[row0 + nrows - 1];
  const int jlo = (a.window > 0 && pos_first - a.window + 1 > 0) ? pos_first - a.window + 1 : 0;
  const int blo = jlo / kPfKeys, bhi = pos_last / kPfKeys;
  const int last_page = pos_last / kPage;

  // this lane's two MMA rows (g, g + 8): query row and head
  int qrow[2], qpos[2], qhead[2];
  bool qok[2];
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int i = g + 8 * h;
    qrow[h] = warp * QR + i / G;
    qhead[h] = kvh * G + i % G;
    qok[h] = qrow[h] < nrows;
    qpos[h] = qok[h] ? a.row_pos[row0 + qrow[h]] : -1;
  }
  const int wpos_max = max(qpos[0], qpos[1]);  // per lane; the warp max below
  int warp_max = wpos_max;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) warp_max = max(warp_max, __shfl_xor_sync(0xffffffffu, warp_max, off));

  // Q fragments (A operand, m16 x k16 per k step) as f16 hi / lo pairs
  uint32_t qh[KS][4], ql[KS][4];
#pragma unroll
  for (int ks = 0; ks < KS; ks++)
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int h = r & 1, d = ks * 16 + 2 * t + 8 * (r >> 1);
      float x0 = 0.f, x1 = 0.f;
      if (qok[h]) {
        const float* qp = a.q + (size_t)(row0 + qrow[h]) * a.ldq + (size_t)qhead[h] * HD + d;
        x0 = qp[0], x1 = qp[1];
      }
      pf_split(x0, x1, qh[ks][r], ql[ks][r]);
    }

  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(pf_s);
  auto load_block = [&](int b, int stage) {
    // 2 * 64 * CH chunks: K then V; chunk (key kk, c) lands at kk*CH + (c ^ (kk & 7))
    for (int i = tid; i < 2 * kPfKeys * CH; i += kPfThreads) {
      const int kv = i / (kPfKeys * CH), rem = i - kv * kPfKeys * CH;
      const int kk = rem / CH, c = rem - kk * CH;
      const int pgi = (b * kPfKeys + kk) / kPage;
      const bool ok = pgi <= last_page;
      const int pg = ok ? table[pgi] : 0;
      const __half* src = (kv ? a.kv.v : a.kv.k) +
                          (((size_t)pg * a.kv.kv_heads + kvh) * kPage + (kk % kPage)) * HD + c * 8;
      const uint32_t dst = sbase + (uint32_t)(((stage * 2 + kv) * BLK + (kk * CH + (c ^ (kk & 7))) * 8) * 2);
      pf_cp16(dst, src, ok);
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };

  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

  load_block(blo, 0);
  for (int b = blo; b <= bhi; b++) {
    const int stage = (b - blo) & 1;
    if (b + 1 <= bhi) {
      load_block(b + 1, stage ^ 1);
      asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    }
    __syncthreads();
    const int key0 = b * kPfKeys;
    if (key0 <= warp_max) {  // blocks wholly past this warp's rows are all masked
      const uint32_t ks_base = sbase + (uint32_t)((stage * 2 + 0) * BLK * 2);
      const uint32_t vs_base = sbase + (uint32_t)((stage * 2 + 1) * BLK * 2);
      float sc[8][4];
#pragma unroll
      for (int n = 0; n < 8; n++) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
      const int mi = lane >> 3, lr = lane & 7;
#pragma unroll
      for (int ks = 0; ks < KS; ks++)
#pragma unroll
        for (int jp = 0; jp < 4; jp++) {
          const int kk = jp * 16 + (mi >> 1) * 8 + lr, c = ks * 2 + (mi & 1);
          uint32_t b0, b1, b2, b3;
          pf_ldsm4(ks_base + (uint32_t)((kk * CH + (c ^ (kk & 7))) * 16), b0, b1, b2, b3);
          pf_mma(sc[2 * jp], qh[ks], b0, b1);
          pf_mma(sc[2 * jp], ql[ks], b0, b1);
          pf_mma(sc[2 * jp + 1], qh[ks], b2, b3);
          pf_mma(sc[2 * jp + 1], ql[ks], b2, b3);
        }
      // mask, scale, online softmax (rows g and g + 8)
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int n = 0; n < 8; n++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int h = e >> 1, j = key0 + n * 8 + 2 * t + (e & 1);
          const bool ok = qok[h] && j <= qpos[h] && (a.window <= 0 || j > qpos[h] - a.window);
          sc[n][e] = ok ? sc[n][e] * scale : -INFINITY;
          mx[h] = fmaxf(mx[h], sc[n][e]);
        }
      float alpha[2];
#pragma unroll
      for (int h = 0; h < 2; h++) {
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
        const float mnew = fmaxf(mrow[h], mx[h]);
        alpha[h] = mrow[h] == -INFINITY ? 0.f : expf(mrow[h] - mnew);
        mrow[h] = mnew;
      }
      float sum[2] = {0.f, 0.f};
#pragma unroll
      for (int n = 0; n < 8; n++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int h = e >> 1;
          const float p = sc[n][e] == -INFINITY ? 0.f : expf(sc[n][e] - mrow[h]);
          sc[n][e] = p;
          sum[h] += p;
        }
#pragma unroll
      for (int h = 0; h < 2; h++) {
        sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 1);
        sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 2);
        lrow[h] = lrow[h] * alpha[h] + sum[h];
      }
#pragma unroll
      for (int n = 0; n < NT; n++) {
        o[n][0] *= alpha[0], o[n][1] *= alpha[0];
        o[n][2] *= alpha[1], o[n][3] *= alpha[1];
      }
      // O += P V over the block's four 16-key steps
#pragma unroll
      for (int kc = 0; kc < 4; kc++) {
        uint32_t ph[4], pl[4];
        pf_split(sc[2 * kc][0], sc[2 * kc][1], ph[0], pl[0]);
        pf_split(sc[2 * kc][2], sc[2 * kc][3], ph[1], pl[1]);
        pf_split(sc[2 * kc + 1][0], sc[2 * kc + 1][1], ph[2], pl[2]);
        pf_split(sc[2 * kc + 1][2], sc[2 * kc + 1][3], ph[3], pl[3]);
#pragma unroll
        for (int n = 0; n < NT; n += 2) {
          const int kk = kc * 16 + (mi & 1) * 8 + lr, c = n + (mi >> 1);
          uint32_t b0, b1, b2, b3;
          pf_ldsm4t(vs_base + (uint32_t)((kk * CH + (c ^ (kk & 7))) * 16), b0, b1, b2, b3);
          pf_mma(o[n], ph, b0, b1);
          pf_mma(o[n], pl, b0, b1);
          pf_mma(o[n + 1], ph, b2, b3);
          pf_mma(o[n + 1], pl, b2, b3);
        }
      }
    }
    __syncthreads();  // the stage is rewritten by the load two blocks on
  }
#pragma unroll
  for (int h = 0; h < 2; h++) {
    if (!qok[h]) continue;
    const float inv = lrow[h] > 0.f ? 1.0f / lrow[h] : 0.f;
    const size_t ob = (size_t)(row0 + qrow[h]) * a.ldo + (size_t)qhead[h] * HD;
#pragma unroll
    for (int n = 0; n < NT; n++) {
      put_out(a.out, a.out_plane, ob + n * 8 + 2 * t, o[n][2 * h] * inv);
      put_out(a.out, a.out_plane, ob + n * 8 + 2 * t + 1, o[n][2 * h + 1] * inv);
    }
  }
}

template <int HD, int G>
int launch_prefill_t(const AttnArgs& a, float scale, cudaStream_t st) {
  const size_t smem = (size_t)2 * 2 * kPfKeys * HD * sizeof(__half);
  if (first_use_on_device((const void*)k_attn_prefill<HD, G>))
    WL_CUDA_TRY(cudaFuncSetAttribute(k_attn_prefill<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
  constexpr int CR = 4 * (16 / G);
  return launch_k(k_attn_prefill<HD, G>, dim3((a.rows + CR - 1) / CR, a.kv_heads), dim3(kPfThreads), smem,
                  st, a, scale);
}

template <int HD>
int launch_prefill_hd(const AttnArgs& a, int G, float scale, cudaStream_t st) {
  switch (G) {
    case 1: return launch_prefill_t<HD, 1>(a, scale, st);
    case 2: return launch_prefill_t<HD, 2>(a, scale, st);
    case 4: return launch_prefill_t<HD, 4>(a, scale, st);
    case 8: return launch_prefill_t<HD, 8>(a, scale, st);
  }
  return fail(WL_ERR_UNSUPPORTED, "prefill attention: heads per KV head must be 1, 2, 4 or 8");
}

// ---------------------------------------------------------------- contiguous f32 KV (op API)
template <int HD, int G>
__global__ void __launch_bounds__(kAttnThreads)
    k_attn_f32(const float* q, const float* k, const float* v, int past, int heads, int kvd,
               int window, float scale, float* out) {
  constexpr int LPT = HD / 8;
  constexpr int TPW = 32 / LPT;
  constexpr int NW = kAttnThreads / 32;
  constexpr int DP = HD / 2;
  constexpr int NS = kAttnThreads / DP;
  __shared__ float s_p[G][kTile];
  __shared__ float s_m[G], s_l[G], s_alpha[G];
  __shared__ float s_red[NS][G][HD];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kvh = blockIdx.x, r = blockIdx.y;
  const int ldq = heads * HD;
  const int pos = past + r;
  const int j0 = (window > 0 && pos - window + 1 > 0) ? pos - window + 1 : 0;
  const int sub = lane / LPT, li = lane % LPT;
  float qr[G][8];
#pragma unroll
  for (int h = 0; h < G; h++)
#pragma unroll
    for (int i = 0; i < 8; i++) qr[h][i] = q[(size_t)r * ldq + (size_t)(kvh * G + h) * HD + li * 8 + i];
  if (tid < G) s_m[tid] = -INFINITY, s_l[tid] = 0.f;
  const int stream = tid / DP, dp = tid % DP;
  float o[G][2];
#pragma unroll
  for (int h = 0; h < G; h++) o[h][0] = o[h][1] = 0.f;
  __syncthreads();
  for (int t0 = j0; t0 <= pos; t0 += kTile) {
    const int n = min(kTile, pos + 1 - t0);
    for (int base = warp * TPW; base < n; base += NW * TPW) {
      const int tok = base + sub;
      const bool ok = tok < n;
      float kf[8];
#pragma unroll
      for (int i = 0; i < 8; i++) kf[i] = ok ? k[(size_t)(t0 + tok) * kvd + kvh * HD + li * 8 + i] : 0.f;
#pragma unroll
      for (int h = 0; h < G; h++) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) s += qr[h][i] * kf[i];
#pragma unroll
        for (int off = LPT / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (ok && li == 0) s_p[h][tok] = s * scale;
      }
    }
    __syncthreads();
    for (int h = warp; h < G; h += NW) {
      float mx = -INFINITY;
      for (int i = lane; i < n; i += 32) mx = fmaxf(mx, s_p[h][i]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = s_m[h];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.f;
      for (int i = lane; i < n; i += 32) {
        const float p = expf(s_p[h][i] - m_new);
        s_p[h][i] = p;
        sum += p;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      __syncwarp();
      if (lane == 0) {
        const float alpha = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
        s_alpha[h] = alpha;
        s_l[h] = s_l[h] * alpha + sum;
        s_m[h] = m_new;
      }
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < G; h++) o[h][0] *= s_alpha[h], o[h][1] *= s_alpha[h];
    for (int tok = stream; tok < n; tok += NS) {
      const float2 vv = *reinterpret_cast<const float2*>(v + (size_t)(t0 + tok) * kvd + kvh * HD + 2 * dp);
#pragma unroll
      for (int h = 0; h < G; h++) {
        o[h][0] += s_p[h][tok] * vv.x;
        o[h][1] += s_p[h][tok] * vv.y;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int h = 0; h < G; h++) {
    s_red[stream][h][2 * dp] = o[h][0];
    s_red[stream][h][2 * dp + 1] = o[h][1];
  }
  __syncthreads();
  for (int i = tid; i < G * HD; i += kAttnThreads) {
    const int h = i / HD, d = i % HD;
    float acc = 0.f;
#pragma unroll
    for (int s = 0; s < NS; s++) acc += s_red[s][h][d];
    const float l = s_l[h];
    out[(size_t)r * ldq + (size_t)(kvh * G + h) * HD + d] = l > 0.f ? acc * (1.0f / l) : 0.f;
  }
}

template <int HD>
int launch_f32_hd(const float* q, const float* k, const float* v, int rows, int past, int heads,
                  int kv_heads, int window, float* out, cudaStream_t st) {
  const dim3 grid(kv_heads, rows);
  const float scale = 1.0f / sqrtf((float)HD);
  const int kvd = kv_heads * HD;
  switch (heads / kv_heads) {
    case 1: k_attn_f32<HD, 1><<<grid, kAttnThreads, 0, st>>>(q, k, v, past, heads, kvd, window, scale, out); break;
    case 2: k_attn_f32<HD, 2><<<grid, kAttnThreads, 0, st>>>(q, k, v, past, heads, kvd, window, scale, out); break;
    case 4: k_attn_f32<HD, 4><<<grid, kAttnThreads, 0, st>>>(q, k, v, past, heads, kvd, window, scale, out); break;
    case 8: k_attn_f32<HD, 8><<<grid, kAttnThreads, 0, st>>>(q, k, v, past, heads, kvd, window, scale, out); break;
    default: return fail(WL_ERR_UNSUPPORTED, "attention: heads per KV head must be 1, 2, 4 or 8");
  }
  WL_CUDA_TRY(cudaGetLastError());
  return WL_OK;
}

}  // namespace

int attention_plan_splits(int rows, int kv_heads, int max_len, int num_sms) {
  // CTAs to aim for: 2 per SM for few (KV head, row) pairs (2-page rounds);
  // kAttnSplitCtasPerSm once there is one pair per SM (1-page rounds; the
  // split partials then stay within kAttnSplitCtasPerSm * SMs + rows rows)
  const int ctas = rows * kv_heads;
  const int target = (ctas >= num_sms ? kAttnSplitCtasPerSm : 2) * num_sms;
  int ns = (target + ctas - 1) / ctas;
  const int pages = (max_len + kPage - 1) / kPage;
  const int by_len = (pages + 3) / 4;  // at least ~4 pages per split
  ns = ns < by_len ? ns : by_len;
  if (ns > 64) ns = 64;
  return ns < 1 ? 1 : ns;
}

int launch_attention_paged(const AttnArgs& a, cudaStream_t st) {
  if (a.kv.page != kPage) return fail(WL_ERR_UNSUPPORTED, "attention: KV page must be 16 tokens");
  if (a.heads % a.kv_heads) return fail(WL_ERR_INVALID_ARGUMENT, "attention: heads % kv_heads != 0");
  const int G = a.heads / a.kv_heads;
  const float scale = 1.0f / sqrtf((float)a.head_dim);
  switch (a.head_dim) {
    case 64: return launch_paged_hd<64>(a, G, scale, st);
    case 128: return launch_paged_hd<128>(a, G, scale, st);
    case 256: return launch_paged_hd<256>(a, G, scale, st);
  }
  return fail(WL_ERR_UNSUPPORTED, "attention: head_dim must be 64, 128 or 256");
}

bool attention_prefill_ok(int heads, int kv_heads, int head_dim) {
  if (kv_heads <= 0 || heads % kv_heads) return false;
  const int G = heads / kv_heads;
  return (head_dim == 64 || head_dim == 128) && (G == 1 || G == 2 || G == 4 || G == 8);
}

int launch_attention_prefill(const AttnArgs& a, cudaStream_t st) {
  if (a.kv.page != kPage) return fail(WL_ERR_UNSUPPORTED, "attention: KV page must be 16 tokens");
  if (!attention_prefill_ok(a.heads, a.kv_heads, a.head_dim))
    return fail(WL_ERR_UNSUPPORTED, "prefill attention: head_dim 64 / 128 and 1, 2, 4 or 8 heads per KV head");
  if (a.rows <= 0) return WL_OK;
  const int G = a.heads / a.kv_heads;
  const float scale = 1.0f / sqrtf((float)a.head_dim);
  return a.head_dim == 64 ? launch_prefill_hd<64>(a, G, scale, st) : launch_prefill_hd<128>(a, G, scale, st);
}

int launch_attention_f32(const float* q, const float* k, const float* v, int rows, int past,
                         int heads, int kv_heads, int hd, int window, float* out,
                         cudaStream_t st) {
  if (heads % kv_heads) return fail(WL_ERR_INVALID_ARGUMENT, "attention: heads % kv_heads != 0");
  switch (hd) {
    case 32: return launch_f32_hd<32>(q, k, v, rows, past, heads, kv_heads, window, out, st);
    case 64: return launch_f32_hd<64>(q, k, v, rows, past, heads, kv_heads, window, out, st);
    case 128: return launch_f32_hd<128>(q, k, v, rows, past, heads, kv_heads, window, out, st);
    case 256: return launch_f32_hd<256>(q, k, v, rows, past, heads, kv_heads, window, out, st);
  }
  return fail(WL_ERR_UNSUPPORTED, "attention: head_dim must be 32, 64, 128 or 256");
}

}  // namespace wl
