// GQA attention for decode and prefill rows (sm_100a).
//
// Reference: LazyTransformer::compute_optimized_gqa_attention
// (woolly-core/src/model/lazy_transformer.rs:360-434): for query head h the
// KV head is h / (H / KVH); scores q.k * hd^-1/2 over keys 0..=pos (causal,
// the KV cache holds past ++ new); max-subtracted softmax; output sum p_j v_j.
// The optional window W keeps keys j in (pos - W, pos] (Mistral shape; no
// reference counterpart).
//
// Flash-decoding: one CTA per (KV head, query row, context split).  The CTA
// streams K/V rows of its split once for all G = H/KVH query heads of the
// group (GQA reuse), keeps an online softmax per head, and writes either the
// final row (one split) or an unnormalised partial (o, m, l) that
// k_attn_combine merges with the log-sum-exp rule.  K/V rows are 16-byte
// vector loads of a paged f16 cache (pages of `page` tokens, per-session page
// table), coalesced across the lanes that share a token.
#include <cuda_fp16.h>

#include <cmath>
#include <string>

#include "common.h"
#include "kernels.cuh"

namespace wl {
namespace {

constexpr int kAttnThreads = 128;
constexpr int kTile = 64;  // tokens per softmax tile

struct PagedKV {
  const __half* k;
  const __half* v;
  const int* table;
  int maxp, page, kvd;
  __device__ __forceinline__ size_t row(int sess, int j) const {
    int pg = __ldg(table + (size_t)sess * maxp + j / page);
    return ((size_t)pg * page + (j % page)) * kvd;
  }
  __device__ __forceinline__ void k8(int sess, int j, int off, float* f) const {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(k + row(sess, j) + off));
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float2 t = __half22float2(h[i]);
      f[2 * i] = t.x, f[2 * i + 1] = t.y;
    }
  }
  __device__ __forceinline__ float2 v2(int sess, int j, int off) const {
    return __half22float2(__ldg(reinterpret_cast<const __half2*>(v + row(sess, j) + off)));
  }
};

struct F32KV {
  const float* k;
  const float* v;
  int kvd;
  __device__ __forceinline__ void k8(int, int j, int off, float* f) const {
    const float4* p = reinterpret_cast<const float4*>(k + (size_t)j * kvd + off);
    float4 a = __ldg(p), b = __ldg(p + 1);
    f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
  }
  __device__ __forceinline__ float2 v2(int, int j, int off) const {
    return __ldg(reinterpret_cast<const float2*>(v + (size_t)j * kvd + off));
  }
};

struct RowInfo {
  const int* pos;   // nullptr: pos = past + row
  const int* sess;  // nullptr: session 0
  int past;
};

template <class KV>
struct Params {
  KV kv;
  RowInfo ri;
  const float* q;
  int ldq;
  int heads, kv_heads, window, nsplit;
  float scale;
  float* part_o;
  float* part_ml;
  void* out;
  int ldo, out_f16;
};

template <int HD, int G, class KV>
__global__ void __launch_bounds__(kAttnThreads) k_attn(const Params<KV> a) {
  constexpr int LPT = HD / 8;  // lanes per token in the score phase
  constexpr int TPW = 32 / LPT;
  constexpr int NW = kAttnThreads / 32;
  constexpr int DP = HD / 2;   // dim pairs in the V phase
  constexpr int NS = kAttnThreads / DP;  // token streams in the V phase
  __shared__ float s_p[G][kTile];
  __shared__ float s_m[G], s_l[G], s_alpha[G];
  __shared__ float s_red[NS][G][HD];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kvh = blockIdx.x, r = blockIdx.y, sp = blockIdx.z;
  const int pos = a.ri.pos ? a.ri.pos[r] : a.ri.past + r;
  const int sess = a.ri.sess ? a.ri.sess[r] : 0;
  const int j0 = (a.window > 0 && pos - a.window + 1 > 0) ? pos - a.window + 1 : 0;
  const int len = pos + 1 - j0;
  const int chunk = (len + a.nsplit - 1) / a.nsplit;
  const int ja = j0 + sp * chunk;
  const int jb = min(pos + 1, ja + chunk);

  const int sub = lane / LPT, li = lane % LPT;
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

  for (int t0 = ja; t0 < jb; t0 += kTile) {
    const int n = min(kTile, jb - t0);
    for (int base = warp * TPW; base < n; base += NW * TPW) {
      const int tok = base + sub;
      const bool ok = tok < n;
      float kf[8];
      if (ok)
        a.kv.k8(sess, t0 + tok, kvh * HD + li * 8, kf);
      else
#pragma unroll
        for (int i = 0; i < 8; i++) kf[i] = 0.f;
#pragma unroll
      for (int h = 0; h < G; h++) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) s += qr[h][i] * kf[i];
#pragma unroll
        for (int off = LPT / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (ok && li == 0) s_p[h][tok] = s * a.scale;
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
        float p = expf(s_p[h][i] - m_new);
        s_p[h][i] = p;
        sum += p;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      __syncwarp();
      if (lane == 0) {
        float alpha = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
        s_alpha[h] = alpha;
        s_l[h] = s_l[h] * alpha + sum;
        s_m[h] = m_new;
      }
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < G; h++) {
      float al = s_alpha[h];
      o[h][0] *= al, o[h][1] *= al;
    }
    for (int tok = stream; tok < n; tok += NS) {
      float2 vv = a.kv.v2(sess, t0 + tok, kvh * HD + 2 * dp);
#pragma unroll
      for (int h = 0; h < G; h++) {
        float p = s_p[h][tok];
        o[h][0] += p * vv.x;
        o[h][1] += p * vv.y;
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
    const int qh = kvh * G + h;
    if (a.nsplit == 1) {
      const float l = s_l[h];
      const float v = l > 0.f ? acc * (1.0f / l) : 0.f;
      const size_t oi = (size_t)r * a.ldo + (size_t)qh * HD + d;
      if (a.out_f16)
        reinterpret_cast<__half*>(a.out)[oi] = __float2half_rn(v);
      else
        reinterpret_cast<float*>(a.out)[oi] = v;
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
                               void* out, int ldo, int out_f16) {
  const int r = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const size_t base = ((size_t)r * heads + h) * nsplit;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; s++) M = fmaxf(M, part_ml[(base + s) * 2]);
  float L = 0.f, acc = 0.f;
  for (int s = 0; s < nsplit; s++) {
    float m = part_ml[(base + s) * 2];
    if (m == -INFINITY) continue;
    float w = expf(m - M);
    L += part_ml[(base + s) * 2 + 1] * w;
    acc += part_o[(base + s) * HD + d] * w;
  }
  float v = L > 0.f ? acc * (1.0f / L) : 0.f;
  size_t oi = (size_t)r * ldo + (size_t)h * HD + d;
  if (out_f16)
    reinterpret_cast<__half*>(out)[oi] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(out)[oi] = v;
}

template <int HD, class KV>
int launch_g(const Params<KV>& p, int rows, int G, cudaStream_t st) {
  dim3 grid(p.kv_heads, rows, p.nsplit);
  switch (G) {
    case 1: k_attn<HD, 1, KV><<<grid, kAttnThreads, 0, st>>>(p); break;
    case 2: k_attn<HD, 2, KV><<<grid, kAttnThreads, 0, st>>>(p); break;
    case 4: k_attn<HD, 4, KV><<<grid, kAttnThreads, 0, st>>>(p); break;
    case 8: k_attn<HD, 8, KV><<<grid, kAttnThreads, 0, st>>>(p); break;
    default:
      return fail(WL_ERR_UNSUPPORTED,
                  "attention: heads per KV head must be 1, 2, 4 or 8 (got " + std::to_string(G) + ")");
  }
  WL_CUDA_TRY(cudaGetLastError());
  if (p.nsplit > 1) {
    k_attn_combine<HD><<<dim3(rows, p.heads), HD, 0, st>>>(p.part_o, p.part_ml, p.heads,
                                                            p.nsplit, p.out, p.ldo, p.out_f16);
    WL_CUDA_TRY(cudaGetLastError());
  }
  return WL_OK;
}

template <class KV>
int launch_any(const Params<KV>& p, int rows, int hd, cudaStream_t st) {
  if (p.heads % p.kv_heads) return fail(WL_ERR_INVALID_ARGUMENT, "attention: heads % kv_heads != 0");
  int G = p.heads / p.kv_heads;
  switch (hd) {
    case 32: return launch_g<32>(p, rows, G, st);
    case 64: return launch_g<64>(p, rows, G, st);
    case 128: return launch_g<128>(p, rows, G, st);
    case 256: return launch_g<256>(p, rows, G, st);
  }
  return fail(WL_ERR_UNSUPPORTED, "attention: head_dim must be 32, 64, 128 or 256");
}

}  // namespace

int attention_plan_splits(int rows, int kv_heads, int max_len, int num_sms) {
  int ctas = rows * kv_heads;
  int target = 2 * num_sms;
  int ns = (target + ctas - 1) / ctas;
  int by_len = (max_len + kTile - 1) / kTile;  // at least one tile per split
  ns = ns < by_len ? ns : by_len;
  if (ns > 64) ns = 64;
  return ns < 1 ? 1 : ns;
}

int launch_attention_paged(const AttnArgs& a, cudaStream_t st) {
  Params<PagedKV> p;
  p.kv = PagedKV{a.kv.k, a.kv.v, a.kv.page_table, a.kv.max_pages, a.kv.page, a.kv.kvd};
  p.ri = RowInfo{a.row_pos, a.row_sess, 0};
  p.q = a.q;
  p.ldq = a.ldq;
  p.heads = a.heads;
  p.kv_heads = a.kv_heads;
  p.window = a.window;
  p.nsplit = a.nsplit;
  p.scale = 1.0f / sqrtf((float)a.head_dim);
  p.part_o = a.part_o;
  p.part_ml = a.part_ml;
  p.out = a.out;
  p.ldo = a.ldo;
  p.out_f16 = a.out_f16;
  return launch_any(p, a.rows, a.head_dim, st);
}

int launch_attention_f32(const float* q, const float* k, const float* v, int rows, int past,
                         int heads, int kv_heads, int hd, int window, float* out,
                         cudaStream_t st) {
  Params<F32KV> p;
  p.kv = F32KV{k, v, kv_heads * hd};
  p.ri = RowInfo{nullptr, nullptr, past};
  p.q = q;
  p.ldq = heads * hd;
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.window = window;
  p.nsplit = 1;
  p.scale = 1.0f / sqrtf((float)hd);
  p.part_o = nullptr;
  p.part_ml = nullptr;
  p.out = out;
  p.ldo = heads * hd;
  p.out_f16 = 0;
  return launch_any(p, rows, hd, st);
}

}  // namespace wl
