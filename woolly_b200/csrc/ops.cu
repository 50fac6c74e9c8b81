// Row-wise and element-wise kernels: RMSNorm(+RoPE), embedding gather,
// SwiGLU, RoPE, block dequantization.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <string>

#include "common.h"
#include "kernels.cuh"
#include "pdl.cuh"

namespace wl {
namespace {

constexpr int kNormThreads = 256;

// rms_norm (woolly-core tensor_utils.rs:446-480): rms = sqrt(sum(x^2)/d + eps),
// y = (x / rms) * w, with an optional NeoX rotation (RoPE::apply_f32,
// woolly-tensor/src/ops/mod.rs:476-527) of the normalised row, head by head.
__device__ __forceinline__ void put_y(void* y, int mode, size_t plane, size_t i, float v) {
  if (mode == 0) {
    reinterpret_cast<float*>(y)[i] = v;
  } else {
    const __half hi = __float2half_rn(v);
    reinterpret_cast<__half*>(y)[i] = hi;
    if (mode == 2) reinterpret_cast<__half*>(y)[i + plane] = __float2half_rn(v - __half2float(hi));
  }
}

__global__ void __launch_bounds__(kNormThreads)
    k_rmsnorm(const float* x, const float* w, int dim, float eps, int rope, const int* pos,
              int hd, float theta, void* y, int y_mode, size_t y_plane) {
  extern __shared__ float srow[];  // normalised row when rope is on
  __shared__ float sred[kNormThreads / 32];
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x, tid = threadIdx.x;
  const float* xr = x + (size_t)r * dim;
  float ss = 0.f;
  for (int i = tid; i < dim; i += kNormThreads) ss += xr[i] * xr[i];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((tid & 31) == 0) sred[tid >> 5] = ss;
  __syncthreads();
  if (tid < 32) {
    float v = tid < kNormThreads / 32 ? sred[tid] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (tid == 0) sred[0] = v;
  }
  __syncthreads();
  const float rms = sqrtf(sred[0] / (float)dim + eps);
  if (!rope) {
    for (int i = tid; i < dim; i += kNormThreads)
      put_y(y, y_mode, y_plane, (size_t)r * dim + i, __fdiv_rn(xr[i], rms) * w[i]);
    return;
  }
  for (int i = tid; i < dim; i += kNormThreads) srow[i] = __fdiv_rn(xr[i], rms) * w[i];
  __syncthreads();
  const int half = hd / 2;
  const float p = (float)pos[r];
  for (int j = tid; j < dim / 2; j += kNormThreads) {
    int h = j / half, ii = j % half;
    int c1 = h * hd + ii, c2 = c1 + half;
    float freq = 1.0f / powf(theta, 2.0f * (float)ii / (float)hd);
    float sn, cs;
    sincosf(p * freq, &sn, &cs);
    float x1 = srow[c1], x2 = srow[c2];
    put_y(y, y_mode, y_plane, (size_t)r * dim + c1, x1 * cs - x2 * sn);
    put_y(y, y_mode, y_plane, (size_t)r * dim + c2, x1 * sn + x2 * cs);
  }
}

// Same RMSNorm without rotation, one CTA per row with up to 1024 threads: each
// thread keeps V4 float4 chunks of the row in registers (one read), the sum of
// squares is reduced across the CTA, and the outputs are stored 4 at a time.
// With pr.nranks > 0 the row is first completed from the tensor-parallel
// partial sums the ranks pushed into pr.slots (x += sum over ranks, in rank
// order, written back to x) after a bounded wait for every rank's arrivals;
// CTAs at or past nrows only take part in the wait (a drain launch).
template <int V4>
__global__ void __launch_bounds__(1024) k_rmsnorm_v(const float* x, const float* w, int dim, float eps,
                                                    void* y, int y_mode, size_t y_plane,
                                                    PeerReduce pr, int nrows) {
  __shared__ float sred[32];
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  const int n4 = dim >> 2;
  if (pr.nranks) peer_wait(pr);
  if (r < nrows) {
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)r * dim);
    float4 v[V4];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < V4; j++) {
      const int i = tid + j * nt;
      v[j] = i < n4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      if (pr.nranks && i < n4) {
        for (int src = 0; src < pr.nranks; src++) {
          const float4 p = __ldcg(reinterpret_cast<const float4*>(
                                      pr.slots + ((size_t)src * kPeerRows + pr.row0 + r) * dim) + i);
          v[j].x += p.x;
          v[j].y += p.y;
          v[j].z += p.z;
          v[j].w += p.w;
        }
        reinterpret_cast<float4*>(const_cast<float*>(x) + (size_t)r * dim)[i] = v[j];
      }
      ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((tid & 31) == 0) sred[tid >> 5] = ss;
    __syncthreads();
    if (tid < 32) {
      float t = tid < (nt >> 5) ? sred[tid] : 0.f;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
      if (tid == 0) sred[0] = t;
    }
    __syncthreads();
    const float rms = sqrtf(sred[0] / (float)dim + eps);
    const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
    for (int j = 0; j < V4; j++) {
      const int i = tid + j * nt;
      if (i >= n4) break;
      const float4 wv = w4[i];
      const float o[4] = {__fdiv_rn(v[j].x, rms) * wv.x, __fdiv_rn(v[j].y, rms) * wv.y,
                          __fdiv_rn(v[j].z, rms) * wv.z, __fdiv_rn(v[j].w, rms) * wv.w};
      const size_t at = (size_t)r * dim + 4 * (size_t)i;
      if (y_mode == 0) {
        reinterpret_cast<float4*>(y)[at >> 2] = make_float4(o[0], o[1], o[2], o[3]);
      } else {
        __half hi[4], lo[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          hi[q] = __float2half_rn(o[q]);
          lo[q] = __float2half_rn(o[q] - __half2float(hi[q]));
        }
        __half* yh = reinterpret_cast<__half*>(y);
        *reinterpret_cast<uint2*>(yh + at) = *reinterpret_cast<const uint2*>(hi);
        if (y_mode == 2) *reinterpret_cast<uint2*>(yh + at + y_plane) = *reinterpret_cast<const uint2*>(lo);
      }
    }
  }
  if (pr.nranks) peer_release(pr);
}

// h[r][j] = E[j*V + id]: token_embd is [d][V] in woolly's reading
// (lazy_transformer.rs:1252-1262).  Out-of-range ids raise a flag and read id 0.
__global__ void k_embed(const float* E, int d, int V, const uint32_t* ids, int rows, float* h,
                        int* err, int token_rows) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.y;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= d || r >= rows) return;
  uint32_t t = ids[r];
  if (t >= (uint32_t)V) {
    if (err && j == 0) atomicOr(err, 1);
    t = 0;
  }
  h[(size_t)r * d + j] = __ldg(E + (token_rows ? (size_t)t * d + j : (size_t)j * V + t));
}

// Layout-A (ggml orientation) attention input: the q/k/v projections as f32
// rows; NeoX RoPE (RoPE::apply_f32, woolly-tensor/src/ops/mod.rs:476-527) on
// the q and k heads at each row's position when `rope`, q written back as
// f32, k and v appended to the row's KV page as f16.
__global__ void k_qkv_post(float* q, const float* k, const float* v, int rows, int H, int KVH, int hd,
                           int rope, float theta, const int* row_pos, const int* row_sess,
                           KvPages kv) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.y;
  const int half = hd / 2;
  const int nq = H * half, nk = KVH * half;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows || i >= nq + 2 * nk) return;
  const int pos = row_pos[r];
  const int pg = kv.page_table[(size_t)row_sess[r] * kv.max_pages + pos / kv.page];
  auto rot = [&](float a, float b, int ii, float& x1, float& x2) {
    if (!rope) {
      x1 = a, x2 = b;
      return;
    }
    const float freq = 1.0f / powf(theta, 2.0f * (float)ii / (float)hd);
    float sn, cs;
    sincosf((float)pos * freq, &sn, &cs);
    x1 = a * cs - b * sn;
    x2 = a * sn + b * cs;
  };
  if (i < nq) {  // q pair (h, ii), (h, ii + hd/2)
    const int h = i / half, ii = i % half;
    float* qr = q + (size_t)r * H * hd + (size_t)h * hd;
    float x1, x2;
    rot(qr[ii], qr[ii + half], ii, x1, x2);
    qr[ii] = x1;
    qr[ii + half] = x2;
  } else if (i < nq + nk) {  // k pair
    const int j = i - nq, h = j / half, ii = j % half;
    const float* kr = k + (size_t)r * KVH * hd + (size_t)h * hd;
    float x1, x2;
    rot(kr[ii], kr[ii + half], ii, x1, x2);
    kv.k[kv_offset(kv, pg, pos % kv.page, h, ii)] = __float2half_rn(x1);
    kv.k[kv_offset(kv, pg, pos % kv.page, h, ii + half)] = __float2half_rn(x2);
  } else {  // v pair (no rotation)
    const int j = i - nq - nk, h = j / half, ii = j % half;
    const float* vr = v + (size_t)r * KVH * hd + (size_t)h * hd;
    kv.v[kv_offset(kv, pg, pos % kv.page, h, ii)] = __float2half_rn(vr[ii]);
    kv.v[kv_offset(kv, pg, pos % kv.page, h, ii + half)] = __float2half_rn(vr[ii + half]);
  }
}


// swiglu (tensor_utils.rs:512-532): silu(g) * u with silu(g) = g * (1 / (1 + exp(-g)))
__global__ void k_swiglu(const float* g, const float* u, size_t n, float* out) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  float gi = g[i];
  out[i] = gi * (1.0f / (1.0f + expf(-gi))) * u[i];
}

// RoPE::apply_f32 (woolly-tensor/src/ops/mod.rs:476-527)
__global__ void k_rope(const float* x, float* out, const int* pos, float base, int batch, int seq,
                       int heads, int hd) {
  const int half = hd / 2;
  size_t total = (size_t)batch * seq * heads * half;
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= total) return;
  int ii = (int)(i % half);
  size_t rowh = i / half;  // (batch, seq, head)
  int s = (int)((rowh / heads) % seq);
  float freq = 1.0f / powf(base, 2.0f * (float)ii / (float)hd);
  float ang = (float)pos[s] * freq;
  float sn, cs;
  sincosf(ang, &sn, &cs);
  size_t b1 = rowh * hd + ii, b2 = b1 + half;
  float x1 = x[b1], x2 = x[b2];
  out[b1] = x1 * cs - x2 * sn;
  out[b2] = x1 * sn + x2 * cs;
}

// woolly_gguf::dequantize (dequantize.rs:286-327, :337-378, :553-586), one
// thread per 32-value block; bit-exact: (q-8)*d, q*d then +m (two roundings,
// no FMA), q*d with d widened exactly from f16.
// K-quant super-blocks of 256 values as woolly_gguf::dequantize reads them
// (one thread per value): Q4_K dequantize.rs:404-462 = d*scale[i/32]*q + dmin
// with 8 six-bit scales and nibble i%2 of byte i/2; Q6_K dequantize.rs:465-537
// = d*scale[i/16]*(q6 - 32)/64 with the reference's ql/qh indexing.  Each
// product and sum is rounded separately (no FMA), as in the Rust code.
__global__ void k_dequant_k(int type, const uint8_t* blocks, size_t n, float* out) {
  const size_t i_all = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i_all >= n) return;
  const size_t b = i_all / 256;
  const int i = (int)(i_all % 256);
  float v;
  if (type == 12) {
    const uint8_t* blk = blocks + b * 144;
    const int si = i / 32, src = (si * 3) / 2;
    const int sc = (si % 2 == 0) ? (blk[src] & 63) : (((blk[src] >> 6) | ((blk[src + 1] & 15) << 2)) & 63);
    const float d = __half2float(__ushort_as_half((uint16_t)(blk[12] | (blk[13] << 8))));
    const float dmin = __half2float(__ushort_as_half((uint16_t)(blk[14] | (blk[15] << 8))));
    const int q = (i % 2 == 0) ? (blk[16 + i / 2] & 15) : ((blk[16 + i / 2] >> 4) & 15);
    v = __fadd_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), dmin);
  } else {
    const uint8_t* blk = blocks + b * 210;
    const uint8_t *ql = blk, *qh = blk + 128, *scales = blk + 192;
    const float d = __half2float(__ushort_as_half((uint16_t)(blk[208] | (blk[209] << 8))));
    const int ql_idx = 64 * (i / 128) + 32 * ((i % 128) / 64) + 16 * ((i % 64) / 32) + (i % 16);
    const int qh_idx = 32 * (i / 128) + 16 * ((i % 128) / 64) + 8 * ((i % 64) / 32) + (i % 32) / 4;
    const int qh_shift = 2 * ((i % 32) % 4);
    const int qv = qh[qh_idx];
    const int q1_ext = (qv >> qh_shift) & 3;
    const int q2_ext = qh_shift < 6 ? ((qv >> (qh_shift + 2)) & 3) : (qh_idx + 1 < 64 ? (qh[qh_idx + 1] & 3) : 0);
    const int q1 = (ql[ql_idx] & 15) | (q1_ext << 4), q2 = (ql[ql_idx] >> 4) | (q2_ext << 4);
    const int q = i < 128 ? q1 : q2;
    v = __fdiv_rn(__fmul_rn(__fmul_rn(d, (float)scales[i / 16]), (float)(q - 32)), 64.0f);
  }
  out[i_all] = v;
}

__global__ void k_dequant(int type, const uint8_t* blocks, size_t n, float* out) {
  size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t nb = (n + 31) / 32;
  if (b >= nb) return;
  const int S = type == WL_Q4_0 ? 18 : type == WL_Q4_1 ? 20 : 34;
  const uint8_t* p = blocks + b * S;
  float d = __half2float(__ushort_as_half((uint16_t)(p[0] | (p[1] << 8))));
  size_t o0 = b * 32;
  for (int i = 0; i < 32 && o0 + i < n; i++) {
    float v;
    if (type == WL_Q4_0) {
      int q = i < 16 ? (p[2 + i] & 15) - 8 : ((p[2 + i - 16] >> 4) & 15) - 8;
      v = __fmul_rn((float)q, d);
    } else if (type == WL_Q4_1) {
      float m = __half2float(__ushort_as_half((uint16_t)(p[2] | (p[3] << 8))));
      int q = i < 16 ? (p[4 + i] & 15) : ((p[4 + i - 16] >> 4) & 15);
      v = __fadd_rn(__fmul_rn((float)q, d), m);
    } else {
      v = __fmul_rn((float)(int8_t)p[2 + i], d);
    }
    out[o0 + i] = v;
  }
}

__global__ void k_f16_to_f32(const uint8_t* src, size_t n, float* out) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) out[i] = __half2float(__ushort_as_half((uint16_t)(src[2 * i] | (src[2 * i + 1] << 8))));
}

}  // namespace

int launch_qkv_post(float* q, const float* k, const float* v, int rows, int H, int KVH, int hd,
                    int rope, float theta, const int* row_pos, const int* row_sess, const KvPages& kv,
                    cudaStream_t st) {
  if (!rows) return WL_OK;
  const int n = (H + 2 * KVH) * (hd / 2);
  return launch_k(k_qkv_post, dim3((n + 255) / 256, rows), dim3(256), 0, st, q, k, v, rows, H, KVH, hd,
                  rope, theta, row_pos, row_sess, kv);
}

static int rmsnorm_v(const float* x, const float* w, int rows, int dim, float eps, void* y,
                     int y_mode, size_t y_plane, const PeerReduce& pr, cudaStream_t st) {
  const int n4 = dim / 4;
  const int v4 = (n4 + 1023) / 1024;
  int nt = (n4 + v4 - 1) / v4;
  nt = std::max(32, (nt + 31) / 32 * 32);
  const dim3 grid(std::max(rows, 1));
  switch (v4) {
    case 1: return launch_k(k_rmsnorm_v<1>, grid, dim3(nt), 0, st, x, w, dim, eps, y, y_mode, y_plane, pr, rows);
    case 2: return launch_k(k_rmsnorm_v<2>, grid, dim3(nt), 0, st, x, w, dim, eps, y, y_mode, y_plane, pr, rows);
    case 3: return launch_k(k_rmsnorm_v<3>, grid, dim3(nt), 0, st, x, w, dim, eps, y, y_mode, y_plane, pr, rows);
    default: return launch_k(k_rmsnorm_v<4>, grid, dim3(nt), 0, st, x, w, dim, eps, y, y_mode, y_plane, pr, rows);
  }
}

int launch_rmsnorm_peer(float* x, const float* w, int rows, int dim, float eps, void* y,
                        size_t y_plane, const PeerReduce& pr, cudaStream_t st) {
  if (pr.nranks < 1 || pr.nranks > kMaxPeers || !pr.slots || !pr.flags || !pr.done)
    return fail(WL_ERR_INVALID_ARGUMENT, "rmsnorm_peer: bad peer arguments");
  if (dim % 4 || dim > 16384 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(y) & 15) || y_plane % 4 ||
      rows < 0 || pr.row0 + rows > kPeerRows)
    return fail(WL_ERR_INVALID_ARGUMENT, "rmsnorm_peer: dim % 4, alignment or rows out of range");
  return rmsnorm_v(x, w, rows, dim, eps, y, 2, y_plane, pr, st);
}

int launch_rmsnorm(const float* x, const float* w, int rows, int dim, float eps, int rope,
                   const int* pos, int head_dim, float theta, void* y, int y_mode,
                   size_t y_plane, cudaStream_t st) {
  if (rows <= 0) return WL_OK;
  // vector path: no rotation, dim % 4 == 0, aligned rows and (for planes) an 8-byte aligned lo plane
  const bool vec_ok = !rope && dim % 4 == 0 && dim <= 16384 &&
                      (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(y) & 15) == 0 && (y_mode != 2 || y_plane % 4 == 0);
  if (vec_ok) {
    const int n4 = dim / 4;
    const int v4 = (n4 + 1023) / 1024;
    int nt = (n4 + v4 - 1) / v4;
    nt = (nt + 31) / 32 * 32;
    return rmsnorm_v(x, w, rows, dim, eps, y, y_mode, y_plane, PeerReduce{}, st);
  }
  size_t smem = rope ? (size_t)dim * sizeof(float) : 0;
  if (rope && (head_dim <= 0 || dim % head_dim || head_dim % 2))
    return fail(WL_ERR_INVALID_ARGUMENT, "rmsnorm_rope: dim must be a multiple of an even head_dim");
  if (smem > 48 * 1024) {
    WL_CUDA_TRY(cudaFuncSetAttribute(k_rmsnorm, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
  }
  return launch_k(k_rmsnorm, dim3(rows), dim3(kNormThreads), smem, st, x, w, dim, eps, rope, pos,
                  head_dim, theta, y, y_mode, y_plane);
}

int launch_embed(const float* E, int d, int V, const uint32_t* ids, int rows, float* h,
                 int* err_flag, cudaStream_t st, int token_rows) {
  if (rows <= 0) return WL_OK;
  dim3 grid((d + 255) / 256, rows);
  return launch_k(k_embed, grid, dim3(256), 0, st, E, d, V, ids, rows, h, err_flag, token_rows);
}

int launch_swiglu(const float* g, const float* u, size_t n, float* out, cudaStream_t st) {
  if (!n) return WL_OK;
  k_swiglu<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(g, u, n, out);
  WL_CUDA_TRY(cudaGetLastError());
  return WL_OK;
}

int launch_rope(const float* x, float* out, const int* pos, float base, int batch, int seq,
                int heads, int hd, cudaStream_t st) {
  size_t total = (size_t)batch * seq * heads * (hd / 2);
  if (!total) return WL_OK;
  k_rope<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(x, out, pos, base, batch, seq, heads, hd);
  WL_CUDA_TRY(cudaGetLastError());
  return WL_OK;
}

__global__ void k_gather_cols(const float* src, int T, int rows, int cols, float* dst) {
  pdl_wait();
  pdl_trigger();
  const size_t n = (size_t)T * rows * cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % cols);
    const size_t tr = i / cols;
    const int r = (int)(tr % rows), t = (int)(tr / rows);
    dst[((size_t)r * T + t) * cols + c] = src[i];
  }
}

int launch_gather_cols(const float* src, int T, int rows, int cols, float* dst, cudaStream_t st) {
  const size_t n = (size_t)T * rows * cols;
  if (!n) return WL_OK;
  return launch_k(k_gather_cols, dim3((unsigned)std::min<size_t>((n + 255) / 256, 4096)), dim3(256), 0,
                  st, src, T, rows, cols, dst);
}

__global__ void k_err_clear(int* err, int bits) { atomicAnd(err, ~bits); }

int launch_err_clear(int* err, int bits, cudaStream_t st) {
  k_err_clear<<<1, 1, 0, st>>>(err, bits);
  WL_CUDA_TRY(cudaGetLastError());
  return WL_OK;
}

int launch_dequant(int type, const void* blocks, size_t n, float* out, cudaStream_t st) {
  if (!n) return WL_OK;
  if (type == WL_F32) {
    WL_CUDA_TRY(cudaMemcpyAsync(out, blocks, n * 4, cudaMemcpyDeviceToDevice, st));
    return WL_OK;
  }
  if (type == WL_F16) {
    k_f16_to_f32<<<(unsigned)((n + 255) / 256), 256, 0, st>>>((const uint8_t*)blocks, n, out);
    WL_CUDA_TRY(cudaGetLastError());
    return WL_OK;
  }
  if (type == 12 || type == 14) {
    if (n) k_dequant_k<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(type, (const uint8_t*)blocks, n, out);
    WL_CUDA_TRY(cudaGetLastError());
    return WL_OK;
  }
  if (type == 6 || type == 7 || type == 13 || type == 15) {  // reference zero stubs
    if (n) WL_CUDA_TRY(cudaMemsetAsync(out, 0, n * sizeof(float), st));
    return WL_OK;
  }
  if (!(type == WL_Q4_0 || type == WL_Q4_1 || type == WL_Q8_0))
    return fail(WL_ERR_UNSUPPORTED, "dequantize: type " + std::to_string(type) + " not supported");
  const size_t nb = (n + 31) / 32;
  k_dequant<<<(unsigned)((nb + 127) / 128), 128, 0, st>>>(type, (const uint8_t*)blocks, n, out);
  WL_CUDA_TRY(cudaGetLastError());
  return WL_OK;
}

}  // namespace wl
