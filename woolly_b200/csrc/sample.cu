// Next-token sampling on the GPU (one CTA per row of logits), sm_100a.
//
// Reference: the server's decode loop samples each new token from the last
// row of logits with sample_next_token (woolly-server/src/handlers/
// inference.rs:441-483) and its helpers (:551-654):
//   probs = softmax((logits - max) / max(temperature, 0.01))
//   top_k > 0 (and < V): zero every prob below the k-th largest, renormalise
//   top_p < 1: keep the shortest prefix (descending prob, ties in index
//     order) whose cumulative sum exceeds top_p, zero the rest, renormalise;
//     when no prefix exceeds top_p nothing is kept (all zeros)
//   temperature == 0: the last index of the largest prob
//   else: the first index whose running sum (index order) exceeds a uniform
//     draw u in [0, 1); the last index when none does.
// The uniform draw of each row is an input, so the host keeps the random
// stream (one per request).
//
// Design: the row's probabilities live in shared memory (V <= kSampleMaxVocab);
// thread t owns the contiguous index range [t * NJ, (t + 1) * NJ), so every
// "in index order" rule is a per-thread sequential pass plus one block scan.
// The k-th largest value and the top-p cut value are found by a 4-pass
// most-significant-digit radix select over the IEEE bit patterns of the
// (non-negative) probabilities, with per-digit counts (top-k) or masses in
// integer fixed point (top-p), so the result does not depend on scheduling.
// Float sums run in a fixed tree order that differs from the reference's
// sequential f32 sums, so a draw within a few ulps of a cumulative boundary
// may pick the neighbouring token.
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>
#include <string>

#include "common.h"
#include "kernels.cuh"
#include "pdl.cuh"

namespace wl {
namespace {

constexpr int kST = 1024;  // threads per row
constexpr int kW = kST / 32;

template <class T, class Op>
__device__ __forceinline__ T block_reduce(T v, Op op, T* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();  // red may still be read from the previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = red[lane < kW ? lane : 0];
  if (warp == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// exclusive prefix sum over threads in thread order (fixed tree order)
template <class T>
__device__ __forceinline__ T block_exclusive_scan(T v, T* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) red[warp] = x;
  __syncthreads();
  if (warp == 0) {
    T w = red[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    red[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  return (warp ? red[warp - 1] : T(0)) + x - v;
}

// shared-memory slot of element e: one pad word per 32, so that the
// contiguous per-thread ranges (stride NJ) fall into different banks
__device__ __forceinline__ int pad(int e) { return e + (e >> 5); }

struct FMax {
  __device__ float operator()(float a, float b) const { return fmaxf(a, b); }
};
struct FAdd {
  __device__ float operator()(float a, float b) const { return a + b; }
};
struct IAdd {
  __device__ int operator()(int a, int b) const { return a + b; }
};
// (prob, index) argmax keeping the largest index among equal probs
struct ArgMaxLast {
  __device__ unsigned long long operator()(unsigned long long a, unsigned long long b) const {
    return a > b ? a : b;
  }
};

__global__ void __launch_bounds__(kST) k_sample(const float* logits, int V, int ld,
                                               const wl_sample_params* prm, uint32_t* out) {
  extern __shared__ float ps_[];  // [V + V / 32]: element e at e + e / 32 (no bank conflicts)
  __shared__ float redf[kW];
  __shared__ int redi[kW];
  __shared__ unsigned long long redu[kW];
  __shared__ unsigned hist[256];
  __shared__ unsigned long long mass[256];
  __shared__ int sel_digit, sel_rest;
  __shared__ unsigned long long sel_mass;
  const int r = blockIdx.x, tid = threadIdx.x;
  pdl_wait();
  pdl_trigger();
  const wl_sample_params P = prm[r];
  const float* x = logits + (size_t)r * ld;
  const int NJ = (V + kST - 1) / kST;
  const int j0 = min(V, tid * NJ), j1 = min(V, j0 + NJ);

  // softmax with temperature (inference.rs:551-565)
  float mx = -INFINITY;
  for (int i = tid; i < V; i += kST) {
    const float v = x[i];
    ps_[pad(i)] = v;
    mx = fmaxf(mx, v);
  }
  mx = block_reduce(mx, FMax(), redf);
  const float t = fmaxf(P.temperature, 0.01f);
  float s = 0.f;
  for (int i = j0; i < j1; i++) {
    const float e = expf((ps_[pad(i)] - mx) / t);
    ps_[pad(i)] = e;
    s += e;
  }
  s = block_reduce(s, FAdd(), redf);
  for (int i = j0; i < j1; i++) ps_[pad(i)] = ps_[pad(i)] / s;

  // top-k (inference.rs:568-591): threshold = the k-th largest prob, found
  // by a most-significant-digit radix select over the IEEE bit patterns
  // (probs are >= 0, so their patterns order like the values)
  if (P.top_k > 0 && P.top_k < V) {
    uint32_t pre = 0, msk = 0;
    int krem = P.top_k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += kST) hist[i] = 0;
      __syncthreads();
      for (int i = j0; i < j1; i++) {
        const uint32_t key = __float_as_uint(ps_[pad(i)]);
        const bool in = (key & msk) == pre;
        const unsigned dig = in ? (key >> shift) & 255u : 256u;
        // one atomic per distinct digit of the warp (probs cluster in few digits)
        const unsigned grp = __match_any_sync(__activemask(), dig);
        if (in && (__ffs(grp) - 1) == (int)(threadIdx.x & 31)) atomicAdd(&hist[dig], (unsigned)__popc(grp));
      }
      __syncthreads();
      if (tid < 32) {  // digit holding the krem-th largest of the group
        unsigned c8[8], tot = 0;
#pragma unroll
        for (int q = 0; q < 8; q++) c8[q] = hist[255 - (tid * 8 + q)], tot += c8[q];
        unsigned incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
          if (tid >= o) incl += y;
        }
        unsigned run = incl - tot;  // keys in higher digits than this lane's first
#pragma unroll
        for (int q = 0; q < 8; q++) {
          if (run < (unsigned)krem && run + c8[q] >= (unsigned)krem) {
            sel_digit = 255 - (tid * 8 + q);
            sel_rest = krem - (int)run;
          }
          run += c8[q];
        }
      }
      __syncthreads();
      pre |= (uint32_t)sel_digit << shift;
      msk |= 255u << shift;
      krem = sel_rest;
      __syncthreads();
    }
    const float thr = __uint_as_float(pre);
    float ks = 0.f;
    for (int i = j0; i < j1; i++) {
      if (ps_[pad(i)] < thr) ps_[pad(i)] = 0.f;
      ks += ps_[pad(i)];
    }
    ks = block_reduce(ks, FAdd(), redf);
    if (ks > 0.f)
      for (int i = j0; i < j1; i++) ps_[pad(i)] = ps_[pad(i)] / ks;
  }

  // top-p (inference.rs:594-630): the cut value tau is the largest bit
  // pattern b with mass(p >= b) > top_p (radix select over the patterns with
  // per-digit masses in 2^-40 fixed point, deterministic); every prob above
  // tau is kept and the probs equal to tau are kept in index order until the
  // running mass exceeds top_p.  No such b: nothing is kept.
  if (P.top_p < 1.0f) {
    bool any;
    {
      float m0 = 0.f;
      for (int i = j0; i < j1; i++) m0 += ps_[pad(i)];
      any = block_reduce(m0, FAdd(), redf) > P.top_p;
    }
    const unsigned long long target = __float2ull_rz(P.top_p * 1099511627776.0f);
    uint32_t pre = 0, msk = 0;
    unsigned long long above_fx = 0;  // mass of keys in higher digit groups
    for (int shift = 24; any && shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += kST) mass[i] = 0ull;
      __syncthreads();
      for (int i = j0; i < j1; i++) {
        const uint32_t key = __float_as_uint(ps_[pad(i)]);
        const bool in = (key & msk) == pre && ps_[pad(i)] > 0.f;
        const unsigned dig = in ? (key >> shift) & 255u : 256u;
        // p * 2^40 is exact in f32 (a power-of-two scale) and < 2^41
        unsigned long long fx = in ? __float2ull_rz(ps_[pad(i)] * 1099511627776.0f) : 0ull;
        const unsigned grp = __match_any_sync(__activemask(), dig);
        if (in) {
          // the group's sum in two exact 32-bit reductions (16 + 25 bits)
          const unsigned lo = __reduce_add_sync(grp, (unsigned)(fx & 0xFFFFu));
          const unsigned mid = __reduce_add_sync(grp, (unsigned)(fx >> 16));
          if ((__ffs(grp) - 1) == (int)(threadIdx.x & 31))
            atomicAdd(&mass[dig], ((unsigned long long)mid << 16) + lo);
        }
      }
      __syncthreads();
      if (tid < 32) {  // the highest digit d with above + mass(digits >= d) > target
        unsigned long long m8[8], tot = 0;
#pragma unroll
        for (int q = 0; q < 8; q++) m8[q] = mass[255 - (tid * 8 + q)], tot += m8[q];
        unsigned long long incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned long long y = __shfl_up_sync(0xffffffffu, incl, o);
          if (tid >= o) incl += y;
        }
        unsigned long long run = above_fx + incl - tot;
#pragma unroll
        for (int q = 0; q < 8; q++) {
          if (run <= target && run + m8[q] > target) {
            sel_digit = 255 - (tid * 8 + q);
            sel_mass = run;
          }
          run += m8[q];
        }
        if (tid == 31 && run <= target) sel_digit = -1;  // rounding: no digit crosses
      }
      __syncthreads();
      if (sel_digit < 0) {
        pre = 0, msk = 0;
        break;
      }
      pre |= (uint32_t)sel_digit << shift;
      msk |= 255u << shift;
      above_fx = sel_mass;
      __syncthreads();
    }
    const uint32_t lo = pre;
    const float tau = __uint_as_float(lo);
    float above = 0.f;
    int ties = 0;
    for (int i = j0; i < j1; i++) {
      if (ps_[pad(i)] > tau) above += ps_[pad(i)];
      ties += ps_[pad(i)] == tau;
    }
    above = block_reduce(above, FAdd(), redf);
    // ties needed: the smallest n with above + n * tau > top_p
    int need = 0;
    if (any && tau > 0.f) {
      float acc = above;
      while (acc <= P.top_p && need < V) acc += tau, need++;
    }
    const int before = block_exclusive_scan(ties, redi);
    float ps = 0.f;
    int seen = before;
    for (int i = j0; i < j1; i++) {
      bool keep = any && ps_[pad(i)] > tau;
      if (any && ps_[pad(i)] == tau) keep = seen++ < need;
      if (!keep) ps_[pad(i)] = 0.f;
      ps += ps_[pad(i)];
    }
    ps = block_reduce(ps, FAdd(), redf);
    if (ps > 0.f)
      for (int i = j0; i < j1; i++) ps_[pad(i)] = ps_[pad(i)] / ps;
  }

  if (P.temperature == 0.0f) {
    // greedy: the last index of the largest prob (Rust max_by keeps the last)
    unsigned long long best = 0;
    for (int i = j0; i < j1; i++) {
      const unsigned long long key = ((unsigned long long)__float_as_uint(ps_[pad(i)]) << 32) | (unsigned)i;
      best = best > key ? best : key;
    }
    best = block_reduce(best, ArgMaxLast(), redu);
    if (tid == 0) out[r] = (uint32_t)(best & 0xFFFFFFFFu);
    return;
  }
  // inverse CDF in index order (inference.rs:638-654)
  float cs = 0.f;
  for (int i = j0; i < j1; i++) cs += ps_[pad(i)];
  const float base = block_exclusive_scan(cs, redf);
  int hit = V;
  float run = base;
  for (int i = j0; i < j1; i++) {
    run += ps_[pad(i)];
    if (run > P.u) {
      hit = i;
      break;
    }
  }
  struct IMin {
    __device__ int operator()(int a, int b) const { return a < b ? a : b; }
  };
  hit = block_reduce(hit, IMin(), redi);
  if (tid == 0) out[r] = (uint32_t)(hit < V ? hit : V - 1);
}

}  // namespace

int launch_sample(const float* logits, int rows, int V, int ld, const wl_sample_params* prm,
                  uint32_t* out, cudaStream_t st) {
  if (rows <= 0 || V <= 0 || V > kSampleMaxVocab || ld < V)
    return fail(WL_ERR_INVALID_ARGUMENT,
                "sample: needs 0 < V <= " + std::to_string(kSampleMaxVocab) + " and ld >= V");
  const size_t smem = (size_t)(V + V / 32 + 1) * sizeof(float);
  if (first_use_on_device((const void*)k_sample))
    WL_CUDA_TRY(cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (kSampleMaxVocab + kSampleMaxVocab / 32 + 1) * (int)sizeof(float)));
  return launch_k(k_sample, dim3(rows), dim3(kST), smem, st, logits, V, ld, prm, out);
}

}  // namespace wl
