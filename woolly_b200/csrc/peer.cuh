// Tensor-parallel exchange over NVLink peer memory: the row-parallel GEMV
// pushes each rank's partial sums into every rank's receive slots (EPI_PEER),
// the following RMSNorm waits for all of them and completes the rows.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace wl {

constexpr int kMaxPeers = 8;   // ranks of one tensor-parallel group
constexpr int kPeerRows = 32;  // rows per exchange (one decode GEMV launch)
constexpr int kPeerSpin = 1 << 21;  // polls (with ~128 ns sleeps) before a wait gives up

// Consumer side of one exchange, all pointers in this rank's own buffer.
struct PeerReduce {
  int nranks = 0;                 // 0: no exchange
  const float* slots = nullptr;   // [nranks][kPeerRows][dim] partial rows from each rank
  unsigned* flags = nullptr;      // [nranks] arrived CTAs of each rank's GEMV
  unsigned* done = nullptr;       // consumer CTAs past the wait; the last one re-arms flags
  unsigned expect = 0;            // CTAs of each rank's GEMV launch
  int row0 = 0;                   // slot row of this launch's first row
  int* err = nullptr;             // bit 8 set when the wait gave up
};

#ifdef __CUDACC__
// Bounded wait until every rank's GEMV CTAs have signalled (acquire, system
// scope); then the CTA may read the slots.
__device__ __forceinline__ void peer_wait(const PeerReduce& pr) {
  if ((int)threadIdx.x < pr.nranks) {
    const unsigned* f = pr.flags + threadIdx.x;
    bool ok = false;
    for (int it = 0; it < kPeerSpin; it++) {
      unsigned v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(f) : "memory");
      if (v >= pr.expect) {
        ok = true;
        break;
      }
      __nanosleep(128);
    }
    if (!ok && pr.err) atomicOr(pr.err, 8);
  }
  __syncthreads();
}

// After the last consumer CTA has read the slots, take this exchange's
// arrivals off the counters so that the next use of the buffer starts at 0.
// No rank can signal that next use before this rank has passed its own next
// exchange, which follows this kernel in stream order.
__device__ __forceinline__ void peer_release(const PeerReduce& pr) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned old = atomicAdd(pr.done, 1u);
    if (old == gridDim.x - 1) {
      // take off at most `expect`: after a wait that gave up, a counter that
      // never reached it returns to 0 instead of wrapping around (which would
      // let the next exchange pass its wait on stale slots)
      for (int s = 0; s < pr.nranks; s++) {
        unsigned* f = pr.flags + s;
        unsigned v = *(volatile unsigned*)f;
        for (int it = 0; it < 64; it++) {
          const unsigned w = atomicCAS(f, v, v - min(v, pr.expect));
          if (w == v) break;
          v = w;
        }
      }
      atomicExch(pr.done, 0u);
    }
  }
}
#endif

}  // namespace wl
