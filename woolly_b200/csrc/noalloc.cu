// wl_qgemv_noalloc: the layout-B quantized GEMV for callers that cannot
// allocate device memory.
//
// wl_qgemv splits its f32 activations into f16 hi/lo planes in a temporary it
// allocates on the stream.  Some callers cannot allow that: serving processes
// that reserve all device memory up front and treat any later allocation as a
// failure, code that runs where an allocation could block or synchronise the
// device (inside tight decode loops with fixed memory budgets), or hosts whose
// allocator is owned by another framework.  This variant keeps the planes in a
// fixed device array that lives in the library instead.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "common.h"
#include "qgemv.cuh"

namespace wl {
namespace {

// Largest B*K the entry point accepts (each of the two f16 planes holds this
// many elements): 2 MiB of device memory per GPU that loads the library.
constexpr size_t kNoAllocMaxElems = size_t(1) << 19;

// The activation planes: [2][kNoAllocMaxElems] halves, hi plane then lo plane.
// Host code must not pass `g_noalloc_planes` itself to a kernel (on the host
// the name is only a stand-in); it uses the device address looked up below.
static __device__ __align__(256) __half g_noalloc_planes[2 * kNoAllocMaxElems];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
__half* g_addr[kMaxDevices] = {};

// Device address of the planes on the current device, looked up once per
// device (with that device current).
int planes_on_current_device(__half** out) {
  int dev = 0;
  WL_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(WL_ERR_INVALID_ARGUMENT, "device index too large");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_planes);
    if (e != cudaSuccess || !p)
      return fail(WL_ERR_CUDA, std::string("cudaGetSymbolAddress(noalloc planes): ") +
                                   cudaGetErrorString(e));
    g_addr[dev] = static_cast<__half*>(p);
  }
  *out = g_addr[dev];
  return WL_OK;
}

}  // namespace

// Set-up of the current device (wl_init calls it, so that the device code that
// holds the array is loaded while the caller still budgets memory).
int noalloc_setup_current_device() {
  __half* p = nullptr;
  return planes_on_current_device(&p);
}

namespace {

int block_bytes(int t) { return t == WL_Q4_0 ? 18 : t == WL_Q4_1 ? 20 : t == WL_Q8_0 ? 34 : 0; }

}  // namespace
}  // namespace wl

using namespace wl;

extern "C" int wl_qgemv_noalloc(int type, const void* W, int K, int N, const float* x, int B,
                                float* y, void* stream) {
  if (!W || !x || !y || K <= 0 || N <= 0 || B <= 0)
    return fail(WL_ERR_INVALID_ARGUMENT, "qgemv_noalloc: bad argument");
  const int S = block_bytes(type);
  if (!S) return fail(WL_ERR_UNSUPPORTED, "qgemv_noalloc: type must be Q4_0, Q4_1 or Q8_0");
  const size_t n = (size_t)B * K;
  if (n > kNoAllocMaxElems)
    return fail(WL_ERR_INVALID_ARGUMENT,
                "qgemv_noalloc: B*K = " + std::to_string(n) + " exceeds the fixed maximum of " +
                    std::to_string(kNoAllocMaxElems) + " elements");
  const int pitch = N / 32 * S;
  if (N % 32 || !qgemv_b_fast_ok(type, K, N, pitch, W))
    return fail(WL_ERR_INVALID_ARGUMENT,
                "qgemv_noalloc: needs N % 32 == 0, K % 16 == 0 and 16-byte aligned rows");
  __half* planes = nullptr;
  WL_TRY(planes_on_current_device(&planes));
  cudaStream_t st = (cudaStream_t)stream;
  // every element the GEMV reads (B*K per plane) is written here first
  WL_TRY(launch_split_planes(x, planes, n, kNoAllocMaxElems, st));
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  GemvArgs a;
  a.type = type;
  a.nseg = 1;
  a.seg[0].W = (const uint8_t*)W;
  a.seg[0].N = N;
  a.seg[0].pitch = pitch;
  a.seg[0].groups = (N + 255) / 256;
  a.K = K;
  a.ldx = K;
  a.xkind = X_PLANES;
  a.x_plane = kNoAllocMaxElems;
  a.epi.kind = EPI_F32;
  a.epi.ldy[0] = N;
  for (int r0 = 0; r0 < B; r0 += 32) {
    a.B = std::min(32, B - r0);
    a.x = planes + (size_t)r0 * K;
    a.epi.y[0] = y + (size_t)r0 * N;
    qgemv_plan(a, WL_LAYOUT_B, sms);
    WL_TRY(launch_qgemv_b(a, st));
  }
  return WL_OK;
}
