// Model runtime: GGUF -> HBM loader, paged-KV sessions, batched forward,
// CUDA-graph decode, tensor-parallel sharding with NCCL allreduce.
//
// Replaces LazyTransformer (woolly-core/src/model/lazy_transformer.rs):
//   from_gguf (:29-95)      -> wl_model_load_gguf: blocks uploaded unchanged
//                              (a TP shard copies its column/row byte slice)
//   process_layer (:98-258) -> run_rows(): RMSNorm -> fused QKV GEMV with
//                              paged-KV append -> flash-decoding attention ->
//                              o GEMV (+residual) -> RMSNorm -> gate/up GEMV
//                              with SiLU*up epilogue -> down GEMV (+residual)
//   forward (:1155-1336)    -> embedding gather, layers, final norm, LM head
//   OptimizedKVCache        -> per-session page tables over a device page pool
#include "model.h"

#include <dlfcn.h>

#include <algorithm>
#include <chrono>
#include <thread>
#include <cstdlib>
#include <cstring>
#include <string>

#include "common.h"

namespace wl {
namespace {

// ---- NCCL, resolved at run time so single-GPU use needs no NCCL ----
struct Nccl {
  bool ok = false;
  int (*GetUniqueId)(void*) = nullptr;
  int (*CommInitRank)(void**, int, /*ncclUniqueId by value*/ ...) = nullptr;
  int (*AllReduce)(const void*, void*, size_t, int, int, void*, cudaStream_t) = nullptr;
  int (*AllGather)(const void*, void*, size_t, int, void*, cudaStream_t) = nullptr;
  int (*CommDestroy)(void*) = nullptr;
  int (*CommAbort)(void*) = nullptr;
  const char* (*GetErrorString)(int) = nullptr;
};

Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    n.GetUniqueId = (int (*)(void*))dlsym(h, "ncclGetUniqueId");
    n.CommInitRank = (int (*)(void**, int, ...))dlsym(h, "ncclCommInitRank");
    n.AllReduce = (int (*)(const void*, void*, size_t, int, int, void*, cudaStream_t))dlsym(
        h, "ncclAllReduce");
    n.AllGather = (int (*)(const void*, void*, size_t, int, void*, cudaStream_t))dlsym(
        h, "ncclAllGather");
    n.CommDestroy = (int (*)(void*))dlsym(h, "ncclCommDestroy");
    n.CommAbort = (int (*)(void*))dlsym(h, "ncclCommAbort");
    n.GetErrorString = (const char* (*)(int))dlsym(h, "ncclGetErrorString");
    n.ok = n.GetUniqueId && n.CommInitRank && n.AllReduce && n.CommDestroy;
  });
  return n;
}

struct UniqueId {
  char internal[128];
};

int block_bytes(uint32_t t) { return t == WL_Q4_0 ? 18 : t == WL_Q4_1 ? 20 : t == WL_Q8_0 ? 34 : 0; }

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// One tensor's placement in the device weight buffer and how to fill it.
struct Piece {
  const uint8_t* src = nullptr;  // host bytes (mmap)
  size_t src_pitch = 0;          // bytes per source row
  size_t col_byte0 = 0;          // first byte of the slice within a row
  size_t row_bytes = 0;          // bytes copied per row
  size_t rows = 0;               // rows copied (starting at row0)
  size_t row0 = 0;
  size_t dst_pitch = 0;
  size_t dst_off = 0;
  size_t dst_bytes = 0;
};

int upload_pieces(uint8_t* dbase, const std::vector<Piece>& ps, cudaStream_t st) {
  // contiguous pieces go straight from the mapping; sliced ones are packed
  // row by row into a pinned staging buffer first.
  const size_t kStage = 64u << 20;
  uint8_t* stage = nullptr;
  WL_CUDA_TRY(cudaMallocHost(&stage, 2 * kStage));
  cudaEvent_t ev[2];
  cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming);
  cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming);
  int which = 0;
  bool used[2] = {false, false};
  int st_code = WL_OK;
  for (const Piece& p : ps) {
    bool contiguous = p.src_pitch == p.row_bytes && p.dst_pitch == p.row_bytes && p.col_byte0 == 0;
    if (contiguous) {
      const uint8_t* src = p.src + p.row0 * p.src_pitch;
      size_t total = p.rows * p.row_bytes;
      for (size_t off = 0; off < total; off += kStage) {
        size_t n = std::min(kStage, total - off);
        if (used[which]) cudaEventSynchronize(ev[which]);
        memcpy(stage + which * kStage, src + off, n);
        cudaError_t e = cudaMemcpyAsync(dbase + p.dst_off + off, stage + which * kStage, n,
                                        cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) {
          st_code = fail(WL_ERR_CUDA, std::string("weight upload: ") + cudaGetErrorString(e));
          break;
        }
        cudaEventRecord(ev[which], st);
        used[which] = true;
        which ^= 1;
      }
    } else {
      size_t rows_per = std::max<size_t>(1, kStage / p.dst_pitch);
      for (size_t r = 0; r < p.rows; r += rows_per) {
        size_t nr = std::min(rows_per, p.rows - r);
        if (used[which]) cudaEventSynchronize(ev[which]);
        uint8_t* s = stage + which * kStage;
        memset(s, 0, nr * p.dst_pitch);
        for (size_t i = 0; i < nr; i++)
          memcpy(s + i * p.dst_pitch, p.src + (p.row0 + r + i) * p.src_pitch + p.col_byte0,
                 p.row_bytes);
        cudaError_t e = cudaMemcpyAsync(dbase + p.dst_off + r * p.dst_pitch, s, nr * p.dst_pitch,
                                        cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) {
          st_code = fail(WL_ERR_CUDA, std::string("weight upload: ") + cudaGetErrorString(e));
          break;
        }
        cudaEventRecord(ev[which], st);
        used[which] = true;
        which ^= 1;
      }
    }
    if (st_code) break;
  }
  cudaStreamSynchronize(st);
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  cudaFreeHost(stage);
  return st_code;
}

struct Loader {
  GgufFile* g;
  wl_model* m;
  std::vector<Piece> pieces;
  size_t cursor = 0;
  std::string err;

  const GgufTensor* need(const std::string& name) {
    const GgufTensor* t = g->find(name);
    if (!t) err = "Tensor not found: " + name;
    return t;
  }
  // reserve a device region, 256-byte aligned, with 256 spare bytes
  size_t reserve(size_t bytes) {
    size_t off = cursor;
    cursor = align_up(cursor + bytes + 256, 256);
    return off;
  }
  // token_embd.weight: F32 is copied whole; any other type woolly_gguf::
  // dequantize reads (dequantize.rs:189-205) is staged and dequantized into an
  // f32 table on the device after the upload (embd_type != WL_F32)
  uint32_t embd_type = WL_F32;
  size_t embd_staged = 0, embd_n = 0;
  bool add_embd(const std::string& name, uint64_t expect, size_t* off) {
    const GgufTensor* t = need(name);
    if (!t) return false;
    if (t->type == WL_F32) return add_f32(name, expect, off);
    const uint32_t ty = t->type;
    const bool ok_type = ty == WL_F16 || ty == WL_Q4_0 || ty == WL_Q4_1 || ty == WL_Q8_0 || ty == 12 ||
                         ty == 14 || ty == 6 || ty == 7 || ty == 13 || ty == 15;
    if (!ok_type) {
      err = name + ": unsupported type " + std::to_string(ty);
      return false;
    }
    if (t->nelems() != expect) {
      err = name + ": unexpected element count " + std::to_string(t->nelems());
      return false;
    }
    const uint8_t* src = g->data(*t);
    if (!src) {
      err = name + ": data out of bounds";
      return false;
    }
    Piece p;
    p.src = src;
    p.src_pitch = p.row_bytes = p.dst_pitch = p.dst_bytes = t->nbytes();
    p.rows = 1;
    p.dst_off = embd_staged = tcursor;
    tcursor = align_up(tcursor + p.dst_bytes + 256, 256);
    tpieces.push_back(p);
    embd_type = ty;
    embd_n = expect;
    *off = reserve(expect * sizeof(float));
    return true;
  }
  // f32 vector / matrix copied whole
  bool add_f32(const std::string& name, uint64_t expect, size_t* off) {
    const GgufTensor* t = need(name);
    if (!t) return false;
    if (t->type != WL_F32) {
      err = name + ": expected F32, got type " + std::to_string(t->type);
      return false;
    }
    if (t->nelems() != expect) {
      err = name + ": unexpected element count " + std::to_string(t->nelems());
      return false;
    }
    const uint8_t* src = g->data(*t);
    if (!src) {
      err = name + ": data out of bounds";
      return false;
    }
    Piece p;
    p.src = src;
    p.src_pitch = p.row_bytes = p.dst_pitch = t->nbytes();
    p.rows = 1;
    p.dst_bytes = t->nbytes();
    p.dst_off = *off = reserve(p.dst_bytes);
    pieces.push_back(p);
    return true;
  }
  // layout-B matrix [K][N] (dims [K, N]); keeps rows [r0, r0+Kl) and
  // columns [c0, c0+Nl) (c0, Nl multiples of 32).
  // ggml orientation (m->ggml): the same dims [K, N] hold N rows of K values
  // (blocks run along K), copied whole (no tensor-parallel slicing).
  bool add_mat(const std::string& name, int K, int N, int r0, int Kl, int c0, int Nl, QMat* out,
               size_t* off) {
    if (m->ggml) return add_rows(name, K, N, out, off);
    return add_mat_b(name, K, N, r0, Kl, c0, Nl, out, off);
  }
  bool add_rows(const std::string& name, int K, int N, QMat* out, size_t* off) {
    const GgufTensor* t = need(name);
    if (!t) return false;
    if (t->n_dims != 2 || t->dims[0] != (uint64_t)K || t->dims[1] != (uint64_t)N) {
      err = name + ": expected dims [" + std::to_string(K) + ", " + std::to_string(N) + "]";
      return false;
    }
    const uint8_t* src = g->data(*t);
    if (!src) {
      err = name + ": data out of bounds";
      return false;
    }
    const bool kq = kquant_type((int)t->type);
    const int S = t->type == WL_F32 ? 0 : kq ? kquant_block_bytes((int)t->type) : block_bytes(t->type);
    if (t->type != WL_F32 && (!S || K % (kq ? 256 : 32))) {
      err = name + ": layout-A weights must be F32, Q4_0, Q4_1, Q8_0 (K % 32 == 0) or Q4_K, Q6_K (K % 256 == 0)";
      return false;
    }
    Piece p;
    p.src = src;
    p.rows = (size_t)N;
    p.src_pitch = p.row_bytes = t->type == WL_F32 ? (size_t)K * 4 : (size_t)K / (kq ? 256 : 32) * S;
    p.dst_pitch = p.row_bytes;
    p.dst_bytes = p.dst_pitch * p.rows;
    if (kq) {  // staged; the GEMV reads a copy with 16-byte aligned super-blocks
      p.dst_off = tcursor;
      tcursor = align_up(tcursor + p.dst_bytes + 256, 256);
      *off = p.dst_off | kStaged;
      tpieces.push_back(p);
    } else {
      p.dst_off = *off = reserve(p.dst_bytes);
      pieces.push_back(p);
    }
    out->type = t->type;
    out->K = K;
    out->N = N;
    out->pitch = (int)p.dst_pitch;
    return true;
  }
  bool add_mat_b(const std::string& name, int K, int N, int r0, int Kl, int c0, int Nl, QMat* out,
                 size_t* off) {
    const GgufTensor* t = need(name);
    if (!t) return false;
    if (t->n_dims != 2 || t->dims[0] != (uint64_t)K || t->dims[1] != (uint64_t)N) {
      err = name + ": expected dims [" + std::to_string(K) + ", " + std::to_string(N) + "]";
      return false;
    }
    const uint8_t* src = g->data(*t);
    if (!src) {
      err = name + ": data out of bounds";
      return false;
    }
    Piece p;
    p.src = src;
    p.rows = (size_t)Kl;
    p.row0 = (size_t)r0;
    if (t->type == WL_F32) {
      p.src_pitch = (size_t)N * 4;
      p.col_byte0 = (size_t)c0 * 4;
      p.row_bytes = (size_t)Nl * 4;
      p.dst_pitch = align_up(p.row_bytes, 16);
    } else {
      // K-quant super-blocks hold 256 columns of one row
      const bool kq = kquant_type((int)t->type);
      const int S = kq ? kquant_block_bytes((int)t->type) : block_bytes(t->type);
      const int BE = kq ? 256 : 32;
      if (!S) {
        err = name + ": weight type " + std::to_string(t->type) +
              " is not supported (F32, Q4_0, Q4_1, Q8_0, Q4_K, Q6_K)";
        return false;
      }
      if (N % BE || c0 % BE || Nl % BE) {
        err = name + ": quantized columns must be multiples of " + std::to_string(BE);
        return false;
      }
      if (kq && Kl % 16) {
        err = name + ": K-quant weights need a multiple of 16 rows";
        return false;
      }
      p.src_pitch = (size_t)N / BE * S;
      p.col_byte0 = (size_t)c0 / BE * S;
      p.row_bytes = (size_t)Nl / BE * S;
      p.dst_pitch = align_up(p.row_bytes, 16);
    }
    p.dst_bytes = p.dst_pitch * p.rows;
    // quantized projections that the runtime re-lays-out into its tiled copy
    // (which both the decode GEMV and the prefill GEMM read) are uploaded to a
    // staging buffer that is freed after the repack
    if (t->type != WL_F32 && Kl % 16 == 0 && Nl % 32 == 0) {
      p.dst_off = tcursor;
      tcursor = align_up(tcursor + p.dst_bytes + 256, 256);
      *off = p.dst_off | kStaged;
      tpieces.push_back(p);
    } else {
      p.dst_off = *off = reserve(p.dst_bytes);
      pieces.push_back(p);
    }
    out->type = t->type;
    out->K = Kl;
    out->N = Nl;
    out->pitch = (int)p.dst_pitch;
    return true;
  }
  static constexpr size_t kStaged = size_t(1) << 62;  // offset flag: in the staging buffer
  std::vector<Piece> tpieces;
  size_t tcursor = 0;
};

template <class T>
int dalloc(T** p, size_t n) {
  WL_CUDA_TRY(cudaMalloc((void**)p, std::max<size_t>(n, 1) * sizeof(T)));
  return WL_OK;
}

}  // namespace

int nccl_unique_id(void* out128) {
  Nccl& n = nccl();
  if (!n.ok) return fail(WL_ERR_NCCL, "NCCL library not available");
  int r = n.GetUniqueId(out128);
  if (r) return fail(WL_ERR_NCCL, std::string("ncclGetUniqueId: ") + n.GetErrorString(r));
  return WL_OK;
}

int nccl_comm_init(int nranks, const void* id128, int rank, void** comm) {
  Nccl& n = nccl();
  if (!n.ok) return fail(WL_ERR_NCCL, "NCCL library not available");
  UniqueId id;
  memcpy(id.internal, id128, 128);
  using Fn = int (*)(void**, int, UniqueId, int);
  int r = ((Fn)n.CommInitRank)(comm, nranks, id, rank);
  if (r) return fail(WL_ERR_NCCL, std::string("ncclCommInitRank: ") + n.GetErrorString(r));
  return WL_OK;
}

int nccl_comm_destroy(void* comm) {
  Nccl& n = nccl();
  if (!n.ok || !comm) return WL_OK;
  n.CommDestroy(comm);
  return WL_OK;
}

int nccl_comm_abort(void* comm) {
  Nccl& n = nccl();
  if (!n.ok || !comm || !n.CommAbort) return WL_OK;
  n.CommAbort(comm);
  return WL_OK;
}

// Waits for everything queued on the model's stream.  Under tensor
// parallelism a rank that stopped participating leaves the others' NCCL
// kernels waiting forever, so the wait is bounded by the collective timeout:
// on expiry the communicator is aborted (its kernels return), the model is
// marked unusable and WL_ERR_TIMEOUT is returned; close and reload it.
static int wait_for(wl_model* m, cudaEvent_t ev) {
  if (m->tp_size == 1) {
    WL_CUDA_TRY(cudaEventSynchronize(ev));
    return WL_OK;
  }
  const int ms = m->opt.collective_timeout_ms > 0 ? m->opt.collective_timeout_ms : 60000;
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) return WL_OK;
    if (q != cudaErrorNotReady) WL_CUDA_TRY(q);
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(ms)) break;
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  nccl_comm_abort(m->nccl);
  m->aborted = true;
  return fail(WL_ERR_TIMEOUT, "a tensor-parallel step did not finish within " + std::to_string(ms) +
                                  " ms (a rank stopped participating?): the NCCL communicator was "
                                  "aborted; close and reload the model");
}

static int sync_stream(wl_model* m) {
  WL_CUDA_TRY(cudaEventRecord(m->sync_ev, m->st));
  return wait_for(m, m->sync_ev);
}

static int check_alive(const wl_model* m) {
  if (m->aborted)
    return fail(WL_ERR_NCCL, "the tensor-parallel communicator was aborted after a timeout: close "
                             "and reload the model");
  return WL_OK;
}

static int allreduce_sum(wl_model* m, float* buf, size_t count) {
  Nccl& n = nccl();
  // ncclFloat32 = 7, ncclSum = 0
  int r = n.AllReduce(buf, buf, count, 7, 0, m->nccl, m->st);
  if (r) return fail(WL_ERR_NCCL, std::string("ncclAllReduce: ") + n.GetErrorString(r));
  return WL_OK;
}

// ------------------------------------------------------------------ GEMV dispatch
// Rows from which a projection runs as one tcgen05 GEMM instead of 32-row GEMVs.
constexpr int kGemmMinRows = 64;
// rows r in [0, R) of x (f16 hi/lo planes, lo plane x_plane elements after
// hi), up to 32 rows per launch.
// `ctas` (optional) receives the CTA count of the (single) GEMV launch.
static int gemv(wl_model* m, int nseg, const QMat* mats, int R, const __half* x, size_t x_plane,
                int ldx, Epilogue epi, unsigned* ctas = nullptr) {
  if (epi.kind == EPI_PEER && R > kPeerRows)
    return fail(WL_ERR_INVALID_ARGUMENT, "peer exchange: more rows than one GEMV launch");
  bool mixed = false;
  for (int s = 1; s < nseg; s++) mixed = mixed || mats[s].type != mats[0].type;
  if (mixed) {
    // a fused projection over weights of different types (the K-quant mixes
    // store attn_v as Q6_K beside Q4_K q and k) runs as one launch per
    // segment; the other segments keep their index with zero columns, so the
    // epilogue routes every output as in the fused launch
    if (epi.kind == EPI_SWIGLU || epi.kind == EPI_PEER)
      return fail(WL_ERR_UNSUPPORTED, "SwiGLU and peer GEMV segments must share a quantization type");
    for (int s = 0; s < nseg; s++) {
      QMat one[3];
      for (int j = 0; j < nseg; j++) {
        one[j] = mats[s];
        if (j != s) one[j].N = 0;
      }
      WL_TRY(gemv(m, nseg, one, R, x, x_plane, ldx, epi));
    }
    return WL_OK;
  }
  bool fast = block_bytes(mats[0].type) != 0 || kquant_type((int)mats[0].type);
  for (int s = 0; s < nseg && fast; s++)  // (zero-width segments: see the mixed-type split above)
    fast = mats[s].N == 0 || qgemv_b_fast_ok(mats[s].type, mats[s].K, mats[s].N, mats[s].pitch, mats[s].w);
  if (!fast && (nseg != 1 || !(epi.kind == EPI_F32 || epi.kind == EPI_ADD)))
    return fail(WL_ERR_UNSUPPORTED, "GEMV: unaligned or F32 weights only support plain outputs");
  const bool sw = epi.kind == EPI_SWIGLU;
  if (sw && (nseg != 2 || mats[0].N != mats[1].N))
    return fail(WL_ERR_INVALID_ARGUMENT, "SwiGLU GEMV needs gate and up of equal width");
  // prompts: every row in one tensor-core GEMM launch when the shape allows
  bool all_tiled = true;
  for (int s = 0; s < nseg; s++) all_tiled = all_tiled && mats[s].wt != nullptr;
  if (fast && all_tiled && R >= kGemmMinRows) {
    GemvArgs a;
    a.type = (int)mats[0].type;
    a.nseg = nseg;
    a.tiled = 1;
    for (int s = 0; s < nseg; s++) {
      a.seg[s].W = mats[s].wt;
      a.seg[s].N = mats[s].N;
      a.seg[s].pitch = mats[s].pitch;
    }
    a.K = mats[0].K;
    a.B = R;
    a.xkind = X_PLANES;
    a.x = x;
    a.x_plane = x_plane;
    a.ldx = ldx;
    a.epi = epi;
    a.err = m->err;
    if (qgemm_b_ok(a, R)) return launch_qgemm_b(a, R, m->st);
  }
  for (int r0 = 0; r0 < R; r0 += 32) {
    const int b = std::min(32, R - r0);
    Epilogue e = epi;
    for (int s = 0; s < 3; s++)
      if (e.y[s])
        e.y[s] = (uint8_t*)e.y[s] + (size_t)r0 * e.ldy[s] * (sw ? sizeof(__half) : sizeof(float));
    if (e.row_pos) e.row_pos += r0;
    if (e.row_sess) e.row_sess += r0;
    const __half* xr = x + (size_t)r0 * ldx;
    if (!fast) {
      WL_TRY(launch_qgemv_generic(mats[0].type, WL_LAYOUT_B, mats[0].w, mats[0].K, mats[0].N,
                                  mats[0].pitch, xr, x_plane, ldx, b, (float*)e.y[0], e.ldy[0],
                                  e.kind == EPI_ADD, m->st));
      continue;
    }
    GemvArgs a;
    a.type = (int)mats[0].type;
    a.nseg = nseg;
    bool tiled = true;
    for (int s = 0; s < nseg; s++) tiled = tiled && mats[s].wt != nullptr;
    a.tiled = tiled ? 1 : 0;
    int gb = 0;
    for (int s = 0; s < nseg; s++) {
      a.seg[s].W = tiled ? mats[s].wt : mats[s].w;
      a.seg[s].N = mats[s].N;
      a.seg[s].pitch = mats[s].pitch;
      a.seg[s].groups = (mats[s].N + 255) / 256;
      a.seg[s].group_base = gb;
      gb += a.seg[s].groups;
    }
    a.K = mats[0].K;
    a.B = b;
    a.xkind = X_PLANES;
    a.x = xr;
    a.x_plane = x_plane;
    a.ldx = ldx;
    a.epi = e;
    qgemv_plan(a, WL_LAYOUT_B, m->sms);
    if (ctas) {
      int groups = 0;
      for (int s = 0; s < nseg; s++) groups += a.seg[s].groups;
      *ctas = (unsigned)(groups * a.csplit);
    }
    WL_TRY(launch_qgemv_b(a, m->st));
  }
  return WL_OK;
}

// ---- NVLink peer exchange (tensor parallel decode) ----
static float* peer_slots(const wl_model* m, int rank, int par, int src) {
  return reinterpret_cast<float*>(m->pbase[rank] + 256) +
         (size_t)(par * m->tp_size + src) * kPeerRows * m->d;
}
static unsigned* peer_flags(const wl_model* m, int rank) {
  return reinterpret_cast<unsigned*>(m->pbase[rank]);
}

// Row-parallel GEMV epilogue of exchange `par`: push into slot (par, this
// rank) of every rank's buffer.
static Epilogue peer_push(const wl_model* m, int par) {
  Epilogue e;
  e.kind = EPI_PEER;
  e.ldy[0] = m->d;
  e.nranks = m->tp_size;
  for (int r = 0; r < m->tp_size; r++) {
    e.peer[r] = peer_slots(m, r, par, m->tp_rank);
    e.pflag[r] = peer_flags(m, r) + par * kMaxPeers + m->tp_rank;
  }
  return e;
}

static PeerReduce peer_take(const wl_model* m, int par, unsigned expect, int row0) {
  PeerReduce pr;
  pr.nranks = m->tp_size;
  pr.slots = peer_slots(m, m->tp_rank, par, 0);
  pr.flags = peer_flags(m, m->tp_rank) + par * kMaxPeers;
  pr.done = peer_flags(m, m->tp_rank) + 2 * kMaxPeers + par;
  pr.expect = expect;
  pr.row0 = row0;
  pr.err = m->err;
  return pr;
}

// One buffer per rank, mapped into every other rank through CUDA IPC (handles
// exchanged with one ncclAllGather).  Opt-in with WL_TP_PEER set at load: on
// 2 B200s the exchange measured slower than ncclAllReduce (70B shape: bs1 171
// vs 147 us per layer), so NCCL is the default.  Also left off for more than
// kMaxPeers ranks or when a row-parallel weight cannot take the fast GEMV.
static int peer_setup(wl_model* m) {
  const int T = m->tp_size, rk = m->tp_rank;
  if (T < 2 || T > kMaxPeers || !getenv("WL_TP_PEER")) return WL_OK;
  for (const Layer& y : m->layers)
    for (const QMat* q : {&y.wo, &y.wd})
      if (!block_bytes(q->type) || !qgemv_b_fast_ok(q->type, q->K, q->N, q->pitch, q->w)) return WL_OK;
  Nccl& n = nccl();
  if (!n.AllGather) return WL_OK;
  const size_t bytes = 256 + (size_t)2 * T * kPeerRows * m->d * sizeof(float);
  WL_CUDA_TRY(cudaMalloc(&m->pmem, bytes));
  WL_CUDA_TRY(cudaMemset(m->pmem, 0, bytes));
  cudaIpcMemHandle_t h;
  WL_CUDA_TRY(cudaIpcGetMemHandle(&h, m->pmem));
  uint8_t* dh = nullptr;
  WL_CUDA_TRY(cudaMalloc(&dh, (size_t)T * sizeof(h)));
  std::vector<cudaIpcMemHandle_t> all(T);
  cudaError_t ce = cudaMemcpy(dh + (size_t)rk * sizeof(h), &h, sizeof(h), cudaMemcpyHostToDevice);
  int nr = 0;
  if (ce == cudaSuccess) {
    nr = n.AllGather(dh + (size_t)rk * sizeof(h), dh, sizeof(h), /*ncclUint8*/ 1, m->nccl, m->st);
    if (!nr) ce = cudaStreamSynchronize(m->st);
    if (!nr && ce == cudaSuccess) ce = cudaMemcpy(all.data(), dh, (size_t)T * sizeof(h), cudaMemcpyDeviceToHost);
  }
  cudaFree(dh);
  if (nr) return fail(WL_ERR_NCCL, std::string("ncclAllGather: ") + n.GetErrorString(nr));
  WL_CUDA_TRY(ce);
  for (int r = 0; r < T; r++) {
    if (r == rk) {
      m->pbase[r] = m->pmem;
      continue;
    }
    void* p = nullptr;
    WL_CUDA_TRY(cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess));
    m->pbase[r] = static_cast<uint8_t*>(p);
  }
  m->peer = true;
  return WL_OK;
}

// Device error flags of the finished calls (the pinned mirror is copied at the
// end of each call): bit 1 token id out of range; 2, 4, 8, 16 a bounded wait
// (attention ring, cluster reduction, peer exchange, GEMM ring) gave up.
static int take_err(wl_model* m) {
  const int e = *m->h_err;
  if (!e) return WL_OK;
  *m->h_err = 0;
  // clear only the bits reported here: calls queued after the copy may have
  // set others, which the next read reports
  launch_err_clear(m->err, e, m->st);
  if (e & 1) return fail(WL_ERR_TOKEN_OUT_OF_RANGE, "token id exceeds vocabulary size (device check)");
  return fail(WL_ERR_TIMEOUT, "a bounded device wait gave up (flags " + std::to_string(e) +
                                  (e & 8 ? ": tensor-parallel peer exchange" : "") +
                                  "); results of that call are invalid");
}

// The whole forward for R rows whose ids/positions/sessions are on device.
// Logits are produced for rows [lfirst, R) into m->logits (row 0 = lfirst).
static int run_rows_body(wl_model* m, int R, int nsplit, int lfirst);

// The forward's kernels chain with programmatic dependent launch unless
// WL_NO_PDL is set in the environment.
static int run_rows(wl_model* m, int R, int nsplit, int lfirst) {
  static const bool pdl = getenv("WL_NO_PDL") == nullptr;
  set_pdl(pdl && (m->tp_size == 1 || (m->peer && R <= kPeerRows)));
  const int s = run_rows_body(m, R, nsplit, lfirst);
  set_pdl(false);
  return s;
}

// y[r][n] (+)= sum_k x[r][k] W[n][k] for a layout-A (ggml orientation) matrix,
// rows in launches of 32; f32 activations.
static int gemv_a(wl_model* m, const QMat& W, int R, const float* x, int ldx, float* y, int ldy,
                  bool add) {
  const bool fast = W.type != WL_F32 && qgemv_a_fast_ok(W.type, W.K, W.N, W.pitch, W.w);
  if (!fast)
    return launch_qgemv_generic(W.type, WL_LAYOUT_A, W.w, W.K, W.N, W.pitch, x, 0, ldx, R, y, ldy, add,
                                m->st);
  const int gcols = qgemv_group_cols(WL_LAYOUT_A);
  for (int r0 = 0; r0 < R; r0 += 32) {
    GemvArgs a;
    a.type = (int)W.type;
    a.nseg = 1;
    a.seg[0].W = W.w;
    a.seg[0].N = W.N;
    a.seg[0].pitch = W.pitch;
    a.seg[0].groups = (W.N + gcols - 1) / gcols;
    a.K = W.K;
    a.B = std::min(32, R - r0);
    a.xkind = X_F32;
    a.x = x + (size_t)r0 * ldx;
    a.ldx = ldx;
    a.epi.kind = add ? EPI_ADD : EPI_F32;
    a.epi.y[0] = y + (size_t)r0 * ldy;
    a.epi.ldy[0] = ldy;
    a.err = m->err;
    qgemv_plan(a, WL_LAYOUT_A, m->sms);
    WL_TRY(launch_qgemv_a(a, m->st));
  }
  return WL_OK;
}

// Prompt chunks of >= kPrefillMmaRows rows run attention on tensor cores;
// decode rows (one per session) and short chunks the flash-decoding kernel.
constexpr int kPrefillMmaRows = 16;
static int attention(const wl_model* m, const AttnArgs& a, cudaStream_t st) {
  if (m->prefill_chunk && a.rows >= kPrefillMmaRows && attention_prefill_ok(a.heads, a.kv_heads, a.head_dim))
    return launch_attention_prefill(a, st);
  return launch_attention_paged(a, st);
}

// The forward on weights in ggml orientation (llama.cpp checkpoints): the
// same layer as the reference's (lazy_transformer.rs:98-258) with its
// projections read as rows of K (quantized_matvec's layout,
// quantization.rs:1100-1163), the embedding as one row per token, and
// optional NeoX RoPE (embedding.rs:183-242) applied to q and k.
static int run_rows_a(wl_model* m, int R, int nsplit, int lfirst) {
  cudaStream_t st = m->st;
  const int d = m->d, qd = m->Hl * m->hd, kvd = m->kvdl, ff = m->ffl;
  WL_TRY(launch_embed(m->embd, d, m->V, m->ids, R, m->h, m->err, st, /*token_rows=*/1));
  for (int l = 0; l < m->L; l++) {
    const Layer& y = m->layers[l];
    WL_TRY(launch_rmsnorm(m->h, y.attn_norm, R, d, m->eps, 0, nullptr, 0, 0.f, m->xf, 0, 0, st));
    WL_TRY(gemv_a(m, y.wq, R, m->xf, d, m->q, qd, false));
    WL_TRY(gemv_a(m, y.wk, R, m->xf, d, m->kf, kvd, false));
    WL_TRY(gemv_a(m, y.wv, R, m->xf, d, m->vf, kvd, false));
    KvPages kv;
    const size_t layer_halves = (size_t)m->n_pages * m->page * m->kvdl;
    kv.k = reinterpret_cast<__half*>(m->kvbuf) + (size_t)l * 2 * layer_halves;
    kv.v = kv.k + layer_halves;
    kv.page_table = m->d_tables;
    kv.max_pages = m->max_pages;
    kv.page = m->page;
    kv.kv_heads = m->KVHl;
    kv.head_dim = m->hd;
    WL_TRY(launch_qkv_post(m->q, m->kf, m->vf, R, m->Hl, m->KVHl, m->hd, m->rope, m->theta,
                           m->row_pos, m->row_sess, kv, st));
    AttnArgs a;
    a.q = m->q;
    a.ldq = qd;
    a.kv = kv;
    a.row_pos = m->row_pos;
    a.row_sess = m->row_sess;
    a.rows = R;
    a.heads = m->Hl;
    a.kv_heads = m->KVHl;
    a.head_dim = m->hd;
    a.window = m->window;
    a.nsplit = nsplit;
    a.part_o = m->part_o;
    a.part_ml = m->part_ml;
    a.out = m->attf;
    a.ldo = qd;
    a.out_plane = 0;
    a.err = m->err;
    WL_TRY(attention(m, a, st));
    WL_TRY(gemv_a(m, y.wo, R, m->attf, qd, m->h, d, true));
    WL_TRY(launch_rmsnorm(m->h, y.ffn_norm, R, d, m->eps, 0, nullptr, 0, 0.f, m->xf, 0, 0, st));
    WL_TRY(gemv_a(m, y.wg, R, m->xf, d, m->gf, ff, false));
    WL_TRY(gemv_a(m, y.wu, R, m->xf, d, m->uf, ff, false));
    WL_TRY(launch_swiglu(m->gf, m->uf, (size_t)R * ff, m->gf, st));
    WL_TRY(gemv_a(m, y.wd, R, m->gf, ff, m->h, d, true));
  }
  const int nl = R - lfirst;
  if (nl > 0) {
    WL_TRY(launch_rmsnorm(m->h + (size_t)lfirst * d, m->out_norm, nl, d, m->eps, 0, nullptr, 0, 0.f,
                          m->xf, 0, 0, st));
    WL_TRY(gemv_a(m, m->out, nl, m->xf, d, m->logits, m->V, false));
  }
  return WL_OK;
}

static int run_rows_body(wl_model* m, int R, int nsplit, int lfirst) {
  if (m->ggml) return run_rows_a(m, R, nsplit, lfirst);
  cudaStream_t st = m->st;
  const bool tp = m->tp_size > 1;
  const int qd = m->Hl * m->hd;
  const size_t xpl = (size_t)m->MR * m->d;  // lo-plane offsets
  const size_t apl = (size_t)m->MR * qd;
  const size_t fpl = (size_t)m->MR * m->ffl;
  // tensor parallel decode: the row-parallel GEMVs push their partial sums to
  // every rank (exchange 0 after attn_output, 1 after ffn_down) and the next
  // RMSNorm completes h; prompts use ncclAllReduce
  const bool peer = tp && m->peer && R <= kPeerRows;
  unsigned ctas_o = 0, ctas_d = 0;
  WL_TRY(launch_embed(m->embd, m->d, m->V, m->ids, R, m->h, m->err, st));
  for (int l = 0; l < m->L; l++) {
    const Layer& y = m->layers[l];
    if (peer && l > 0)
      WL_TRY(launch_rmsnorm_peer(m->h, y.attn_norm, R, m->d, m->eps, m->xn, xpl,
                                 peer_take(m, 1, ctas_d, 0), st));
    else
      WL_TRY(launch_rmsnorm(m->h, y.attn_norm, R, m->d, m->eps, 0, nullptr, 0, 0.f, m->xn, 2, xpl, st));
    KvPages kv;
    const size_t layer_halves = (size_t)m->n_pages * m->page * m->kvdl;
    kv.k = reinterpret_cast<__half*>(m->kvbuf) + (size_t)l * 2 * layer_halves;
    kv.v = kv.k + layer_halves;
    kv.page_table = m->d_tables;
    kv.max_pages = m->max_pages;
    kv.page = m->page;
    kv.kv_heads = m->KVHl;
    kv.head_dim = m->hd;
    {
      Epilogue e;
      e.kind = EPI_QKV;
      e.y[0] = m->q;
      e.ldy[0] = qd;
      e.rope = m->rope;
      e.head_dim = m->hd;
      e.theta = m->theta;
      e.row_pos = m->row_pos;
      e.row_sess = m->row_sess;
      e.kv = kv;
      QMat segs[3] = {y.wq, y.wk, y.wv};
      WL_TRY(gemv(m, 3, segs, R, m->xn, xpl, m->d, e));
    }
    {
      AttnArgs a;
      a.q = m->q;
      a.ldq = qd;
      a.kv = kv;
      a.row_pos = m->row_pos;
      a.row_sess = m->row_sess;
      a.rows = R;
      a.heads = m->Hl;
      a.kv_heads = m->KVHl;
      a.head_dim = m->hd;
      a.window = m->window;
      a.nsplit = nsplit;
      a.part_o = m->part_o;
      a.part_ml = m->part_ml;
      a.out = m->att;
      a.ldo = qd;
      a.out_plane = apl;
      a.err = m->err;
      WL_TRY(attention(m, a, st));
    }
    if (peer) {
      WL_TRY(gemv(m, 1, &y.wo, R, m->att, apl, qd, peer_push(m, 0), &ctas_o));
      WL_TRY(launch_rmsnorm_peer(m->h, y.ffn_norm, R, m->d, m->eps, m->xn, xpl,
                                 peer_take(m, 0, ctas_o, 0), st));
    } else {
      Epilogue e;
      e.kind = (tp && m->tp_rank != 0) ? EPI_F32 : EPI_ADD;  // rank 0 carries the residual
      e.y[0] = m->h;
      e.ldy[0] = m->d;
      WL_TRY(gemv(m, 1, &y.wo, R, m->att, apl, qd, e));
      if (tp) WL_TRY(allreduce_sum(m, m->h, (size_t)R * m->d));
      WL_TRY(launch_rmsnorm(m->h, y.ffn_norm, R, m->d, m->eps, 0, nullptr, 0, 0.f, m->xn, 2, xpl, st));
    }
    {
      Epilogue e;
      e.kind = EPI_SWIGLU;
      e.y[0] = m->act;
      e.ldy[0] = m->ffl;
      e.y_plane = fpl;
      QMat segs[2] = {y.wg, y.wu};
      WL_TRY(gemv(m, 2, segs, R, m->xn, xpl, m->d, e));
    }
    if (peer) {
      WL_TRY(gemv(m, 1, &y.wd, R, m->act, fpl, m->ffl, peer_push(m, 1), &ctas_d));
    } else {
      Epilogue e;
      e.kind = (tp && m->tp_rank != 0) ? EPI_F32 : EPI_ADD;
      e.y[0] = m->h;
      e.ldy[0] = m->d;
      WL_TRY(gemv(m, 1, &y.wd, R, m->act, fpl, m->ffl, e));
      if (tp) WL_TRY(allreduce_sum(m, m->h, (size_t)R * m->d));
    }
  }
  const int nl = R - lfirst;
  if (peer)  // completes the logit rows (or, with none, only drains exchange 1)
    WL_TRY(launch_rmsnorm_peer(m->h + (size_t)lfirst * m->d, m->out_norm, nl, m->d, m->eps, m->xn,
                               xpl, peer_take(m, 1, ctas_d, lfirst), st));
  if (nl > 0) {
    if (!peer)
      WL_TRY(launch_rmsnorm(m->h + (size_t)lfirst * m->d, m->out_norm, nl, m->d, m->eps, 0, nullptr,
                            0, 0.f, m->xn, 2, xpl, st));
    Epilogue e;
    e.kind = EPI_F32;
    const bool vshard = m->Vl != m->V;
    e.y[0] = vshard ? m->logits_part : m->logits;
    e.ldy[0] = m->Vl;
    WL_TRY(gemv(m, 1, &m->out, nl, m->xn, xpl, m->d, e));
    if (vshard) {
      Nccl& n = nccl();
      const size_t cnt = (size_t)nl * m->Vl;
      // ncclFloat32 = 7; rank r's [nl][Vl] block lands at gather + r * cnt
      const int r = n.AllGather(m->logits_part, m->logits_gather, cnt, 7, m->nccl, st);
      if (r) return fail(WL_ERR_NCCL, std::string("ncclAllGather: ") + n.GetErrorString(r));
      WL_TRY(launch_gather_cols(m->logits_gather, m->tp_size, nl, m->Vl, m->logits, st));
    }
  }
  return WL_OK;
}

static int ensure_pages(wl_model* m, wl_session* s, int upto) {
  int need = (upto + m->page - 1) / m->page;
  if (need > m->max_pages)
    return fail(WL_ERR_CONTEXT_FULL, "session context full: " + std::to_string(upto) + " > " +
                                         std::to_string(m->max_pages * m->page) + " tokens");
  int first_new = (int)s->pages.size();
  while ((int)s->pages.size() < need) {
    if (m->free_pages.empty()) return fail(WL_ERR_OUT_OF_MEMORY, "KV page pool exhausted");
    int pg = m->free_pages.back();
    m->free_pages.pop_back();
    m->h_tables[(size_t)s->slot * m->max_pages + s->pages.size()] = pg;
    s->pages.push_back(pg);
  }
  if ((int)s->pages.size() > first_new) {
    size_t off = (size_t)s->slot * m->max_pages + first_new;
    WL_CUDA_TRY(cudaMemcpyAsync(m->d_tables + off, m->h_tables.data() + off,
                                (s->pages.size() - first_new) * sizeof(int),
                                cudaMemcpyHostToDevice, m->st));
  }
  return WL_OK;
}

static int upload_meta(wl_model* m, int R) {
  WL_CUDA_TRY(cudaMemcpyAsync(m->ids, m->h_meta, (size_t)R * 4, cudaMemcpyHostToDevice, m->st));
  WL_CUDA_TRY(cudaMemcpyAsync(m->row_pos, m->h_meta + m->MR, (size_t)R * 4,
                              cudaMemcpyHostToDevice, m->st));
  WL_CUDA_TRY(cudaMemcpyAsync(m->row_sess, m->h_meta + 2 * m->MR, (size_t)R * 4,
                              cudaMemcpyHostToDevice, m->st));
  return WL_OK;
}

// one batched decode step over B sessions whose metadata is already on device
static int decode_launch(wl_model* m, int B) {
  if (!m->opt.use_graphs) {
    int max_len = 0;
    for (int i = 0; i < B; i++) max_len = std::max(max_len, m->h_meta[m->MR + i] + 1);
    return run_rows(m, B, attention_plan_splits(B, m->KVHl, max_len, m->sms), 0);
  }
  const int nsplit = attention_plan_splits(B, m->KVHl, m->opt.max_context, m->sms);
  auto it = m->graphs.find(B);
  if (it == m->graphs.end()) {
    if (m->graph_warm[B]++ == 0) return run_rows(m, B, nsplit, 0);  // first call runs eagerly
    cudaGraph_t g;
    WL_CUDA_TRY(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
    int rs = run_rows(m, B, nsplit, 0);
    cudaError_t ce = cudaStreamEndCapture(m->st, &g);
    if (rs) return rs;
    if (ce != cudaSuccess) return fail(WL_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
    cudaGraphExec_t ex;
    cudaError_t ie = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) return fail(WL_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(ie));
    it = m->graphs.emplace(B, ex).first;
  }
  WL_CUDA_TRY(cudaGraphLaunch(it->second, m->st));
  return WL_OK;
}

static int check_sessions(wl_model* m, wl_session* const* ss, int n) {
  WL_CHECK_ARG(n >= 1, "n_sess must be >= 1");
  for (int i = 0; i < n; i++) {
    WL_CHECK_ARG(ss[i] && ss[i]->m == m, "session does not belong to this model");
    for (int j = 0; j < i; j++) WL_CHECK_ARG(ss[i] != ss[j], "a session appears twice in one call");
  }
  return WL_OK;
}

// ------------------------------------------------------------------ public (C++)
int model_load(wl_ctx* ctx, const char* path, const wl_model_options* o, wl_model** out) {
  *out = nullptr;
  WL_CHECK_ARG(ctx && path, "null argument");
  wl_model_options opt;
  wl_model_options_default(&opt);
  if (o) opt = *o;
  WL_CHECK_ARG(opt.max_sessions >= 1 && opt.max_context >= 1 && opt.max_batch >= 1 &&
                   opt.max_prefill >= 1,
               "model options: sizes must be >= 1");
  WL_CHECK_ARG(opt.tp_size >= 1 && opt.tp_rank >= 0 && opt.tp_rank < opt.tp_size,
               "model options: bad tensor-parallel rank/size");
  WL_CUDA_TRY(cudaSetDevice(ctx->device));
  GgufFile* g = nullptr;
  WL_TRY(gguf_open_file(path, &g));
  std::unique_ptr<GgufFile> gh(g);
  auto m = std::make_unique<wl_model>();
  m->ctx = ctx;
  m->dev = ctx->device;
  m->sms = ctx->num_sms;
  m->st = ctx->stream;
  m->opt = opt;
  m->tp_rank = opt.tp_rank;
  m->tp_size = opt.tp_size;
  m->ggml = opt.ggml_layout != 0;
  if (m->ggml && m->tp_size > 1)
    return fail(WL_ERR_UNSUPPORTED, "the ggml weight orientation is single-GPU only");
  m->nccl = opt.nccl_comm;
  if (m->tp_size > 1 && (!m->nccl || !nccl().ok))
    return fail(WL_ERR_NCCL, "tensor parallel load needs an NCCL communicator");
  // config, GGUFModelLoader::extract_config (model/loader.rs:104-156)
  std::string arch;
  if (!g->get_str("general.architecture", &arch))
    return fail(WL_ERR_INVALID_FORMAT, "No architecture specified in GGUF");
  wl_model_config& c = m->cfg;
  memset(&c, 0, sizeof(c));
  snprintf(c.architecture, sizeof(c.architecture), "%s", arch.c_str());
  uint32_t u;
  float f;
  c.vocab_size = g->get_u32(arch + ".vocab_size", &u) ? u : (g->get_u32("tokenizer.ggml.tokens.len", &u) ? u : 32000);
  c.hidden_size = g->get_u32(arch + ".embedding_length", &u) ? u : (g->get_u32(arch + ".embed_dim", &u) ? u : 4096);
  c.num_layers = g->get_u32(arch + ".block_count", &u) ? u : (g->get_u32(arch + ".layer_count", &u) ? u : 32);
  c.num_heads = g->get_u32(arch + ".attention.head_count", &u) ? u : 32;
  c.context_length = g->get_u32(arch + ".context_length", &u) ? u : (g->get_u32("tokenizer.ggml.context_length", &u) ? u : 2048);
  c.intermediate_size = g->get_u32(arch + ".feed_forward_length", &u) ? u : c.hidden_size * 4;
  c.num_kv_heads_meta = g->get_u32(arch + ".attention.head_count_kv", &u) ? u : 0;
  c.rope_theta = g->get_f32(arch + ".rope.freq_base", &f) ? f : (g->get_f32(arch + ".attention.rope_theta", &f) ? f : 0.f);
  c.layer_norm_epsilon = g->get_f32(arch + ".attention.layer_norm_epsilon", &f) ? f : (g->get_f32(arch + ".layer_norm_epsilon", &f) ? f : 1e-5f);
  m->d = (int)c.hidden_size;
  m->L = (int)c.num_layers;
  m->H = (int)c.num_heads;
  m->V = (int)c.vocab_size;
  m->eps = c.layer_norm_epsilon;
  m->theta = c.rope_theta > 0 ? c.rope_theta : 10000.f;
  m->rope = opt.rope_mode == WL_ROPE_NEOX;
  if (m->H <= 0 || m->d % m->H) return fail(WL_ERR_INVALID_FORMAT, "hidden size not divisible by heads");
  m->hd = m->d / m->H;
  // KV width from attn_k's shape (lazy_transformer.rs:284-287); FFN from ffn_gate (:496)
  const GgufTensor* tk = g->find("blk.0.attn_k.weight");
  const GgufTensor* tg = g->find("blk.0.ffn_gate.weight");
  if (!tk || !tg || tk->n_dims != 2 || tg->n_dims != 2)
    return fail(WL_ERR_TENSOR_NOT_FOUND, "Tensor not found: blk.0.attn_k.weight / ffn_gate.weight");
  m->kvd = (int)tk->dims[1];
  m->ff = (int)tg->dims[1];
  if (m->kvd % m->hd) return fail(WL_ERR_INVALID_FORMAT, "attn_k width not a multiple of head_dim");
  m->KVH = m->kvd / m->hd;
  if (m->H % m->KVH) return fail(WL_ERR_INVALID_FORMAT, "heads not divisible by kv heads");
  uint32_t sw = 0;
  if (opt.sliding_window > 0)
    m->window = opt.sliding_window;
  else if (opt.sliding_window == 0 && g->get_u32(arch + ".attention.sliding_window", &sw))
    m->window = (int)sw;
  // tensor-parallel shard sizes
  const int T = m->tp_size, rk = m->tp_rank;
  if (m->H % T || m->KVH % T || m->ff % (32 * T))
    return fail(WL_ERR_INVALID_ARGUMENT, "tp_size must divide heads, kv heads and ffn/32");
  m->Hl = m->H / T;
  m->KVHl = m->KVH / T;
  m->kvdl = m->KVHl * m->hd;
  m->ffl = m->ff / T;
  if ((m->hd % 32) || (m->Hl * m->hd) % 32 || m->kvdl % 32)
    return fail(WL_ERR_UNSUPPORTED, "head_dim must be a multiple of 32");
  if (m->hd != 64 && m->hd != 128 && m->hd != 256)
    return fail(WL_ERR_UNSUPPORTED, "head_dim must be 64, 128 or 256");

  // ---- plan the weight buffer ----
  Loader ld{g, m.get()};
  const int d = m->d, kvd = m->kvd, ff = m->ff, V = m->V;
  size_t off_embd, off_onorm, off_out;
  bool ok = ld.add_embd("token_embd.weight", (uint64_t)d * V, &off_embd) &&
            ld.add_f32("output_norm.weight", (uint64_t)d, &off_onorm);
  bool tied = ok && !g->find("output.weight");
  // LM head under tensor parallelism: each rank keeps V / T vocabulary
  // columns and the logit rows are gathered (ncclAllGather) after the head
  // GEMV; replicated when V does not split into whole 32-column blocks or
  // the head is the tied f32 embedding
  m->Vl = V;
  {
    const GgufTensor* ot = tied ? nullptr : g->find("output.weight");
    const int vb = ot && kquant_type((int)ot->type) ? 256 : 32;
    if (m->tp_size > 1 && !tied && V % (vb * m->tp_size) == 0 && nccl().AllGather) m->Vl = V / m->tp_size;
  }
  if (ok && !tied) ok = ld.add_mat("output.weight", d, V, 0, d, m->tp_rank * m->Vl, m->Vl, &m->out, &off_out);
  struct LOff {
    size_t an, fn, q, k, v, o, g, u, dn;
  };
  std::vector<LOff> lo(m->L);
  m->layers.resize(m->L);
  for (int l = 0; l < m->L && ok; l++) {
    std::string p = "blk." + std::to_string(l) + ".";
    Layer& y = m->layers[l];
    LOff& z = lo[l];
    const int qc = m->Hl * m->hd;
    ok = ld.add_f32(p + "attn_norm.weight", d, &z.an) && ld.add_f32(p + "ffn_norm.weight", d, &z.fn) &&
         ld.add_mat(p + "attn_q.weight", d, d, 0, d, rk * qc, qc, &y.wq, &z.q) &&
         ld.add_mat(p + "attn_k.weight", d, kvd, 0, d, rk * m->kvdl, m->kvdl, &y.wk, &z.k) &&
         ld.add_mat(p + "attn_v.weight", d, kvd, 0, d, rk * m->kvdl, m->kvdl, &y.wv, &z.v) &&
         ld.add_mat(p + "attn_output.weight", d, d, rk * qc, qc, 0, d, &y.wo, &z.o) &&
         ld.add_mat(p + "ffn_gate.weight", d, ff, 0, d, rk * m->ffl, m->ffl, &y.wg, &z.g) &&
         ld.add_mat(p + "ffn_up.weight", d, ff, 0, d, rk * m->ffl, m->ffl, &y.wu, &z.u) &&
         ld.add_mat(p + "ffn_down.weight", ff, d, rk * m->ffl, m->ffl, 0, d, &y.wd, &z.dn);
  }
  if (!ok) return fail(ld.err.rfind("Tensor not found", 0) == 0 ? WL_ERR_TENSOR_NOT_FOUND : WL_ERR_INVALID_FORMAT, ld.err);
  m->weight_bytes = ld.cursor;
  WL_CUDA_TRY(cudaMalloc(&m->dweights, m->weight_bytes));
  {
    int s = upload_pieces(m->dweights, ld.pieces, m->st);
    if (s) return s;
  }
  uint8_t* staged = nullptr;  // GGUF bytes of the re-laid-out projections, freed below
  if (ld.tcursor) {
    WL_CUDA_TRY(cudaMalloc(&staged, ld.tcursor));
    const int s = upload_pieces(staged, ld.tpieces, m->st);
    if (s) {
      cudaFree(staged);
      return s;
    }
  }
  struct StagedFree {
    uint8_t*& p;
    ~StagedFree() { cudaFree(p); }
  } staged_guard{staged};
  uint8_t* B0 = m->dweights;
  auto at = [&](size_t off) -> uint8_t* {
    return (off & Loader::kStaged) ? staged + (off & ~Loader::kStaged) : B0 + off;
  };
  uint8_t* B = m->dweights;
  m->embd = (const float*)(B + off_embd);
  if (ld.embd_type != WL_F32)
    WL_TRY(launch_dequant((int)ld.embd_type, staged + ld.embd_staged, ld.embd_n, (float*)(B + off_embd), m->st));
  m->out_norm = (const float*)(B + off_onorm);
  if (tied) {
    m->out.w = B + off_embd;
    m->out.type = WL_F32;
    m->out.K = d;
    m->out.N = V;
    m->out.pitch = m->ggml ? d * 4 : V * 4;  // ggml: one row of d per token
  } else {
    m->out.w = at(off_out);
  }
  for (int l = 0; l < m->L; l++) {
    Layer& y = m->layers[l];
    LOff& z = lo[l];
    y.attn_norm = (const float*)(B + z.an);
    y.ffn_norm = (const float*)(B + z.fn);
    y.wq.w = at(z.q);
    y.wk.w = at(z.k);
    y.wv.w = at(z.v);
    y.wo.w = at(z.o);
    y.wg.w = at(z.g);
    y.wu.w = at(z.u);
    y.wd.w = at(z.dn);
  }
  // ---- tiled decode copies (the GEMV's lane-ready layout) of every quantized projection;
  //      in the ggml orientation, K-quant rows with 16-byte aligned super-blocks ----
  {
    std::vector<QMat*> mats;
    for (Layer& y : m->layers)
      for (QMat* q : {&y.wq, &y.wk, &y.wv, &y.wo, &y.wg, &y.wu, &y.wd}) mats.push_back(q);
    mats.push_back(&m->out);
    size_t total = 0;
    std::vector<size_t> offs;
    for (QMat* q : mats) {
      size_t bytes = 0;
      if (m->ggml) {
        // layout A: q->K values per row, q->N rows (the loader's [K, N] dims)
        if (kquant_type((int)q->type)) bytes = (size_t)q->N * (q->K / 256) * kq_padded_bytes((int)q->type);
      } else if ((block_bytes(q->type) || kquant_type((int)q->type)) &&
                 qgemv_b_fast_ok(q->type, q->K, q->N, q->pitch, q->w)) {
        bytes = qtile_bytes((int)q->type, q->K, q->N);
      }
      offs.push_back(bytes ? total : SIZE_MAX);
      if (bytes) total = align_up(total + bytes, 256);
    }
    m->weight_bytes += total;
    if (total) {
      WL_CUDA_TRY(cudaMalloc(&m->dtiled, total));
      for (size_t i = 0; i < mats.size(); i++) {
        if (offs[i] == SIZE_MAX) continue;
        QMat* q = mats[i];
        if (m->ggml) {
          WL_TRY(launch_kq_pad((int)q->type, q->w, (size_t)q->pitch, q->N, q->K, m->dtiled + offs[i], m->st));
          q->w = m->dtiled + offs[i];
          q->pitch = q->K / 256 * kq_padded_bytes((int)q->type);
          q->wt = q->w;
        } else {
          WL_TRY(launch_repack_tiled((int)q->type, q->w, q->K, q->N, q->pitch, m->dtiled + offs[i], m->st));
          q->wt = m->dtiled + offs[i];
        }
      }
      WL_CUDA_TRY(cudaStreamSynchronize(m->st));
    }
    // every staged projection now lives only in its tiled copy
    for (QMat* q : mats)
      if (staged && q->w >= staged && q->w < staged + ld.tcursor) {
        if (!q->wt) return fail(WL_ERR_CUDA, "internal: a staged projection has no tiled copy");
        q->w = nullptr;
      }
    cudaFree(staged);
    staged = nullptr;
  }
  // ---- KV page pool ----
  m->max_sessions = opt.max_sessions;
  m->max_pages = (opt.max_context + m->page - 1) / m->page;
  m->n_pages = m->max_sessions * m->max_pages;
  m->kv_bytes = (size_t)m->L * 2 * m->n_pages * m->page * m->kvdl * sizeof(__half);
  WL_CUDA_TRY(cudaMalloc(&m->kvbuf, m->kv_bytes));
  WL_CUDA_TRY(cudaMemsetAsync(m->kvbuf, 0, m->kv_bytes, m->st));
  m->free_pages.resize(m->n_pages);
  for (int i = 0; i < m->n_pages; i++) m->free_pages[i] = m->n_pages - 1 - i;
  m->h_tables.assign((size_t)m->max_sessions * m->max_pages, 0);
  WL_TRY(dalloc(&m->d_tables, m->h_tables.size()));
  WL_CUDA_TRY(cudaMemsetAsync(m->d_tables, 0, m->h_tables.size() * sizeof(int), m->st));
  m->slots.assign(m->max_sessions, nullptr);
  // ---- scratch ----
  const int MR = m->MR = std::max(opt.max_batch, opt.max_prefill);
  WL_TRY(dalloc(&m->h, (size_t)MR * d));
  WL_TRY(dalloc(&m->xn, (size_t)2 * MR * d));
  WL_TRY(dalloc(&m->q, (size_t)MR * m->Hl * m->hd));
  if (m->ggml) {
    WL_TRY(dalloc(&m->xf, (size_t)MR * d));
    WL_TRY(dalloc(&m->kf, (size_t)MR * m->kvdl));
    WL_TRY(dalloc(&m->vf, (size_t)MR * m->kvdl));
    WL_TRY(dalloc(&m->attf, (size_t)MR * m->Hl * m->hd));
    WL_TRY(dalloc(&m->gf, (size_t)MR * m->ffl));
    WL_TRY(dalloc(&m->uf, (size_t)MR * m->ffl));
  }
  WL_TRY(dalloc(&m->att, (size_t)2 * MR * m->Hl * m->hd));
  WL_TRY(dalloc(&m->act, (size_t)2 * MR * m->ffl));
  WL_TRY(dalloc(&m->logits, (size_t)MR * V));
  if (m->Vl != V) {
    WL_TRY(dalloc(&m->logits_part, (size_t)MR * m->Vl));
    WL_TRY(dalloc(&m->logits_gather, (size_t)MR * V));
  }
  m->part_rows = (size_t)kAttnSplitCtasPerSm * m->sms + MR;
  WL_TRY(dalloc(&m->part_o, m->part_rows * m->Hl * m->hd));
  WL_TRY(dalloc(&m->part_ml, m->part_rows * m->Hl * 2));
  WL_TRY(dalloc(&m->row_pos, (size_t)MR));
  WL_TRY(dalloc(&m->row_sess, (size_t)MR));
  WL_TRY(dalloc(&m->ids, (size_t)MR));
  WL_TRY(dalloc(&m->err, 1));
  WL_CUDA_TRY(cudaMemsetAsync(m->err, 0, sizeof(int), m->st));
  WL_CUDA_TRY(cudaMallocHost(&m->h_meta, (size_t)3 * MR * sizeof(int)));
  WL_CUDA_TRY(cudaMallocHost(&m->h_ring, (size_t)wl_model::kMetaRing * 2 * MR * sizeof(int)));
  for (auto& e : m->ring_ev) WL_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  WL_CUDA_TRY(cudaMallocHost(&m->h_err, sizeof(int)));
  *m->h_err = 0;
  WL_CUDA_TRY(cudaEventCreateWithFlags(&m->err_ev, cudaEventDisableTiming));
  WL_CUDA_TRY(cudaEventCreateWithFlags(&m->sync_ev, cudaEventDisableTiming));
  WL_CUDA_TRY(cudaStreamSynchronize(m->st));
  WL_TRY(peer_setup(m.get()));
  *out = m.release();
  return WL_OK;
}

void model_free(wl_model* m) {
  if (!m) return;
  cudaSetDevice(m->dev);
  cudaStreamSynchronize(m->st);
  for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
  for (wl_session* s : m->slots)
    if (s) s->m = nullptr;
  cudaFree(m->dweights);
  cudaFree(m->dtiled);
  cudaFree(m->kvbuf);
  cudaFree(m->d_tables);
  cudaFree(m->h);
  cudaFree(m->xn);
  cudaFree(m->q);
  cudaFree(m->att);
  cudaFree(m->act);
  cudaFree(m->logits);
  for (float* f : {m->xf, m->kf, m->vf, m->attf, m->gf, m->uf}) cudaFree(f);
  cudaFree(m->logits_part);
  cudaFree(m->logits_gather);
  cudaFree(m->part_o);
  cudaFree(m->part_ml);
  cudaFree(m->row_pos);
  cudaFree(m->row_sess);
  cudaFree(m->ids);
  cudaFree(m->err);
  cudaFreeHost(m->h_meta);
  cudaFreeHost(m->h_ring);
  for (auto& e : m->ring_ev)
    if (e) cudaEventDestroy(e);
  cudaFreeHost(m->h_err);
  if (m->err_ev) cudaEventDestroy(m->err_ev);
  if (m->sync_ev) cudaEventDestroy(m->sync_ev);
  for (int r = 0; r < m->tp_size && r < kMaxPeers; r++)
    if (m->pbase[r] && m->pbase[r] != m->pmem) cudaIpcCloseMemHandle(m->pbase[r]);
  cudaFree(m->pmem);
  delete m;
}

int session_create(wl_model* m, wl_session** out) {
  *out = nullptr;
  WL_CHECK_ARG(m, "null model");
  std::lock_guard<std::mutex> lk(m->mu);
  for (int i = 0; i < m->max_sessions; i++)
    if (!m->slots[i]) {
      auto* s = new wl_session();
      s->m = m;
      s->slot = i;
      m->slots[i] = s;
      *out = s;
      return WL_OK;
    }
  return fail(WL_ERR_OUT_OF_MEMORY, "all " + std::to_string(m->max_sessions) + " session slots in use");
}

int session_reset(wl_session* s) {
  WL_CHECK_ARG(s, "null session");
  wl_model* m = s->m;
  if (m) {
    std::lock_guard<std::mutex> lk(m->mu);
    for (int pg : s->pages) m->free_pages.push_back(pg);
  }
  s->pages.clear();
  s->len = 0;
  return WL_OK;
}

void session_free(wl_session* s) {
  if (!s) return;
  session_reset(s);
  if (s->m) {
    std::lock_guard<std::mutex> lk(s->m->mu);
    s->m->slots[s->slot] = nullptr;
  }
  delete s;
}

int forward(wl_model* m, wl_session* const* ss, int n, const uint32_t* ids, const int* n_ids,
            float* logits, int mode) {
  WL_CHECK_ARG(m && ids && n_ids && logits, "null argument");
  WL_TRY(check_sessions(m, ss, n));
  WL_CHECK_ARG(mode == WL_LOGITS_LAST || mode == WL_LOGITS_ALL, "bad logits mode");
  WL_TRY(check_alive(m));
  std::lock_guard<std::mutex> lk(m->mu);
  WL_CUDA_TRY(cudaSetDevice(m->dev));
  size_t total = 0;
  bool all_one = true;
  for (int i = 0; i < n; i++) {
    WL_CHECK_ARG(n_ids[i] >= 1, "each session needs at least one token");
    all_one &= n_ids[i] == 1;
    total += (size_t)n_ids[i];
  }
  for (size_t i = 0; i < total; i++)
    if (ids[i] >= (uint32_t)m->V)
      return fail(WL_ERR_TOKEN_OUT_OF_RANGE, "Token ID " + std::to_string(ids[i]) +
                                                 " exceeds vocabulary size " + std::to_string(m->V));
  const size_t V = (size_t)m->V;
  if (all_one && n <= m->opt.max_batch) {
    for (int i = 0; i < n; i++) WL_TRY(ensure_pages(m, ss[i], ss[i]->len + 1));
    for (int i = 0; i < n; i++) {
      m->h_meta[i] = (int)ids[i];
      m->h_meta[m->MR + i] = ss[i]->len;
      m->h_meta[2 * m->MR + i] = ss[i]->slot;
    }
    WL_TRY(upload_meta(m, n));
    WL_TRY(decode_launch(m, n));
    WL_CUDA_TRY(cudaMemcpyAsync(logits, m->logits, (size_t)n * V * 4, cudaMemcpyDeviceToHost, m->st));
    WL_CUDA_TRY(cudaMemcpyAsync(m->h_err, m->err, sizeof(int), cudaMemcpyDeviceToHost, m->st));
    WL_TRY(sync_stream(m));
    for (int i = 0; i < n; i++) ss[i]->len += 1;
    return take_err(m);
  }
  // per-session prefill, chunked by max_prefill rows
  size_t id_off = 0, lg_off = 0;
  for (int i = 0; i < n; i++) {
    wl_session* s = ss[i];
    const int cnt = n_ids[i];
    for (int c0 = 0; c0 < cnt; c0 += m->opt.max_prefill) {
      const int c = std::min(m->opt.max_prefill, cnt - c0);
      WL_TRY(ensure_pages(m, s, s->len + c));
      for (int r = 0; r < c; r++) {
        m->h_meta[r] = (int)ids[id_off + c0 + r];
        m->h_meta[m->MR + r] = s->len + r;
        m->h_meta[2 * m->MR + r] = s->slot;
      }
      WL_TRY(upload_meta(m, c));
      const bool last_chunk = c0 + c == cnt;
      int lfirst = mode == WL_LOGITS_ALL ? 0 : (last_chunk ? c - 1 : c);
      const int nsplit = attention_plan_splits(c, m->KVHl, s->len + c, m->sms);
      m->prefill_chunk = true;
      const int rs = run_rows(m, c, nsplit, lfirst);
      m->prefill_chunk = false;
      WL_TRY(rs);
      if (c - lfirst > 0) {
        WL_CUDA_TRY(cudaMemcpyAsync(logits + lg_off, m->logits, (size_t)(c - lfirst) * V * 4,
                                    cudaMemcpyDeviceToHost, m->st));
        lg_off += (size_t)(c - lfirst) * V;
      }
      WL_CUDA_TRY(cudaMemcpyAsync(m->h_err, m->err, sizeof(int), cudaMemcpyDeviceToHost, m->st));
      WL_TRY(sync_stream(m));
      s->len += c;
      WL_TRY(take_err(m));
    }
    id_off += (size_t)cnt;
  }
  return WL_OK;
}

int decode_step_device(wl_model* m, wl_session* const* ss, int n, const uint32_t* d_ids,
                       float* d_logits, cudaStream_t user) {
  WL_CHECK_ARG(m && d_ids && d_logits, "null argument");
  WL_TRY(check_sessions(m, ss, n));
  WL_CHECK_ARG(n <= m->opt.max_batch, "n_sess exceeds max_batch");
  WL_TRY(check_alive(m));
  std::lock_guard<std::mutex> lk(m->mu);
  WL_CUDA_TRY(cudaSetDevice(m->dev));
  // asynchronous API: device errors of earlier calls surface here, once the
  // copy into the pinned mirror that the previous call queued has completed
  if (m->err_pending && cudaEventQuery(m->err_ev) == cudaSuccess) {
    m->err_pending = false;
    WL_TRY(take_err(m));
  }
  // order after the caller's work (0 = the legacy default stream); the guard
  // also orders the caller's stream after this step on every return path
  struct StreamJoin {
    cudaStream_t user, own;
    cudaEvent_t ev = nullptr;
    ~StreamJoin() {
      if (!ev) return;
      cudaEventRecord(ev, own);
      cudaStreamWaitEvent(user, ev, 0);
      cudaEventDestroy(ev);
    }
  } join{user, m->st};
  if (user != m->st) {
    WL_CUDA_TRY(cudaEventCreateWithFlags(&join.ev, cudaEventDisableTiming));
    WL_CUDA_TRY(cudaEventRecord(join.ev, user));
    WL_CUDA_TRY(cudaStreamWaitEvent(m->st, join.ev, 0));
  }
  for (int i = 0; i < n; i++) WL_TRY(ensure_pages(m, ss[i], ss[i]->len + 1));
  // per-step positions go through a ring slot the previous user of which has
  // been copied: this call returns before its copies run
  const int k = (int)(m->ring_next++ % wl_model::kMetaRing);
  if (m->ring_used[k]) WL_TRY(wait_for(m, m->ring_ev[k]));
  int* meta = m->h_ring + (size_t)k * 2 * m->MR;
  for (int i = 0; i < n; i++) {
    meta[i] = ss[i]->len;
    meta[m->MR + i] = ss[i]->slot;
    m->h_meta[m->MR + i] = ss[i]->len;  // host copy read by the eager (graph-less) launch
  }
  WL_CUDA_TRY(cudaMemcpyAsync(m->ids, d_ids, (size_t)n * 4, cudaMemcpyDeviceToDevice, m->st));
  WL_CUDA_TRY(cudaMemcpyAsync(m->row_pos, meta, (size_t)n * 4, cudaMemcpyHostToDevice, m->st));
  WL_CUDA_TRY(cudaMemcpyAsync(m->row_sess, meta + m->MR, (size_t)n * 4, cudaMemcpyHostToDevice, m->st));
  WL_CUDA_TRY(cudaEventRecord(m->ring_ev[k], m->st));
  m->ring_used[k] = true;
  WL_TRY(decode_launch(m, n));
  WL_CUDA_TRY(cudaMemcpyAsync(d_logits, m->logits, (size_t)n * m->V * 4, cudaMemcpyDeviceToDevice, m->st));
  if (!m->err_pending) {  // one copy in flight at a time: the host reads h_err only after it
    WL_CUDA_TRY(cudaMemcpyAsync(m->h_err, m->err, sizeof(int), cudaMemcpyDeviceToHost, m->st));
    WL_CUDA_TRY(cudaEventRecord(m->err_ev, m->st));
    m->err_pending = true;
  }
  for (int i = 0; i < n; i++) ss[i]->len += 1;
  return WL_OK;
}

// kernels per decode step: embed + L*(norm, qkv, attn[, combine], o, norm, gateup, down) + norm + head
int decode_kernel_count(const wl_model* m, int n) {
  const int nsplit = attention_plan_splits(n, m->KVHl, m->opt.max_context, m->sms);
  int chunks = (n + 31) / 32;
  int total = 1 + 1 + chunks + (m->Vl != m->V ? 1 : 0);
  for (const Layer& y : m->layers) {
    // q/k/v of different types (K-quant mixes) take one launch each
    const bool mixed = y.wq.type != y.wk.type || y.wq.type != y.wv.type;
    total += 2 + chunks * (3 + (mixed ? 3 : 1)) + 1 + (nsplit > 1 ? 1 : 0);
  }
  return total;
}

}  // namespace wl
