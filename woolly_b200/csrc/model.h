// Model runtime internals: weights in HBM, paged KV sessions, scratch, graphs.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/woolly_cuda.h"
#include "gguf.h"
#include "kernels.cuh"
#include "qgemv.cuh"

struct wl_ctx {
  int device = 0;
  int num_sms = 0;
  cudaStream_t stream = nullptr;
};

namespace wl {

// A layout-B weight matrix [K][N] as GGUF blocks in HBM.
struct QMat {
  const uint8_t* w = nullptr;
  uint32_t type = 0;
  int K = 0, N = 0;
  int pitch = 0;  // bytes per row
  const uint8_t* wt = nullptr;  // tiled decode copy (qtile_bytes), when the type has one
};

struct Layer {
  const float* attn_norm = nullptr;
  const float* ffn_norm = nullptr;
  QMat wq, wk, wv, wo, wg, wu, wd;
};

}  // namespace wl

struct wl_session;

struct wl_model {
  wl_ctx* ctx = nullptr;
  int dev = 0, sms = 0;
  cudaStream_t st = nullptr;
  wl_model_options opt{};
  wl_model_config cfg{};
  // shapes (per shard under tensor parallelism)
  int d = 0, L = 0, H = 0, KVH = 0, hd = 0, kvd = 0, ff = 0, V = 0;
  int Hl = 0, KVHl = 0, kvdl = 0, ffl = 0;  // local heads / kv width / ffn width
  float eps = 1e-5f, theta = 10000.f;
  int window = 0, rope = 0;
  // weights
  uint8_t* dweights = nullptr;
  uint8_t* dtiled = nullptr;  // tiled decode copies of the quantized projections
  size_t weight_bytes = 0;
  const float* embd = nullptr;  // [d][V] f32
  const float* out_norm = nullptr;
  wl::QMat out;                 // [d][V] (a tied embedding is an F32 QMat)
  std::vector<wl::Layer> layers;
  // paged KV
  int page = 16, n_pages = 0, max_pages = 0, max_sessions = 0;
  uint8_t* kvbuf = nullptr;
  size_t kv_bytes = 0;
  std::vector<int> free_pages;
  int* d_tables = nullptr;          // [max_sessions][max_pages]
  std::vector<int> h_tables;
  std::vector<wl_session*> slots;
  // scratch (rows = max(max_batch, max_prefill))
  int MR = 0;
  float* h = nullptr;       // residual stream [MR][d]
  __half* xn = nullptr;     // normalised rows as f16 hi/lo planes [2][MR][d]
  float* q = nullptr;       // queries [MR][Hl*hd]
  __half* att = nullptr;    // attention output planes [2][MR][Hl*hd]
  __half* act = nullptr;    // SwiGLU output planes [2][MR][ffl]
  float* logits = nullptr;  // [MR][V]
  // ggml orientation (llama.cpp files): f32 rows between the layout-A GEMVs
  bool ggml = false;
  // set while run_rows processes one session's prompt chunk (consecutive
  // positions): attention then takes the tensor-core prefill kernel
  bool prefill_chunk = false;
  float *xf = nullptr, *kf = nullptr, *vf = nullptr, *attf = nullptr, *gf = nullptr, *uf = nullptr;
  int Vl = 0;                       // vocabulary columns of this rank's LM head (V unless sharded)
  float* logits_part = nullptr;     // [MR][Vl] this rank's logit columns (sharded head)
  float* logits_gather = nullptr;   // [T][MR][Vl] all ranks' columns after the all-gather
  float* part_o = nullptr;  // attention split partials
  float* part_ml = nullptr;
  size_t part_rows = 0;     // capacity in rows*nsplit
  int* row_pos = nullptr;
  int* row_sess = nullptr;
  uint32_t* ids = nullptr;
  int* err = nullptr;
  // pinned staging for per-step metadata
  int* h_meta = nullptr;  // [3][MR]: ids, pos, sess (synchronous calls)
  // asynchronous decode steps: a ring of pinned [2][MR] (pos, sess) slots; a
  // slot is rewritten only after the event recorded behind its copies has
  // completed, so a host that runs ahead never changes a copy still queued
  static constexpr int kMetaRing = 8;
  int* h_ring = nullptr;
  cudaEvent_t ring_ev[kMetaRing] = {};
  bool ring_used[kMetaRing] = {};
  unsigned ring_next = 0;
  // decode graphs keyed by batch size
  std::map<int, cudaGraphExec_t> graphs;
  std::map<int, int> graph_warm;
  // tensor parallel
  int tp_rank = 0, tp_size = 1;
  void* nccl = nullptr;
  // NVLink peer exchange for decode batches (<= kPeerRows rows): every rank's
  // buffer (own: pmem; peers: CUDA IPC mappings) holds [flags 2x8 u32][done 2
  // u32] at byte 0 and slots [2][tp_size][kPeerRows][d] f32 at byte 256
  bool peer = false;
  uint8_t* pmem = nullptr;
  uint8_t* pbase[wl::kMaxPeers] = {};
  int* h_err = nullptr;  // pinned mirror of err, copied after every call
  cudaEvent_t err_ev = nullptr;  // recorded after the asynchronous step's copy into h_err
  bool err_pending = false;      // err_ev recorded and not yet consumed
  cudaEvent_t sync_ev = nullptr;  // end of a synchronous call's work (bounded wait under TP)
  bool aborted = false;           // the NCCL communicator was aborted after a timeout
  std::mutex mu;
};

struct wl_session {
  wl_model* m = nullptr;
  int slot = -1;
  int len = 0;
  std::vector<int> pages;
};
