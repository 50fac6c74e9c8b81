// extern "C" boundary (include/woolly_cuda.h).  Argument checks mirror the
// reference's error behaviour; device work is stream-ordered.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <set>
#include <string>

#include "common.h"
#include "gguf.h"
#include "kernels.cuh"
#include "model.h"
#include "qgemv.cuh"

namespace wl {

thread_local std::string g_err;
void set_error(const std::string& m) { g_err = m; }
thread_local bool g_pdl = false;

bool first_use_on_device(const void* key) {
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> seen;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  return seen.insert({dev, key}).second;
}
bool pdl_enabled() { return g_pdl; }
void set_pdl(bool on) { g_pdl = on; }

int model_load(wl_ctx*, const char*, const wl_model_options*, wl_model**);
void model_free(wl_model*);
int session_create(wl_model*, wl_session**);
int session_reset(wl_session*);
void session_free(wl_session*);
int forward(wl_model*, wl_session* const*, int, const uint32_t*, const int*, float*, int);
int decode_step_device(wl_model*, wl_session* const*, int, const uint32_t*, float*, cudaStream_t);
int decode_kernel_count(const wl_model*, int);
int noalloc_setup_current_device();
int nccl_unique_id(void*);
int nccl_comm_init(int, const void*, int, void**);
int nccl_comm_destroy(void*);
int nccl_comm_abort(void*);

namespace {

int bb(int t) { return t == WL_Q4_0 ? 18 : t == WL_Q4_1 ? 20 : t == WL_Q8_0 ? 34 : 0; }

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// y[b][n] = sum_k x[b][k] W(k, n) through the tensor-core GEMV, rows in chunks of 32.
// Layout B takes its activations as f16 hi/lo planes, made here in a
// stream-ordered temporary.
int qgemv_op(int type, int layout, const uint8_t* W, int K, int N, const float* x, int B, float* y,
             cudaStream_t st) {
  const int S = bb(type);
  const int pitch = layout == WL_LAYOUT_B ? N / 32 * S : K / 32 * S;
  const bool fast = layout == WL_LAYOUT_B ? qgemv_b_fast_ok(type, K, N, pitch, W)
                                          : qgemv_a_fast_ok(type, K, N, pitch, W);
  if (!fast) return launch_qgemv_generic(type, layout, W, K, N, pitch, x, 0, K, B, y, N, false, st);
  __half* planes = nullptr;
  const size_t n = (size_t)B * K;
  if (layout == WL_LAYOUT_B) {
    WL_CUDA_TRY(cudaMallocAsync((void**)&planes, 2 * n * sizeof(__half), st));
    const int s = launch_split_planes(x, planes, n, n, st);
    if (s) {
      cudaFreeAsync(planes, st);
      return s;
    }
  }
  const int gcols = qgemv_group_cols(layout);
  GemvArgs a;
  a.type = type;
  a.nseg = 1;
  a.seg[0].W = W;
  a.seg[0].N = N;
  a.seg[0].pitch = pitch;
  a.seg[0].groups = (N + gcols - 1) / gcols;
  a.K = K;
  a.ldx = K;
  a.xkind = layout == WL_LAYOUT_B ? X_PLANES : X_F32;
  a.x_plane = n;
  a.epi.kind = EPI_F32;
  a.epi.ldy[0] = N;
  int s = WL_OK;
  for (int r0 = 0; r0 < B && s == WL_OK; r0 += 32) {
    a.B = std::min(32, B - r0);
    a.x = layout == WL_LAYOUT_B ? (const void*)(planes + (size_t)r0 * K)
                                : (const void*)(x + (size_t)r0 * K);
    a.epi.y[0] = y + (size_t)r0 * N;
    qgemv_plan(a, layout, sm_count());
    s = layout == WL_LAYOUT_B ? launch_qgemv_b(a, st) : launch_qgemv_a(a, st);
  }
  if (planes) cudaFreeAsync(planes, st);
  return s;
}

}  // namespace
}  // namespace wl

using namespace wl;

namespace {
// Layout-B GEMV on hi/lo planes, 32 rows per launch; `tiled`: W is the tiled
// decode copy made by wl_qtile_repack.
int qgemv_planes_op(int type, const void* W, int K, int N, const void* xp, size_t x_plane, int B,
                    float* y, bool tiled, cudaStream_t st) {
  GemvArgs a;
  a.type = type;
  a.nseg = 1;
  a.tiled = tiled;
  a.seg[0].W = (const uint8_t*)W;
  a.seg[0].N = N;
  a.seg[0].pitch = N / 32 * bb(type);
  a.seg[0].groups = (N + 255) / 256;
  a.K = K;
  a.ldx = K;
  a.xkind = X_PLANES;
  a.x_plane = x_plane;
  a.epi.kind = EPI_F32;
  a.epi.ldy[0] = N;
  for (int r0 = 0; r0 < B; r0 += 32) {
    a.B = std::min(32, B - r0);
    a.x = (const __half*)xp + (size_t)r0 * K;
    a.epi.y[0] = y + (size_t)r0 * N;
    qgemv_plan(a, WL_LAYOUT_B, sm_count());
    WL_TRY(launch_qgemv_b(a, st));
  }
  return WL_OK;
}
}  // namespace

extern "C" {

const char* wl_last_error(void) { return g_err.c_str(); }
const char* wl_version(void) { return "woolly-b200 0.1 (sm_100a)"; }

size_t wl_block_size(int t) { return type_valid((uint32_t)t) ? type_block_size((uint32_t)t) : 0; }
size_t wl_type_size(int t) { return type_valid((uint32_t)t) ? type_size((uint32_t)t) : 0; }

// ---------------- GGUF ----------------
struct wl_gguf {
  GgufFile* f;
};

int wl_gguf_open(const char* path, wl_gguf** out) {
  if (!path || !out) return fail(WL_ERR_INVALID_ARGUMENT, "null argument");
  GgufFile* f = nullptr;
  WL_TRY(gguf_open_file(path, &f));
  *out = new wl_gguf{f};
  return WL_OK;
}

int wl_gguf_open_memory(const void* bytes, size_t n, wl_gguf** out) {
  if ((!bytes && n) || !out) return fail(WL_ERR_INVALID_ARGUMENT, "null argument");
  GgufFile* f = nullptr;
  WL_TRY(gguf_open_bytes((const uint8_t*)bytes, n, &f));
  *out = new wl_gguf{f};
  return WL_OK;
}

void wl_gguf_close(wl_gguf* g) {
  if (!g) return;
  delete g->f;
  delete g;
}

int wl_gguf_header(const wl_gguf* g, uint32_t* version, uint64_t* tc, uint64_t* kvc,
                   uint32_t* alignment, uint64_t* data_start) {
  if (!g) return fail(WL_ERR_INVALID_ARGUMENT, "null gguf");
  if (version) *version = g->f->version;
  if (tc) *tc = g->f->tensor_count;
  if (kvc) *kvc = g->f->kv_count;
  if (alignment) *alignment = g->f->alignment;
  if (data_start) *data_start = g->f->data_start;
  return WL_OK;
}

int wl_gguf_tensor_count(const wl_gguf* g) { return g ? (int)g->f->tensors.size() : 0; }

static void fill_info(const GgufTensor& t, wl_tensor_info* o) {
  o->name = t.name.c_str();
  o->n_dims = t.n_dims;
  for (int i = 0; i < 4; i++) o->dims[i] = i < (int)t.n_dims ? t.dims[i] : 1;
  o->ggml_type = t.type;
  o->offset = t.offset;
  o->nbytes = t.nbytes();
}

int wl_gguf_tensor(const wl_gguf* g, int i, wl_tensor_info* out) {
  if (!g || !out || i < 0 || i >= (int)g->f->tensors.size())
    return fail(WL_ERR_INVALID_ARGUMENT, "tensor index out of range");
  fill_info(g->f->tensors[i], out);
  return WL_OK;
}

int wl_gguf_find_tensor(const wl_gguf* g, const char* name, wl_tensor_info* out) {
  if (!g || !name || !out) return fail(WL_ERR_INVALID_ARGUMENT, "null argument");
  const GgufTensor* t = g->f->find(name);
  if (!t) return fail(WL_ERR_TENSOR_NOT_FOUND, std::string("Tensor not found: ") + name);
  fill_info(*t, out);
  return WL_OK;
}

int wl_gguf_tensor_data(const wl_gguf* g, const char* name, const void** data, uint64_t* nbytes) {
  if (!g || !name || !data) return fail(WL_ERR_INVALID_ARGUMENT, "null argument");
  const GgufTensor* t = g->f->find(name);
  if (!t) return fail(WL_ERR_TENSOR_NOT_FOUND, std::string("Tensor not found: ") + name);
  const uint8_t* p = g->f->data(*t);
  if (!p)
    return fail(WL_ERR_BUFFER_TOO_SMALL, "Buffer too small: tensor data extends past end of file");
  *data = p;
  if (nbytes) *nbytes = t->nbytes();
  return WL_OK;
}

int wl_gguf_get_u32(const wl_gguf* g, const char* key, uint32_t* out) {
  if (!g || !key || !out) return fail(WL_ERR_INVALID_ARGUMENT, "null argument");
  if (!g->f->get_u32(key, out)) return fail(WL_ERR_TENSOR_NOT_FOUND, std::string("no u32 key ") + key);
  return WL_OK;
}

int wl_gguf_get_f32(const wl_gguf* g, const char* key, float* out) {
  if (!g || !key || !out) return fail(WL_ERR_INVALID_ARGUMENT, "null argument");
  if (!g->f->get_f32(key, out)) return fail(WL_ERR_TENSOR_NOT_FOUND, std::string("no f32 key ") + key);
  return WL_OK;
}

int wl_gguf_get_str(const wl_gguf* g, const char* key, const char** out, uint64_t* len) {
  if (!g || !key || !out) return fail(WL_ERR_INVALID_ARGUMENT, "null argument");
  auto it = g->f->kv.find(key);
  if (it == g->f->kv.end() || it->second.type != 8)
    return fail(WL_ERR_TENSOR_NOT_FOUND, std::string("no string key ") + key);
  *out = it->second.s.c_str();
  if (len) *len = it->second.s.size();
  return WL_OK;
}

// GGUFModelLoader::extract_config (woolly-core/src/model/loader.rs:104-156)
int wl_gguf_model_config(const wl_gguf* g, wl_model_config* c) {
  if (!g || !c) return fail(WL_ERR_INVALID_ARGUMENT, "null argument");
  const GgufFile* f = g->f;
  std::string arch;
  if (!f->get_str("general.architecture", &arch))
    return fail(WL_ERR_INVALID_FORMAT, "No architecture specified in GGUF");
  memset(c, 0, sizeof(*c));
  snprintf(c->architecture, sizeof(c->architecture), "%s", arch.c_str());
  uint32_t u;
  float x;
  c->vocab_size = f->get_u32(arch + ".vocab_size", &u) ? u : (f->get_u32("tokenizer.ggml.tokens.len", &u) ? u : 32000);
  c->hidden_size = f->get_u32(arch + ".embedding_length", &u) ? u : (f->get_u32(arch + ".embed_dim", &u) ? u : 4096);
  c->num_layers = f->get_u32(arch + ".block_count", &u) ? u : (f->get_u32(arch + ".layer_count", &u) ? u : 32);
  c->num_heads = f->get_u32(arch + ".attention.head_count", &u) ? u : 32;
  c->context_length = f->get_u32(arch + ".context_length", &u) ? u : (f->get_u32("tokenizer.ggml.context_length", &u) ? u : 2048);
  c->intermediate_size = f->get_u32(arch + ".feed_forward_length", &u) ? u : c->hidden_size * 4;
  c->num_kv_heads_meta = f->get_u32(arch + ".attention.head_count_kv", &u) ? u : 0;
  c->rope_theta = f->get_f32(arch + ".rope.freq_base", &x) ? x : (f->get_f32(arch + ".attention.rope_theta", &x) ? x : 0.f);
  c->layer_norm_epsilon = f->get_f32(arch + ".attention.layer_norm_epsilon", &x) ? x : (f->get_f32(arch + ".layer_norm_epsilon", &x) ? x : 1e-5f);
  return WL_OK;
}

// ---------------- device ops ----------------
int wl_dequantize(int type, const void* blocks, size_t nbytes, size_t n, float* out, void* stream) {
  if ((!blocks && n) || (!out && n)) return fail(WL_ERR_INVALID_ARGUMENT, "null pointer");
  size_t need;
  if (type == WL_F32 || type == WL_F16) {
    need = n * (type == WL_F32 ? 4 : 2);
    if (nbytes != need)  // dequantize.rs:250-283 require the exact length
      return fail(WL_ERR_BUFFER_TOO_SMALL, "Buffer too small: needed " + std::to_string(need) +
                                                " bytes, but only " + std::to_string(nbytes) + " available");
  } else if (bb(type)) {
    need = (n + 31) / 32 * bb(type);
    if (nbytes < need)
      return fail(WL_ERR_BUFFER_TOO_SMALL, "Buffer too small: needed " + std::to_string(need) +
                                                " bytes, but only " + std::to_string(nbytes) + " available");
  } else if (type == 12 || type == 14) {  // Q4_K / Q6_K: every super-block must be present
    need = (n + 255) / 256 * (type == 12 ? 144 : 210);
    if (nbytes < need)
      return fail(WL_ERR_INVALID_FORMAT, std::string("Invalid tensor info: ") +
                                             (type == 12 ? "Q4_K" : "Q6_K") + " data too small");
  } else if (type == 6 || type == 7 || type == 13 || type == 15) {
    // Q5_0 / Q5_1 / Q5_K / Q8_K: the reference returns zeros (dequantize.rs:539-551, 595-607)
  } else {
    return fail(type_valid((uint32_t)type) ? WL_ERR_UNSUPPORTED : WL_ERR_INVALID_TENSOR_TYPE,
                "dequantize: type " + std::to_string(type) + " not supported");
  }
  return launch_dequant(type, blocks, n, out, (cudaStream_t)stream);
}

int wl_qgemv(int type, int layout, const void* W, int K, int N, const float* x, int B, float* y,
             void* stream) {
  if (!W || !x || !y) return fail(WL_ERR_INVALID_ARGUMENT, "null pointer");
  if (kquant_type(type)) {
    // K-quants run from the tiled copy: made here in a stream-ordered temporary
    if (layout != WL_LAYOUT_B) return fail(WL_ERR_UNSUPPORTED, "qgemv: K-quant weights need layout B");
    if (K <= 0 || K % 16 || N <= 0 || N % 256 || B <= 0)
      return fail(WL_ERR_INVALID_ARGUMENT, "qgemv: K-quants need K % 16 == 0, N % 256 == 0, B > 0");
    cudaStream_t st = (cudaStream_t)stream;
    uint8_t* tiled = nullptr;
    __half* planes = nullptr;
    const size_t n = (size_t)B * K;
    int s = cudaMallocAsync((void**)&tiled, qtile_bytes(type, K, N), st) == cudaSuccess &&
                    cudaMallocAsync((void**)&planes, 2 * n * sizeof(__half), st) == cudaSuccess
                ? WL_OK
                : fail(WL_ERR_CUDA, "qgemv: out of device memory");
    if (!s) s = launch_repack_tiled(type, (const uint8_t*)W, K, N, N / 256 * kquant_block_bytes(type), tiled, st);
    if (!s) s = launch_split_planes(x, planes, n, n, st);
    if (!s) s = qgemv_planes_op(type, tiled, K, N, planes, n, B, y, true, st);
    if (tiled) cudaFreeAsync(tiled, st);
    if (planes) cudaFreeAsync(planes, st);
    return s;
  }
  if (!bb(type)) return fail(WL_ERR_UNSUPPORTED, "qgemv: type must be Q4_0, Q4_1 or Q8_0");
  if (layout != WL_LAYOUT_A && layout != WL_LAYOUT_B) return fail(WL_ERR_INVALID_ARGUMENT, "bad layout");
  if (K <= 0 || N <= 0 || B <= 0) return fail(WL_ERR_INVALID_ARGUMENT, "K, N, B must be positive");
  if ((layout == WL_LAYOUT_B ? N : K) % 32)
    return fail(WL_ERR_INVALID_ARGUMENT, "the blocked dimension must be a multiple of 32");
  return qgemv_op(type, layout, (const uint8_t*)W, K, N, x, B, y, (cudaStream_t)stream);
}

int wl_qgemv_planes(int type, const void* W, int K, int N, const void* xp, size_t x_plane, int B,
                    float* y, void* stream) {
  if (!W || !xp || !y || B <= 0) return fail(WL_ERR_INVALID_ARGUMENT, "bad argument");
  if (!bb(type)) return fail(WL_ERR_UNSUPPORTED, "qgemv: type must be Q4_0, Q4_1 or Q8_0");
  const int pitch = N / 32 * bb(type);
  if (N % 32 || !qgemv_b_fast_ok(type, K, N, pitch, W))
    return fail(WL_ERR_INVALID_ARGUMENT, "qgemv_planes: needs N % 32 == 0, K % 16 == 0, 16-byte rows");
  return qgemv_planes_op(type, W, K, N, xp, x_plane, B, y, false, (cudaStream_t)stream);
}

size_t wl_qtile_bytes(int type, int K, int N) {
  if (!(bb(type) || kquant_type(type)) || K <= 0 || N <= 0 || N % (kquant_type(type) ? 256 : 32)) return 0;
  return qtile_bytes(type, K, N);
}

int wl_qtile_repack(int type, const void* W, int K, int N, void* dst, void* stream) {
  if (!W || !dst) return fail(WL_ERR_INVALID_ARGUMENT, "null pointer");
  const bool kq = kquant_type(type);
  if (!bb(type) && !kq) return fail(WL_ERR_UNSUPPORTED, "qtile: type must be Q4_0, Q4_1, Q8_0, Q4_K or Q6_K");
  if (K <= 0 || N <= 0 || N % (kq ? 256 : 32))
    return fail(WL_ERR_INVALID_ARGUMENT, "qtile: needs K > 0, N % 32 == 0 (N % 256 == 0 for K-quants)");
  const int pitch = kq ? N / 256 * kquant_block_bytes(type) : N / 32 * bb(type);
  return launch_repack_tiled(type, (const uint8_t*)W, K, N, pitch, (uint8_t*)dst, (cudaStream_t)stream);
}

int wl_qgemv_tiled(int type, const void* Wt, int K, int N, const void* xp, size_t x_plane, int B,
                   float* y, void* stream) {
  if (!Wt || !xp || !y || B <= 0) return fail(WL_ERR_INVALID_ARGUMENT, "bad argument");
  const bool kq = kquant_type(type);
  if (!bb(type) && !kq) return fail(WL_ERR_UNSUPPORTED, "qgemv: type must be Q4_0, Q4_1, Q8_0, Q4_K or Q6_K");
  if (K <= 0 || K % 16 || N <= 0 || N % (kq ? 256 : 32) || (reinterpret_cast<uintptr_t>(Wt) & 15))
    return fail(WL_ERR_INVALID_ARGUMENT, "qgemv_tiled: needs K % 16 == 0, N % 32 == 0 (N % 256 == 0 for K-quants), 16-byte aligned copy");
  return qgemv_planes_op(type, Wt, K, N, xp, x_plane, B, y, true, (cudaStream_t)stream);
}

int wl_qgemm_tiled(int type, const void* Wt, int K, int N, const void* xp, size_t x_plane, int M,
                   float* y, void* stream) {
  if (!Wt || !xp || !y || M <= 0) return fail(WL_ERR_INVALID_ARGUMENT, "bad argument");
  const bool kq = kquant_type(type);
  if (!bb(type) && !kq) return fail(WL_ERR_UNSUPPORTED, "qgemm: type must be Q4_0, Q4_1, Q8_0, Q4_K or Q6_K");
  if (kq && N % 256) return fail(WL_ERR_INVALID_ARGUMENT, "qgemm_tiled: K-quants need N % 256 == 0");
  GemvArgs a;
  a.type = type;
  a.nseg = 1;
  a.tiled = 1;
  a.seg[0].W = (const uint8_t*)Wt;
  a.seg[0].N = N;
  a.seg[0].pitch = kq ? N / 256 * kquant_block_bytes(type) : N / 32 * bb(type);
  a.K = K;
  a.ldx = K;
  a.xkind = X_PLANES;
  a.x = xp;
  a.x_plane = x_plane;
  a.epi.kind = EPI_F32;
  a.epi.y[0] = y;
  a.epi.ldy[0] = N;
  if (!qgemm_b_ok(a, M)) return fail(WL_ERR_INVALID_ARGUMENT, "qgemm_tiled: needs K % 64 == 0, N % 128 == 0");
  return launch_qgemm_b(a, M, (cudaStream_t)stream);
}

// Prefill GEMM (tensor_utils.rs:118-157 over a whole sequence): tcgen05 tiles
// when the shape allows, else the GEMV in 32-row launches.
int wl_qgemm(int type, const void* W, int K, int N, const float* x, int M, float* y, void* stream) {
  if (!W || !x || !y) return fail(WL_ERR_INVALID_ARGUMENT, "null pointer");
  const bool kq = kquant_type(type);
  if (!bb(type) && !kq) return fail(WL_ERR_UNSUPPORTED, "qgemm: type must be Q4_0, Q4_1, Q8_0, Q4_K or Q6_K");
  if (K <= 0 || N <= 0 || M <= 0 || N % (kq ? 256 : 32) || (kq && K % 16))
    return fail(WL_ERR_INVALID_ARGUMENT, "qgemm: bad shape");
  cudaStream_t st = (cudaStream_t)stream;
  const int pitch = kq ? N / 256 * kquant_block_bytes(type) : N / 32 * bb(type);
  const bool aligned = kq || (pitch % 16 == 0 && (reinterpret_cast<uintptr_t>(W) & 15) == 0);
  if (!aligned || K % 16) return qgemv_op(type, WL_LAYOUT_B, (const uint8_t*)W, K, N, x, M, y, st);
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
  a.x_plane = (size_t)M * K;
  a.epi.kind = EPI_F32;
  a.epi.y[0] = y;
  a.epi.ldy[0] = N;
  __half* planes = nullptr;
  WL_CUDA_TRY(cudaMallocAsync((void**)&planes, (size_t)2 * M * K * sizeof(__half), st));
  int s = launch_split_planes(x, planes, (size_t)M * K, (size_t)M * K, st);
  a.x = planes;
  // the tensor-core GEMM (and any K-quant GEMV) reads the tiled copy, made here in a temporary
  const bool gemm = K % 64 == 0 && N % 128 == 0;
  uint8_t* tiled = nullptr;
  if (!s && (gemm || kq)) {
    s = cudaMallocAsync((void**)&tiled, qtile_bytes(type, K, N), st) == cudaSuccess
            ? WL_OK : fail(WL_ERR_OUT_OF_MEMORY, "qgemm: tiled copy");
    if (!s) s = launch_repack_tiled(type, (const uint8_t*)W, K, N, pitch, tiled, st);
    if (!s) {
      a.seg[0].W = tiled;
      a.tiled = 1;
    }
  }
  if (!s && gemm) {
    if (qgemm_b_ok(a, M)) s = launch_qgemm_b(a, M, st);
    else s = fail(WL_ERR_UNSUPPORTED, "qgemm: shape");
  } else {
    for (int r0 = 0; r0 < M && !s; r0 += 32) {
      a.B = std::min(32, M - r0);
      a.x = planes + (size_t)r0 * K;
      a.epi.y[0] = y + (size_t)r0 * N;
      qgemv_plan(a, WL_LAYOUT_B, sm_count());
      s = launch_qgemv_b(a, st);
    }
  }
  if (tiled) cudaFreeAsync(tiled, st);
  cudaFreeAsync(planes, st);
  return s;
}

// quantization::simd::quantized_matvec (woolly-tensor/src/quantization.rs:869-909)
int wl_quantized_matvec(int type, const void* W, const float* input, float* output, int m, int k,
                        void* stream) {
  if (type != WL_Q4_0 && type != WL_Q8_0)
    return fail(WL_ERR_UNSUPPORTED, "Quantized matvec not implemented for this scheme");
  if (k % 32) return fail(WL_ERR_INVALID_ARGUMENT, "k must be a multiple of 32");
  if (m <= 0 || k <= 0) return fail(WL_ERR_INVALID_ARGUMENT, "m, k must be positive");
  return wl_qgemv(type, WL_LAYOUT_A, W, k, m, input, 1, output, stream);
}

int wl_rmsnorm_rope(const float* x, const float* w, int rows, int dim, float eps, int rope_mode,
                    const int* pos, int head_dim, float theta, void* y, int y_f16, void* stream) {
  if (!x || !w || !y || rows < 0 || dim <= 0) return fail(WL_ERR_INVALID_ARGUMENT, "bad argument");
  if (rope_mode == WL_ROPE_NEOX && !pos) return fail(WL_ERR_INVALID_ARGUMENT, "rope needs positions");
  return launch_rmsnorm(x, w, rows, dim, eps, rope_mode == WL_ROPE_NEOX, pos, head_dim, theta, y,
                        y_f16 ? 1 : 0, 0, (cudaStream_t)stream);
}

int wl_tp_reduce_rmsnorm(float* h, const float* w, int rows, int dim, float eps, const float* slots,
                         int nranks, unsigned* counters, unsigned expect, void* y_planes,
                         size_t y_plane, int* err, void* stream) {
  if (!h || !w || !slots || !counters || !y_planes || rows < 0 || dim <= 0)
    return fail(WL_ERR_INVALID_ARGUMENT, "bad argument");
  if (nranks < 1 || nranks > kMaxPeers || rows > kPeerRows)
    return fail(WL_ERR_INVALID_ARGUMENT, "tp_reduce: 1..8 ranks and at most 32 rows");
  PeerReduce pr;
  pr.nranks = nranks;
  pr.slots = slots;
  pr.flags = counters;
  pr.done = counters + nranks;
  pr.expect = expect;
  pr.err = err;
  return launch_rmsnorm_peer(h, w, rows, dim, eps, y_planes, y_plane, pr, (cudaStream_t)stream);
}

int wl_swiglu(const float* gate, const float* up, size_t n, float* out, void* stream) {
  if (n && (!gate || !up || !out)) return fail(WL_ERR_INVALID_ARGUMENT, "null pointer");
  return launch_swiglu(gate, up, n, out, (cudaStream_t)stream);
}

int wl_sample(const float* logits, int rows, int vocab, int ld, const wl_sample_params* params,
              uint32_t* out_ids, void* stream) {
  if (rows == 0) return WL_OK;
  if (!logits || !params || !out_ids || rows < 0) return fail(WL_ERR_INVALID_ARGUMENT, "bad argument");
  return launch_sample(logits, rows, vocab, ld, params, out_ids, (cudaStream_t)stream);
}

int wl_rope(const float* x, float* out, const int* positions, float base, int batch, int seq,
            int heads, int head_dim, void* stream) {
  if (!x || !out || !positions || head_dim % 2 || batch < 0 || seq < 0 || heads < 0)
    return fail(WL_ERR_INVALID_ARGUMENT, "bad argument (head_dim must be even)");
  return launch_rope(x, out, positions, base, batch, seq, heads, head_dim, (cudaStream_t)stream);
}

int wl_attention(const float* q, const float* k, const float* v, int rows, int past, int heads,
                 int kv_heads, int head_dim, int window, float* out, void* stream) {
  if (!q || !k || !v || !out || rows <= 0 || past < 0 || heads <= 0 || kv_heads <= 0)
    return fail(WL_ERR_INVALID_ARGUMENT, "bad argument");
  return launch_attention_f32(q, k, v, rows, past, heads, kv_heads, head_dim, window, out,
                              (cudaStream_t)stream);
}

// ---------------- runtime ----------------
void wl_model_options_default(wl_model_options* o) {
  if (!o) return;
  memset(o, 0, sizeof(*o));
  o->rope_mode = WL_ROPE_OFF;
  o->sliding_window = 0;
  o->max_sessions = 16;
  o->max_context = 2048;
  o->max_batch = 16;
  o->max_prefill = 512;
  o->use_graphs = 1;
  o->tp_rank = 0;
  o->tp_size = 1;
  o->nccl_comm = nullptr;
  o->collective_timeout_ms = 60000;
}

int wl_init(int device, wl_ctx** out) {
  if (!out) return fail(WL_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0)
    return fail(WL_ERR_CUDA, std::string("no CUDA device: ") + cudaGetErrorString(e));
  if (device < 0 || device >= n) return fail(WL_ERR_INVALID_ARGUMENT, "device index out of range");
  WL_CUDA_TRY(cudaSetDevice(device));
  cudaDeviceProp p;
  WL_CUDA_TRY(cudaGetDeviceProperties(&p, device));
  if (p.major < 10)
    return fail(WL_ERR_UNSUPPORTED, std::string("woolly-b200 needs an sm_100 GPU, found ") + p.name);
  WL_TRY(noalloc_setup_current_device());
  auto* c = new wl_ctx();
  c->device = device;
  c->num_sms = p.multiProcessorCount;
  e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete c;
    return fail(WL_ERR_CUDA, cudaGetErrorString(e));
  }
  *out = c;
  return WL_OK;
}

void wl_ctx_free(wl_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  cudaStreamDestroy(c->stream);
  delete c;
}

int wl_model_load_gguf(wl_ctx* ctx, const char* path, const wl_model_options* o, wl_model** out) {
  if (!out) return fail(WL_ERR_INVALID_ARGUMENT, "null argument");
  return model_load(ctx, path, o, out);
}

void wl_model_free(wl_model* m) { model_free(m); }

int wl_model_get_config(const wl_model* m, wl_model_config* out) {
  if (!m || !out) return fail(WL_ERR_INVALID_ARGUMENT, "null argument");
  *out = m->cfg;
  return WL_OK;
}

int wl_model_memory(const wl_model* m, uint64_t* wb, uint64_t* kb) {
  if (!m) return fail(WL_ERR_INVALID_ARGUMENT, "null model");
  if (wb) *wb = m->weight_bytes;
  if (kb) *kb = m->kv_bytes;
  return WL_OK;
}

int wl_session_create(wl_model* m, wl_session** out) {
  if (!out) return fail(WL_ERR_INVALID_ARGUMENT, "null argument");
  return session_create(m, out);
}
void wl_session_free(wl_session* s) { session_free(s); }
int wl_session_reset(wl_session* s) { return session_reset(s); }
int wl_session_length(const wl_session* s) { return s ? s->len : -1; }

int wl_forward(wl_model* m, wl_session* const* ss, int n, const uint32_t* ids, const int* n_ids,
               float* logits, int mode) {
  return forward(m, ss, n, ids, n_ids, logits, mode);
}

int wl_decode_step_device(wl_model* m, wl_session* const* ss, int n, const uint32_t* d_ids,
                          float* d_logits, void* stream) {
  return decode_step_device(m, ss, n, d_ids, d_logits, (cudaStream_t)stream);
}

int wl_decode_kernel_count(const wl_model* m, int n) { return m ? decode_kernel_count(m, n) : 0; }

int wl_nccl_unique_id(void* out) {
  if (!out) return fail(WL_ERR_INVALID_ARGUMENT, "null argument");
  return nccl_unique_id(out);
}
int wl_nccl_comm_init(int nranks, const void* id, int rank, void** comm) {
  if (!id || !comm) return fail(WL_ERR_INVALID_ARGUMENT, "null argument");
  return nccl_comm_init(nranks, id, rank, comm);
}
int wl_nccl_comm_destroy(void* comm) { return nccl_comm_destroy(comm); }
int wl_nccl_comm_abort(void* comm) { return nccl_comm_abort(comm); }

}  // extern "C"
