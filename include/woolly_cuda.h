/*
 * woolly_cuda.h — C ABI of the B200 (sm_100a) quantized transformer forward.
 *
 * Drop-in boundary for woolly's CPU hot path.  Every entry point below names
 * the reference interface it replaces (paths inside the woolly repository).
 * Conventions:
 *  - every function returns a wl_status (0 = WL_OK); wl_last_error() gives a
 *    thread-local message for the last failure on the calling thread, the way
 *    CoreError carries code + message (crates/woolly-core/src/lib.rs:30-165);
 *  - "device" pointers are CUDA global memory; "host" pointers are CPU memory;
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *    op-level calls are stream-ordered and do not synchronise;
 *  - a wl_model is read-only after load and may be shared by threads; a
 *    wl_session is used by one host thread at a time.
 */
#ifndef WOOLLY_CUDA_H
#define WOOLLY_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum wl_status {
  WL_OK = 0,
  WL_ERR_INVALID_ARGUMENT = 1, /* CoreError::InvalidInput */
  WL_ERR_IO = 2,               /* woolly_gguf::Error::Io */
  WL_ERR_INVALID_MAGIC = 3,    /* woolly_gguf::Error::InvalidMagic */
  WL_ERR_UNSUPPORTED_VERSION = 4, /* woolly_gguf::Error::UnsupportedVersion */
  WL_ERR_INVALID_FORMAT = 5,   /* InvalidMetadata / InvalidTensorInfo / InvalidString */
  WL_ERR_INVALID_TENSOR_TYPE = 6, /* woolly_gguf::Error::InvalidTensorType */
  WL_ERR_BUFFER_TOO_SMALL = 7, /* woolly_gguf::Error::BufferTooSmall */
  WL_ERR_TENSOR_NOT_FOUND = 8, /* woolly_gguf::Error::TensorNotFound */
  WL_ERR_UNSUPPORTED = 9,      /* QuantizationError::UnsupportedScheme */
  WL_ERR_CUDA = 10,            /* device error (message carries cudaGetErrorString) */
  WL_ERR_OUT_OF_MEMORY = 11,   /* CoreError::Memory / device allocation failure */
  WL_ERR_CONTEXT_FULL = 12,    /* session KV capacity exhausted */
  WL_ERR_TOKEN_OUT_OF_RANGE = 13, /* TENSOR_EMBEDDING_TOKEN_OUT_OF_RANGE */
  WL_ERR_NCCL = 14,            /* collective failure or watchdog abort */
  WL_ERR_TIMEOUT = 15          /* bounded device/host wait expired */
} wl_status;

/* GGML tensor type ids (crates/woolly-gguf/src/tensor_info.rs:15-60). */
enum { WL_F32 = 0, WL_F16 = 1, WL_Q4_0 = 2, WL_Q4_1 = 3, WL_Q8_0 = 8, WL_Q4_K = 12, WL_Q6_K = 14 };

/* Weight layouts.  LAYOUT_A is ggml's row-major [rows][K/32 blocks] used by
 * woolly-tensor's quantized_matvec (quantization.rs:1100-1163).  LAYOUT_B is
 * the woolly-core model convention: the flat dequantized buffer read as a
 * row-major [K_in][N_out] matrix, y[o] = sum_k x[k] W[k*N + o]
 * (crates/woolly-core/src/tensor_utils.rs:118-157). */
enum { WL_LAYOUT_A = 0, WL_LAYOUT_B = 1 };

/* RoPE modes: off is what LazyTransformer::forward does (no rotary call on the
 * live path); NEOX is the half-split rotation of RoPE::apply_f32
 * (crates/woolly-tensor/src/ops/mod.rs:476-527). */
enum { WL_ROPE_OFF = 0, WL_ROPE_NEOX = 1 };

/* logits modes for wl_forward */
enum { WL_LOGITS_LAST = 0, WL_LOGITS_ALL = 1 };

const char* wl_last_error(void);
const char* wl_version(void);

/* ------------------------------------------------------------------ */
/* Block formats (host, no GPU needed)                                 */

/* GGMLType::block_size / type_size (tensor_info.rs:128-177); 0 for unknown. */
size_t wl_block_size(int ggml_type);
size_t wl_type_size(int ggml_type);

/* ------------------------------------------------------------------ */
/* GGUF parsing (host).  Replaces GGUFLoader::from_path (woolly-gguf
 * loader.rs:112-199): header (format.rs:79-105), metadata (metadata.rs:156-179),
 * tensor table (tensor_info.rs:206-236), data start aligned to
 * general.alignment or 32 (loader.rs:151-164). */
typedef struct wl_gguf wl_gguf;

typedef struct wl_tensor_info {
  const char* name;
  uint32_t n_dims;
  uint64_t dims[4];
  uint32_t ggml_type;
  uint64_t offset;    /* relative to the data section */
  uint64_t nbytes;    /* TensorInfo::data_size (tensor_info.rs:244-255) */
} wl_tensor_info;

/* Model hyper-parameters as GGUFModelLoader::extract_config reads them
 * (crates/woolly-core/src/model/loader.rs:104-156). */
typedef struct wl_model_config {
  uint32_t vocab_size, hidden_size, num_layers, num_heads, context_length,
      intermediate_size, num_kv_heads_meta; /* 0 when the key is absent */
  float rope_theta;                          /* 0 when absent */
  float layer_norm_epsilon;
  char architecture[64];
} wl_model_config;

int wl_gguf_open(const char* path, wl_gguf** out);
int wl_gguf_open_memory(const void* bytes, size_t nbytes, wl_gguf** out);
void wl_gguf_close(wl_gguf* g);
int wl_gguf_header(const wl_gguf* g, uint32_t* version, uint64_t* tensor_count,
                   uint64_t* metadata_kv_count, uint32_t* alignment, uint64_t* data_start);
int wl_gguf_tensor_count(const wl_gguf* g);
int wl_gguf_tensor(const wl_gguf* g, int index, wl_tensor_info* out);
int wl_gguf_find_tensor(const wl_gguf* g, const char* name, wl_tensor_info* out);
/* pointer to a tensor's raw bytes inside the mapped file (host memory) */
int wl_gguf_tensor_data(const wl_gguf* g, const char* name, const void** data, uint64_t* nbytes);
int wl_gguf_model_config(const wl_gguf* g, wl_model_config* out);
/* metadata lookups with the exact-type rule of GGUFMetadata::get_* (metadata.rs:195-224) */
int wl_gguf_get_u32(const wl_gguf* g, const char* key, uint32_t* out);
int wl_gguf_get_f32(const wl_gguf* g, const char* key, float* out);
int wl_gguf_get_str(const wl_gguf* g, const char* key, const char** out, uint64_t* len);

/* ------------------------------------------------------------------ */
/* Synthetic model writer (host).  No reference counterpart: writes the seeded
 * LLaMA-architecture GGUF the benchmarks and parity tests use (token_embd
 * N(0,0.02) with dims [d, V], f32 or `embd_type`; projections N(0,0.02)
 * quantized to `weight_type` (attn_v / ffn_down to `vd_type`) with dims
 * [in, out]; norms f32 1+N(0,0.02)). */
typedef struct wl_synth_config {
  uint32_t hidden, layers, heads, kv_heads, ff, vocab, context_length;
  uint32_t weight_type;   /* WL_Q4_0 / WL_Q4_1 / WL_Q8_0 / WL_Q4_K / WL_Q6_K / WL_F32 */
  uint32_t output_type;   /* type of output.weight; 0xFFFFFFFF = tied (omit it) */
  uint32_t sliding_window; /* 0 = none; stored as {arch}.attention.sliding_window */
  float rope_theta, norm_eps;
  uint64_t seed;
  uint32_t vd_type;       /* 0 = weight_type; else the type of attn_v and ffn_down
                           * (the K-quant mixes keep those as Q6_K beside Q4_K) */
  uint32_t embd_type;     /* type of token_embd.weight (WL_F32 = 0 by default) */
} wl_synth_config;

int wl_synth_gguf(const char* path, const wl_synth_config* cfg);
/* quantize n f32 values (n % 32 == 0; n % 256 == 0 for Q4_K / Q6_K) into
 * GGUF blocks (published ggml absmax/min-max block schemes; woolly's own
 * quantizers are stubs; K-quant blocks encoded for woolly's reading of them). */
int wl_quantize(int ggml_type, const float* src, size_t n, void* dst_blocks);
/* fill n f32 with the writer's seeded N(mean, std) stream */
int wl_synth_normal(uint64_t seed, uint64_t stream, float mean, float std, size_t n, float* out);

/* ------------------------------------------------------------------ */
/* Device ops (stream-ordered, device pointers).                       */

/* woolly_gguf::dequantize (woolly-gguf/src/dequantize.rs:189-205) for F32,
 * F16, Q4_0, Q4_1, Q8_0 and the K-quants Q4_K / Q6_K (the reference's own
 * formulas, :381-537), bit-exact with the reference; Q5_0, Q5_1, Q5_K and
 * Q8_K yield zeros as the reference's stubs do (:539-551, :595-607).
 * `nbytes` is the size of `blocks` (BufferTooSmall semantics as the
 * reference; a short Q4_K / Q6_K buffer is WL_ERR_INVALID_FORMAT, its
 * InvalidTensorInfo). */
int wl_dequantize(int ggml_type, const void* blocks, size_t nbytes, size_t n, float* out,
                  void* stream);

/* Quantized GEMV/skinny-GEMM: y[b, o] = sum_k x[b, k] * W(k, o), b < B.
 *  layout B: W is [K][N] (N % 32 == 0), the woolly-core projection
 *            (tensor_utils_simd.rs:1032-1081, tensor_utils.rs:118-157);
 *  layout A: W is [N rows][K] (K % 32 == 0), quantized_matvec
 *            (woolly-tensor/src/quantization.rs:869-909) generalised to B rows
 *            and to Q4_1.
 * x is f32 [B][K] (row stride K), y is f32 [B][N].  B >= 1, any size (rows are
 * processed 32 at a time).
 * K-quants (WL_Q4_K, WL_Q6_K; layout B, N % 256 == 0, K % 16 == 0): W(k, o) is
 * woolly_gguf::dequantize's value of the super-block bytes (dequantize.rs:
 * 381-537); computed from a temporary tiled copy (wl_qtile_repack). */
int wl_qgemv(int ggml_type, int layout, const void* W, int K, int N, const float* x, int B,
             float* y, void* stream);

/* Layout-B GEMV on activations already split into f16 hi/lo planes
 * (x = hi + lo, lo = f16(x - hi); hi plane [B][K], lo plane x_plane elements
 * later) — the operand format the model runtime uses between kernels.  Same
 * math as wl_qgemv layout B (tensor_utils.rs:118-157); requires N % 32 == 0,
 * K % 16 == 0 and 16-byte aligned rows (N/32 * block bytes % 16 == 0). */
int wl_qgemv_planes(int ggml_type, const void* W, int K, int N, const void* x_planes,
                    size_t x_plane, int B, float* y, void* stream);

/* Tiled decode copy of a layout-B matrix (no counterpart in the reference; a
 * re-layout of the same GGUF blocks for the decode GEMV).  For each 256-column
 * group and 64-row stage the codes and f16 scales the GEMV's lanes read are
 * stored as one contiguous block, so a stage is a single coalesced copy and each
 * lane's operands are two aligned 8-byte loads.  Same size as the GGUF matrix
 * rounded up to whole (group, stage) tiles.
 * wl_qtile_bytes: bytes of the copy (0 for an unsupported type or shape).
 * wl_qtile_repack: writes the copy of W ([K][N] GGUF blocks, N % 32 == 0,
 *   row pitch N/32 * block bytes) into dst (wl_qtile_bytes bytes, 16-byte
 *   aligned), asynchronously on `stream`.  Q4_K / Q6_K: [K][N/256]
 *   super-blocks (N % 256 == 0); their copy keeps the codes and, per
 *   32 (Q4_K) or 16 (Q6_K) columns, the sub-block scale d*sc as an exact f16
 *   (hi, lo) pair (22 and 40 bytes per 32 weights).
 * wl_qgemv_tiled: wl_qgemv_planes on the tiled copy (K % 16 == 0): the same
 *   exact per-block products; the K range is split across CTAs in steps of 64
 *   rows instead of 16, so the f32 summation order (not the math) may differ. */
size_t wl_qtile_bytes(int ggml_type, int K, int N);
int wl_qtile_repack(int ggml_type, const void* W, int K, int N, void* dst, void* stream);
int wl_qgemv_tiled(int ggml_type, const void* W_tiled, int K, int N, const void* x_planes,
                   size_t x_plane, int B, float* y, void* stream);
/* Gemm::compute (woolly-tensor/src/ops/matmul.rs:83-259) for a whole prompt
 * on the tcgen05 tensor cores, with the weights given as their tiled copy
 * (the copy the model runtime keeps) and the M activation rows as f16 hi/lo
 * planes (hi plane [M][K], lo plane x_plane elements later): needs
 * K % 64 == 0, N % 128 == 0 (Q4_K / Q6_K: N % 256 == 0). */
int wl_qgemm_tiled(int ggml_type, const void* W_tiled, int K, int N, const void* x_planes,
                   size_t x_plane, int M, float* y, void* stream);

/* Quantized GEMM for prompts (prefill): y[m, o] = sum_k x[m, k] * W(k, o) for
 * all M rows in one launch, layout B (W is [K][N] GGUF blocks), the
 * woolly-core `matmul` over a whole sequence (tensor_utils.rs:118-157;
 * Gemm::compute, woolly-tensor/src/ops/matmul.rs:83-259, is the reference's
 * general GEMM entry).  x f32 [M][K], y f32 [M][N].  Runs on the tcgen05
 * tensor cores when K % 64 == 0, N % 128 == 0 and the weight rows are 16-byte
 * aligned (N/32 * block bytes % 16 == 0); other shapes take the layout-B GEMV
 * path, 32 rows per launch.  Results within f32 rounding of the restatement. */
int wl_qgemm(int ggml_type, const void* W, int K, int N, const float* x, int M, float* y,
             void* stream);

/* Allocation-free variant of wl_qgemv for layout B.  No counterpart in the
 * reference: it exists for callers that may not allocate device memory after
 * start-up (fixed-budget serving processes, hosts whose allocator belongs to
 * another framework, code paths where an allocation could stall the device).
 * Same inputs, outputs and results as wl_qgemv(..., WL_LAYOUT_B, ...).
 * Limits and behaviour:
 *  - B*K <= 524288 (2^19); larger calls fail with WL_ERR_INVALID_ARGUMENT;
 *  - the activations are staged in one fixed 2 MiB device array inside the
 *    library, which every GPU that loads the library keeps until exit;
 *  - all calls share that array: calls that overlap on the GPU (different
 *    streams, or different threads on one device) race and must be ordered by
 *    the caller; each call rewrites every element it reads, so nothing
 *    carries over between calls;
 *  - the array's device address is looked up once per device, with that
 *    device current: by wl_init(device) or, without it, by the first call on
 *    the device.  That set-up may load the library's device code for the
 *    array (lazy module loading), i.e. take device memory once, so do it
 *    (wl_init, or a first small call) before reserving the process's memory
 *    budget and before any stream capture; later calls allocate nothing;
 *  - N % 32 == 0, K % 16 == 0 and 16-byte aligned weight rows. */
int wl_qgemv_noalloc(int ggml_type, const void* W, int K, int N, const float* x, int B,
                     float* y, void* stream);

/* woolly_tensor quantization::simd::quantized_matvec(weights, input, output, m, k)
 * (quantization.rs:869): layout A, one input vector; Q4_0 and Q8_0 (Q4_1 ->
 * WL_ERR_UNSUPPORTED, as the reference). */
int wl_quantized_matvec(int ggml_type, const void* W, const float* input, float* output,
                        int m, int k, void* stream);

/* Reduce side of the tensor-parallel exchange that replaces ncclAllReduce after
 * the row-parallel projections (attn_output, ffn_down; lazy_transformer.rs:
 * 177-179 residual adds) in decode: each rank's GEMV pushes its partial rows
 * into slot [rank] of every rank's buffer over NVLink and adds 1 per CTA to
 * that rank's arrival counter there.  This call waits (bounded, about a
 * second) until counters[r] >= expect for every r < nranks, sets
 * h[i] += sum_r slots[r][i] (ranks in order: identical on every rank), writes
 * h back, and RMS-normalises it (tensor_utils.rs:446-480) into f16 hi/lo
 * planes (lo plane y_plane elements after hi).  slots is [nranks][32][dim]
 * f32; counters is [nranks] arrivals followed by one word the call uses to
 * re-arm them (it subtracts expect once every row is done).  A wait that
 * gives up sets bit 8 in *err (when err is non-null) and the rows are
 * invalid; the model runtime reports that as WL_ERR_TIMEOUT.  rows <= 32,
 * nranks <= 8, dim % 4 == 0. */
int wl_tp_reduce_rmsnorm(float* h, const float* w, int rows, int dim, float eps, const float* slots,
                         int nranks, unsigned* counters, unsigned expect, void* y_planes,
                         size_t y_plane, int* err, void* stream);

/* rms_norm (woolly-core tensor_utils.rs:446-480; TransformerSIMD::rms_norm
 * simd_matmul.rs:811), fused with an optional NeoX RoPE of the normalised row
 * (heads of head_dim, position pos[r]); y may be f32 (y_f16 = 0) or f16. */
int wl_rmsnorm_rope(const float* x, const float* w, int rows, int dim, float eps,
                    int rope_mode, const int* pos, int head_dim, float theta, void* y,
                    int y_f16, void* stream);

/* TransformerSIMD::swiglu_activation (simd_matmul.rs:1002) / swiglu
 * (tensor_utils.rs:512-532), exact SiLU(g) * u. */
int wl_swiglu(const float* gate, const float* up, size_t n, float* out, void* stream);

/* Next-token sampling of the server's decode loop, sample_next_token
 * (woolly-server/src/handlers/inference.rs:441-483, helpers :551-654), on the
 * GPU: per row r of logits (row stride ld, vocab entries), softmax with
 * max(temperature, 0.01), optional top-k and top-p filtering (renormalised;
 * top-p keeps nothing when no prefix exceeds p, as the reference), then
 * greedy (temperature == 0: last index of the largest probability) or the
 * first index whose running sum exceeds the row's uniform draw u (last index
 * when none does).  params and out_ids are device arrays of `rows` entries;
 * vocab <= 51200.  The draw is an input: the caller owns the random stream. */
typedef struct wl_sample_params {
  float temperature;
  int top_k;    /* 0 = off */
  float top_p;  /* >= 1 = off */
  float u;      /* uniform draw in [0, 1) */
} wl_sample_params;
int wl_sample(const float* logits, int rows, int vocab, int ld, const wl_sample_params* params,
              uint32_t* out_ids, void* stream);

/* RoPE::apply_f32 (woolly-tensor/src/ops/mod.rs:476-527), NeoX half split:
 * x [batch, seq, heads, head_dim] f32, positions [seq] (device int32). */
int wl_rope(const float* x, float* out, const int* positions, float base, int batch, int seq,
            int heads, int head_dim, void* stream);

/* GQA attention over an f32 K/V prefix (lazy_transformer.rs:375-434):
 * q [rows, H*hd], k/v [past+rows, KVH*hd]; row i sits at position past+i and
 * attends keys (pos-window, pos] (window 0 = full prefix). out [rows, H*hd]. */
int wl_attention(const float* q, const float* k, const float* v, int rows, int past,
                 int heads, int kv_heads, int head_dim, int window, float* out, void* stream);

/* ------------------------------------------------------------------ */
/* Model runtime.  Replaces LazyTransformer (woolly-core model/lazy_transformer.rs)
 * behind the Model trait (model/mod.rs:32-67) and InferenceSession
 * (session.rs:193-277). */
typedef struct wl_ctx wl_ctx;
typedef struct wl_model wl_model;
typedef struct wl_session wl_session;

typedef struct wl_model_options {
  int rope_mode;        /* WL_ROPE_OFF (reference forward) or WL_ROPE_NEOX */
  int sliding_window;   /* 0: from metadata (or none); -1: force none; >0: window */
  int max_sessions;     /* sessions that may exist at once (KV page pool sizing) */
  int max_context;      /* per-session token capacity */
  int max_batch;        /* largest batched decode (sessions per step) */
  int max_prefill;      /* largest prompt chunk per forward call */
  int use_graphs;       /* capture decode steps in CUDA graphs */
  int tp_rank, tp_size; /* tensor parallel shard (tp_size 1 = whole model) */
  void* nccl_comm;      /* ncclComm_t when tp_size > 1 */
  int ggml_layout;      /* 0: the reference's reading of every 2-D weight [ne0, ne1]
                           as [ne0][ne1] (layout B, its parity semantics); 1: ggml's
                           orientation, ne1 rows of ne0 values and token_embd one
                           row per token (llama.cpp checkpoints; single GPU) */
  int collective_timeout_ms; /* tp_size > 1: longest wait for a step (and its
                                collectives) to finish; on expiry the NCCL
                                communicator is aborted, the call returns
                                WL_ERR_TIMEOUT and later calls WL_ERR_NCCL:
                                close and reload (0 = 60000) */
} wl_model_options;

void wl_model_options_default(wl_model_options* o);

int wl_init(int device, wl_ctx** out);
void wl_ctx_free(wl_ctx* ctx);

/* Loads the GGUF into HBM.  Replaces LazyTransformer::from_gguf
 * (lazy_transformer.rs:29-95) and its dequantization cache.  Projection
 * weights (Q4_0, Q4_1, Q8_0, Q4_K, Q6_K or F32, mixed freely) are kept once,
 * in the lane-ready tiled copy the GEMV and GEMM read (ggml orientation:
 * quantized rows as stored, K-quant super-blocks padded to 16 bytes); a
 * tensor-parallel shard keeps its column / row slice.  token_embd.weight may
 * be F32 or any type wl_dequantize reads; it is held as an f32 table. */
int wl_model_load_gguf(wl_ctx* ctx, const char* path, const wl_model_options* opts,
                       wl_model** out);
void wl_model_free(wl_model* m);
int wl_model_get_config(const wl_model* m, wl_model_config* out);
/* device bytes held by weights and by the KV page pool */
int wl_model_memory(const wl_model* m, uint64_t* weight_bytes, uint64_t* kv_bytes);

int wl_session_create(wl_model* m, wl_session** out);
void wl_session_free(wl_session* s);
int wl_session_reset(wl_session* s);
int wl_session_length(const wl_session* s);

/* Model::forward (lazy_transformer.rs:1155-1336) for n_sess sessions at once:
 * session i appends n_ids[i] host token ids (ids packed back to back) to its
 * KV and gets logits (host f32): mode ALL -> n_ids[i]*V rows, LAST -> V.
 * When every n_ids[i] == 1 the call is one batched decode step. */
int wl_forward(wl_model* m, wl_session* const* sessions, int n_sess, const uint32_t* ids,
               const int* n_ids, float* logits, int mode);

/* Device-resident decode step (no host copies): d_ids [n_sess] device u32,
 * d_logits [n_sess][V] device f32.  Stream-ordered on `stream`. */
int wl_decode_step_device(wl_model* m, wl_session* const* sessions, int n_sess,
                          const uint32_t* d_ids, float* d_logits, void* stream);
/* number of kernels one decode step launches (for launch accounting) */
int wl_decode_kernel_count(const wl_model* m, int n_sess);

/* Tensor parallel helpers: the NCCL unique id is 128 bytes. */
int wl_nccl_unique_id(void* out128);
int wl_nccl_comm_init(int nranks, const void* id128, int rank, void** comm_out);
int wl_nccl_comm_destroy(void* comm);
/* ncclCommAbort: ends every collective in flight on the communicator (the
 * recovery when a rank stopped participating, see collective_timeout_ms). */
int wl_nccl_comm_abort(void* comm);

#ifdef __cplusplus
}
#endif
#endif
