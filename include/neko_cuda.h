/* neko_cuda.h: C ABI of the B200 (sm_100a) compute backend for NekoChat's inference engine.
 *
 * Three layers, all plain C (pointers, sizes, status codes; no C++ or torch types), implemented in
 * nekochat_b200/libneko_cuda.so:
 *
 *  1. neko_cuda_*   the engine's gpu::ComputeBackend contract (app/architecture/shared/cpp/gpu/compute.h:24-48):
 *                   buffers, upload/download, and dispatch of the nine kernels of compute.h:17 with the same
 *                   parameter blocks the GLSL shaders take. nekochat_b200/csrc/cuda_compute.cpp wraps it as a
 *                   C++ ComputeBackend subclass so Model::startGpu (model.cpp:137-148) can pick it.
 *  2. neko_op_*     single operators on device pointers (weight codec, dequant matmul, norms, softmax,
 *                   attention), for the operator sweep and for callers that manage their own memory.
 *  3. neko_model_*  a native GPT-2 / Qwen3 runner built on the same kernels: fused decode steps replayed as
 *                   CUDA graphs, plus batched multi-sequence decode (which the single-sequence
 *                   Model::forward of app/architecture/shared/cpp/model.h:72 cannot express).
 *
 * Every function returns NEKO_OK (0) or a negative status; the message is available from
 * neko_cuda_last_error (per context) or neko_last_error (thread-local, for functions without a context).
 * Streams are passed as void* (a cudaStream_t; NULL = the legacy default stream).
 */
#ifndef NEKO_CUDA_H
#define NEKO_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NEKO_ABI_VERSION 1

enum neko_status {
    NEKO_OK = 0,
    NEKO_ERR_ARG = -1,         /* bad argument or size: the engine's fail() (common.h:31) */
    NEKO_ERR_CUDA = -2,        /* a CUDA runtime call failed */
    NEKO_ERR_NOMEM = -3,       /* device allocation failed */
    NEKO_ERR_DEVICE = -4,      /* a kernel reported an error through the device error word */
    NEKO_ERR_TIMEOUT = -5,     /* a host wait passed its deadline */
    NEKO_ERR_UNSUPPORTED = -6  /* shape or format outside what the kernels implement */
};

/* Weight formats: app/architecture/shared/cpp/quant.h:19 WeightFormat. */
enum neko_format { NEKO_F16 = 0, NEKO_FP8 = 1, NEKO_FP4 = 2 };

/* Kernel ids: app/architecture/shared/cpp/gpu/compute.h:17 (order tied to NEKO_KERNELS, CMakeLists.txt:23). */
enum neko_kernel {
    NEKO_K_EMBED = 0,
    NEKO_K_LAYERNORM = 1,
    NEKO_K_MATMUL = 2,
    NEKO_K_KVSTORE = 3,
    NEKO_K_ATTENTION = 4,
    NEKO_K_ROPE = 5,
    NEKO_K_SILUMUL = 6,
    NEKO_K_MATMUL_Q8 = 7,
    NEKO_K_MATMUL_Q4 = 8
};

/* Matmul flags: gpu/shaders/matmul.comp:5 (1 = gelu, 2 = accumulate into y, 4 = add bias). NEKO_PDL (not in the
 * engine) launches neko_op_matmul with programmatic dependent launch: it may start streaming its weights while
 * the previous kernel on the stream is still running, as the decode step's matmuls do. */
enum neko_matmul_flags { NEKO_GELU = 1, NEKO_ACCUMULATE = 2, NEKO_BIAS = 4, NEKO_PDL = 256 };

typedef struct neko_ctx neko_ctx;
typedef struct neko_buf neko_buf;
typedef struct neko_model neko_model;

/* Thread-local message of the last failed call that has no context argument. */
const char* neko_last_error(void);
int neko_abi_version(void);

/* ------------------------------------------------------------------ 1. ComputeBackend contract */

/* createVulkan / createGles (compute.h:47-48): a backend on CUDA device `device`. NULL on failure with the
 * reason in err. The context owns one stream; every dispatch is ordered after the previous one
 * (compute.h:38). */
neko_ctx* neko_cuda_create(int device, char* err, size_t err_len);
/* ~ComputeBackend: frees every buffer (compute.h:32, buffers live until the backend is destroyed). */
void neko_cuda_destroy(neko_ctx* ctx);
const char* neko_cuda_last_error(neko_ctx* ctx);
/* name() (compute.h:28): "CUDA". */
const char* neko_cuda_name(neko_ctx* ctx);
/* deviceName() (compute.h:29): e.g. "NVIDIA B200 (sm_100, 148 SMs)". Returns the full length. */
int neko_cuda_device_name(neko_ctx* ctx, char* buf, size_t len);
/* maxBufferBytes() (compute.h:30). */
size_t neko_cuda_max_buffer_bytes(neko_ctx* ctx);
/* create(bytes, init, readback) (compute.h:34). readback selects pinned host staging for download. */
neko_buf* neko_cuda_create_buffer(neko_ctx* ctx, size_t bytes, const void* init, int readback);
/* upload / download (compute.h:35-36). download waits for all dispatched work first. */
int neko_cuda_upload(neko_ctx* ctx, neko_buf* b, size_t offset, const void* src, size_t bytes);
int neko_cuda_download(neko_ctx* ctx, neko_buf* b, size_t offset, void* dst, size_t bytes);
/* begin / dispatch / flush / submitAndWait (compute.h:39-44). params are the shaders' PA (0-3) and PB (4-7)
 * blocks with floats passed as raw bits (compute.h:53-58); gx, gy are the reference's workgroup counts,
 * which the backend reads as semantic sizes (rows, heads, tokens) and re-plans. NULL bindings are allowed
 * where the kernel does not read them. */
int neko_cuda_begin(neko_ctx* ctx);
int neko_cuda_dispatch(neko_ctx* ctx, int kernel, neko_buf* const bindings[4], const int32_t params[8], uint32_t gx,
                       uint32_t gy);
int neko_cuda_flush(neko_ctx* ctx);
int neko_cuda_submit_and_wait(neko_ctx* ctx);
/* Buffer introspection (Buffer::size, compute.h:20) and its device address. */
size_t neko_cuda_buffer_size(const neko_buf* b);
void* neko_cuda_buffer_device_ptr(const neko_buf* b);

/* ------------------------------------------------------------------ 2. operators on device pointers */

/* quantRowBytes (quant.cpp:199-208). */
int64_t neko_row_bytes(int format, int cols);
/* quantizeMatrix (quant.cpp:255-279) on the GPU, byte-identical to the engine's CPU quantizer: w is
 * [rows][cols] f32 with row stride ld (floats); out receives rows * neko_row_bytes bytes. cols % 32 == 0 for
 * FP8/FP4. transpose_f16 != 0 reads w as [cols][rows] (Conv1D layout) and rounds each value to f16 first,
 * as Gpt2Model::conv1d does (gpt2_model.cpp:78-82). */
int neko_op_quantize(int format, const float* w, int rows, int cols, int64_t ld, int transpose_f16, uint8_t* out,
                     void* stream);
/* QMatrix::dequantizeRow (quant.cpp:230-253) for every row: out is [rows][cols] f32, bit-exact. */
int neko_op_dequantize(int format, const uint8_t* q, int rows, int cols, float* out, void* stream);
/* cpu::matmul (cpu_ops.h:22-23) / the MatmulQ8, MatmulQ4 and Matmul kernels: y[t][n_off + n] (+)=
 * act(x[t] . W[n] + bias[n]) for n < rows, t < T. x rows have stride K; y rows have stride y_stride. */
int neko_op_matmul(int format, const float* x, int T, int K, const uint8_t* W, int rows, const float* bias,
                   float* y, int y_stride, int n_off, int flags, void* stream);
/* The fused forms the decode step uses, as one operator: norm (0 none, 1 RMSNorm, 2 LayerNorm with gamma/beta,
 * eps) applied to the x rows before the product (the engine's LayerNorm dispatch + Matmul, qwen3_model.cpp:309-311),
 * and swiglu != 0 for a [gate | up] weight of 2 * rows rows whose output is silu(x . gate[n]) * (x . up[n])
 * (Matmul + SiluMul, qwen3_model.cpp:323-325). The norm needs T * K <= 4096, K % 128 == 0 and
 * T * Kp * 4 <= 40 KB, Kp = K rounded up to 256 (F16), 512 (FP8) or 1024 (FP4) weights. */
int neko_op_matmul_fused(int format, const float* x, int T, int K, const uint8_t* W, int rows, int norm,
                         const float* gamma, const float* beta, float eps, int swiglu, const float* bias, float* y,
                         int y_stride, int n_off, int flags, void* stream);
/* cpu::rmsNorm / cpu::layerNorm (cpu_ops.cpp:483-511). beta NULL selects RMSNorm. */
int neko_op_norm(const float* x, float* y, const float* gamma, const float* beta, int rows, int C, float eps,
                 void* stream);
/* Row softmax over rows x C floats (the softmax of cpu::attention, cpu_ops.cpp:556-572, applied to rows). */
int neko_op_softmax(const float* x, float* y, int rows, int C, void* stream);
/* cpu::attention (cpu_ops.cpp:544-575) over caches in the engine layout [ctx][n_kv * hd] f16. */
int neko_op_attention(const float* q, int q_stride, const uint16_t* k_cache, const uint16_t* v_cache, float* out,
                      int T, int n_head, int n_kv, int hd, int pos0, void* stream);
/* neko_op_attention without any device allocation; it has no counterpart in the reference. For callers that
 * cannot let a library allocate device memory behind their back: engines that budget and report every byte
 * they hold (the engine's MemoryStats), callers that must not risk an out-of-memory failure in the middle of a
 * reply, and hosts that forbid allocator calls once decoding has started. The split-KV scratch is a fixed array
 * inside the library (4 MiB of partial state + 8192 tickets, held on every GPU that loads the library until
 * the process exits); shapes that need more are rejected with NEKO_ERR_UNSUPPORTED. All calls share that
 * array, so calls that can overlap on the GPU race: keep them on one stream. The first call on each device
 * looks up the array's address with that device current; make it before any stream capture. */
int neko_op_attention_noalloc(const float* q, int q_stride, const uint16_t* k_cache, const uint16_t* v_cache,
                              float* out, int T, int n_head, int n_kv, int hd, int pos0, void* stream);
/* Index of the first maximum of each row (std::max_element in Sampler::sample, sampler.cpp:24). */
int neko_op_argmax(const float* x, int rows, int C, int* out, void* stream);
/* SamplingParams (sampler.h:12-19) without the seed: the random draw is an input of neko_op_sample. */
typedef struct neko_sampling {
    float temperature;    /* <= 0: greedy */
    int top_k;            /* 0: every token (then at most NEKO_MAX_TOP_K tokens, unless greedy) */
    float top_p;
    float repeat_penalty; /* 1: off */
    int repeat_last_n;
} neko_sampling;
#define NEKO_MAX_TOP_K 1024
/* Sampler::sample (sampler.cpp:14-55) for each of `rows` rows of `logits` [rows][V] (device, modified in place
 * by the repetition penalty, as the engine's are): history [rows][hist_stride] with hist_len[r] valid tokens
 * (device; may be NULL when the penalty is off), u [rows] uniform draws in [0, 1) (device doubles; the engine's
 * draw is u times the kept candidates' sum), out [rows] token ids (device). Candidates that tie in value are
 * ordered by index. top_k above NEKO_MAX_TOP_K (or 0 with V above it) with temperature > 0: NEKO_ERR_UNSUPPORTED. */
int neko_op_sample(float* logits, int rows, int V, const int* history, const int* hist_len, int hist_stride,
                   const double* u, const neko_sampling* params, int* out, void* stream);
/* An FP8 (E4M3) checkpoint weight as f32, TensorStore::rows / toF32 (tensor_store.cpp:543-571, 578-590):
 * out[r][c] = e4m3fn(codes[r][c]) * scales[r / bR][c / bC] (device pointers), the scale tensor being the
 * checkpoint's "<name>_scale_inv" or "<name>_scale" as f32 [scale_rows][scale_cols] (1 x 1 for a per-tensor
 * scale); a block spans 128 elements along an axis when ceil(n / 128) scales cover it, else ceil(n / parts).
 * Codes 0x7F / 0xFF decode to +-480 as in the reference's table. */
int neko_op_fp8_block_dequant(const uint8_t* codes, int64_t rows, int64_t cols, const float* scales,
                              int64_t scale_rows, int64_t scale_cols, float* out, void* stream);

/* ------------------------------------------------------------------ 3. native model runner */

enum neko_arch { NEKO_ARCH_GPT2 = 0, NEKO_ARCH_QWEN3 = 1 };

/* Mirrors Gpt2Config (gpt2/cpp/gpt2_model.h:16-23) and Qwen3Config (qwen3/cpp/qwen3_model.h:17-30). */
typedef struct neko_model_config {
    int arch;          /* neko_arch */
    int vocab;
    int embd;
    int layers;
    int heads;
    int kv_heads;      /* GPT-2: = heads */
    int head_dim;      /* GPT-2: embd / heads */
    int ff;            /* MLP width (GPT-2: 4 * embd) */
    int max_pos;       /* GPT-2 n_positions; Qwen3 max_position_embeddings */
    float eps;
    double rope_theta; /* Qwen3 */
    int weight_format; /* neko_format for every matrix (columns % 32 == 0 required for FP8/FP4) */
    int context;       /* KV positions per sequence slot (<= max_pos) */
    int max_seqs;      /* KV slots: sequences that can be resident at once */
    int max_rows;      /* rows (tokens) one step may process: >= max prefill chunk and >= decode batch */
} neko_model_config;

/* Creates the runner on `device` and allocates weights, KV cache and workspace. */
neko_model* neko_model_create(int device, const neko_model_config* cfg, char* err, size_t err_len);
void neko_model_destroy(neko_model* m);
const char* neko_model_last_error(neko_model* m);
/* Uploads one checkpoint tensor (host f32, row-major as stored in the HF checkpoint; names as in the
 * checkpoint without the "model." / "transformer." prefix, e.g. "layers.3.self_attn.q_proj.weight",
 * "h.0.attn.c_attn.weight"). Matrices are quantized on the GPU into the engine's packed format and
 * concatenated like the reference loaders do (q|k|v and gate|up rows, qwen3_model.cpp:195-209). */
int neko_model_set_tensor(neko_model* m, const char* name, const float* data, int64_t rows, int64_t cols);
/* The same with the f32 data already in device memory of the model's device (no host copy). */
int neko_model_set_tensor_device(neko_model* m, const char* name, const float* d_data, int64_t rows, int64_t cols);
/* The same for an FP8 (E4M3) checkpoint weight (Qwen3-*-FP8): host codes [rows][cols] and its block scales as
 * f32 [scale_rows][scale_cols] (a BF16 scale tensor widened to f32 first); the weight is dequantized on the GPU
 * exactly as neko_op_fp8_block_dequant, then quantized into the engine's format like neko_model_set_tensor. */
int neko_model_set_tensor_fp8(neko_model* m, const char* name, const uint8_t* codes, int64_t rows, int64_t cols,
                              const float* scales, int64_t scale_rows, int64_t scale_cols);
/* Checks that every tensor was provided. Must be called before the first forward. */
int neko_model_finalize(neko_model* m);
/* Model::forward (model.h:72): tokens[0..T) of sequence `slot` at positions [pos0, pos0 + T), T <= max_rows;
 * writes the last token's logits (vocab floats, host memory). */
int neko_model_forward(neko_model* m, int slot, const int* tokens, int T, int pos0, float* logits);
/* One decode step for n sequences: slot[i] gets token[i] at position pos[i]. Host arrays in, host arrays
 * out; logits ([n][vocab]) and/or argmax ([n]) may be NULL. The step is a CUDA graph per distinct n. */
int neko_model_decode(neko_model* m, int n, const int* slots, const int* tokens, const int* pos, float* logits,
                      int* argmax);
/* Device-resident greedy decoding. neko_model_stage copies the inputs of n sequences (slot, first token,
 * its position) to the device; each neko_model_step then enqueues one decode step of those n sequences on
 * `stream` without synchronising: it embeds the staged tokens, runs every layer, takes the greedy argmax
 * (std::max_element, sampler.cpp:24) and writes it back as the next token with position + 1, so K calls decode
 * K tokens per sequence with no host round trip. max_pos must bound every position the step sees.
 * neko_model_tokens synchronises and reads the current tokens and positions back. */
int neko_model_stage(neko_model* m, int n, const int* slots, const int* tokens, const int* pos);
int neko_model_step(neko_model* m, int n, int max_pos, void* stream);
int neko_model_tokens(neko_model* m, int n, int* tokens, int* pos);
/* Stop ids and a token budget for that loop, Engine::generate's loop (engine.cpp:120-134) on the device. With
 * max_new > 0, neko_model_stage takes each staged token as the first sample (a stop id finishes the sequence, else
 * it is logged) and every neko_model_step adds one kernel after the step: a sampled stop id finishes the sequence
 * (stop reason 1, not logged), else the token is logged and the sequence finishes once max_new tokens are logged
 * (reason 0). A finished sequence stays at its last token and position, so later steps re-run that row in place
 * and write no KV beyond it. The context limit stays the caller's (max_pos of neko_model_step). max_new = 0 turns
 * it off. At most NEKO_MAX_STOP_IDS ids, each in [0, vocab). */
/* The runner's pinned host logits buffer (*floats of them; valid until neko_model_destroy). Passed as the
 * `logits` output of neko_model_forward / neko_model_decode it receives the logits straight from the device
 * copy, with no second host copy; each call overwrites it, as the engine's forward overwrites its logits vector. */
float* neko_model_host_logits(neko_model* m, size_t* floats);
#define NEKO_MAX_STOP_IDS 64
int neko_model_set_stop(neko_model* m, const int* stop_ids, int n_stop, int max_new);
/* Synchronises and reads the log of the n staged sequences: tokens [n][max_new] (-1 past each count), counts [n],
 * reasons [n] (the engine's stopReason: 0 max_new reached, 1 stop id; -1 still running). NULL outputs are
 * skipped. */
int neko_model_generated(neko_model* m, int n, int* tokens, int* counts, int* reasons);
/* Bytes held on the device: weights, KV cache, workspace (Model::memory, model.h:91). */
int neko_model_memory(neko_model* m, int64_t* weights, int64_t* kv, int64_t* workspace);
/* Model::setDebugLayers(n, stage) (model.h:93-104): with n >= 0, neko_model_forward writes, instead of the last
 * token's logits, the hidden states [T][embd] after n layers (stage 0) or the intermediate of layer n after
 * `stage` ([T][width], the engine's debugStages numbering: Qwen3 2 qkv, 3 qk-norm+rope, 4 attn, 5 o_proj+res,
 * 8 silu*up, 9 down+res; GPT-2 2 qkv, 3 attn, 4 proj+res, 6 fc+gelu, 7 fc2+res). Stages fused into a neighbour
 * (the norms, gate|up) return NEKO_ERR_UNSUPPORTED. `logits` must hold T * width floats. n < 0 turns it off. */
int neko_model_set_debug(neko_model* m, int layers, int stage);
/* Kernel launches one decode step of n sequences issues (for the bench's launch count). */
int neko_model_step_launches(neko_model* m, int n);
/* Kernel nodes in the most recently captured step graph (each step shape is captured on first use), 0 before any
 * capture: the launch count a step really issues. */
int neko_model_graph_kernels(neko_model* m);
/* Decode steps of 1..4 sequences (decode, step, and forward of one token) run as ONE persistent kernel by
 * default: enable = 0 makes them use the per-operator kernel chain instead (same results; for comparison).
 * enable = 2 is a test of the kernel's bounded waits: the next steps wait for a CTA that does not exist, give
 * up after 50 ms and report NEKO_ERR_DEVICE (the model stays usable; set 1 again afterwards).
 * Returns 1 when the single-kernel path is available for this model, 0 when not, < 0 on error. */
int neko_model_set_decode_kernel(neko_model* m, int enable);
/* Device pointer and byte size of one packed weight matrix ("layers.L.wqkv", "layers.L.wo", "layers.L.wgu",
 * "layers.L.wdown", "head"), for the GEMV roofline measurement and the dequant bit-exactness tests. */
int neko_model_matrix(neko_model* m, const char* which, const uint8_t** ptr, int* rows, int* cols);

#ifdef __cplusplus
}
#endif
#endif /* NEKO_CUDA_H */
