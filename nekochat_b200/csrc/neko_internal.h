// Internal host-side declarations shared by the CUDA translation units of libneko_cuda.so.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/neko_cuda.h"

#include <cstdint>
#include <string>
#include <utility>

namespace neko {

// Launch with optional programmatic dependent launch (the kernel may start while the previous kernel on the
// stream finishes; it synchronises itself with griddepcontrol.wait).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                             Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

int num_sms();  // of the current device, cached per device
// Dynamic shared memory of a kernel on the current device. The library is linked with relocatable device code,
// so the device linker sizes each kernel's static shared memory: budgets are taken from the queried figure, never
// from an assumed margin. max_dyn_smem: the opt-in per-block limit less the kernel's static shared memory.
// ensure_dyn_smem: raises the kernel's attribute to bytes (the attribute only grows; cached per function and
// device); cudaErrorNotSupported, with no CUDA call made, when bytes exceed max_dyn_smem.
int max_dyn_smem(const void* fn);
cudaError_t ensure_dyn_smem(const void* fn, size_t bytes);
template <typename F>
inline int max_dyn_smem(F* fn) { return max_dyn_smem(reinterpret_cast<const void*>(fn)); }
template <typename F>
inline cudaError_t ensure_dyn_smem(F* fn, size_t bytes) { return ensure_dyn_smem(reinterpret_cast<const void*>(fn), bytes); }

// ------------------------------------------------------------------ weight codec (k_quant.cu)
cudaError_t launch_quantize(int fmt, const float* w, int rows, int cols, int64_t ld, int transpose, uint8_t* out,
                            cudaStream_t st);
cudaError_t launch_dequantize(int fmt, const uint8_t* q, int rows, int cols, float* out, cudaStream_t st);

// ------------------------------------------------------------------ dequant GEMV (k_gemv.cu)
enum NormKind : int { kNormNone = 0, kNormRms = 1, kNormLayer = 2 };

struct GemvArgs {
    const uint8_t* W = nullptr;  // packed rows (engine layout)
    int64_t row_bytes = 0;
    int rows = 0;                // output rows (row pairs when pair_off != 0)
    int K = 0;
    int fmt = 0;
    const float* x = nullptr;    // M activation rows, row m at x + m * x_stride
    int64_t x_stride = 0;
    int M = 1;
    int norm = kNormNone;        // applied to x rows while staging them (needs x staged in shared memory)
    const float* gamma = nullptr;
    const float* beta = nullptr;
    float eps = 0.0f;
    const float* bias = nullptr;
    int flags = 0;               // kGelu | kAccumulate | kBias
    float* y = nullptr;          // out row m at y + m * y_stride + n_off
    int64_t y_stride = 0;
    int n_off = 0;
    int64_t pair_off = 0;        // != 0: out n = silu(row n) * row(n + pair_off)  (SwiGLU epilogue)
    unsigned long long* argmax = nullptr;  // M <= 64: per-row atomicMax of (value, ~index) keys (fused greedy argmax)
    // Greedy finalize by the last CTA (the FP8 tensor-core GEMV with argmax): fin_count counts the CTAs done (zero
    // between launches); the last one turns the keys into token ids (fin_argmax), clears them and, with
    // fin_advance, writes the next input token and position + 1 (argmax_finalize_kernel semantics)
    unsigned* fin_count = nullptr;
    int* fin_argmax = nullptr;
    int* fin_tokens = nullptr;
    int* fin_pos = nullptr;
    int fin_context = 0;
    int fin_advance = 0;
    // tensor-core path (5+ rows): workspace for K splits and split activations, tickets zero between launches
    float* ws = nullptr;
    int64_t ws_floats = 0;
    unsigned* ws_tickets = nullptr;
    int ws_ntickets = 0;
    // tensor-core chaining (5..127 rows, FP8 / FP4): each matmul's epilogue prepares the next one's input.
    //  * x_hi / x_lo: the activations already split into f16 hi + lo ([M][K] each); no split kernel runs.
    //  * in_ss: RMSNorm as a row scale. The activations hold x * gamma; y[m] is multiplied by
    //    rstd[m] = 1 / sqrt(sum_{t < in_ss_tiles} in_ss[t * M + m] / K + eps) before the bias / activation.
    //  * out_hi / out_lo: the epilogue also writes the output times (out_gamma ? out_gamma[n] : 1) split into
    //    hi + lo f16 at [m * out_ld + n]; out_ss: the sums of squares of the output over each CTA's columns
    //    (column tile t, row m) at out_ss[t * M + m], for a consumer's in_ss.
    const __half* x_hi = nullptr;
    const __half* x_lo = nullptr;
    const float* in_ss = nullptr;
    int in_ss_tiles = 0;
    __half* out_hi = nullptr;
    __half* out_lo = nullptr;
    int64_t out_ld = 0;
    const float* out_gamma = nullptr;
    float* out_ss = nullptr;
    // launch plan (filled by plan_gemv)
    int x_smem = 0;
    int rows_per_cta = 0;
    int stage_rows = 0;          // weight rows per ring stage (<= 8 warps x rows per warp)
    int nstage = 0;
    int64_t stage_stride = 0;
    int xs_off = 0;
    int ring_off = 0;
};

// Shared-memory budget of one GEMV CTA. Two fit on an SM, so the next kernel's CTAs (launched early by PDL)
// can stream their weights while this one finishes.
constexpr int kGemvSmemBudget = 110 * 1024;
constexpr int kGemvXSmemMax = 40 * 1024;
// Staged activations are zero-padded to whole 512-byte segments of weight codes: 256 f16, 512 FP8 or 1024 FP4
// weights per segment.
inline int64_t gemv_x_bytes(int fmt, int M, int K) {
    const int w = fmt == 2 ? 1024 : fmt == 1 ? 512 : 256;
    return int64_t(M) * ((K + w - 1) / w) * w * 4;
}
// A norm prologue can be fused into the GEMV when M * K <= kGemvNormMaxElems, K % 128 == 0 and the padded
// activations fit the shared-memory budget.
constexpr int kGemvNormMaxElems = 4096;
inline bool gemv_norm_fusable(int fmt, int M, int K) {
    return int64_t(M) * K <= kGemvNormMaxElems && K % 128 == 0 && gemv_x_bytes(fmt, M, K) <= kGemvXSmemMax;
}

cudaError_t launch_gemv(GemvArgs a, cudaStream_t st, bool pdl, int max_ctas = 0);
// The streaming kernel for 1..4 FP8 / FP4 activation rows (k_gemv_stream.cu); cudaErrorNotSupported when the
// call does not fit it (launch_gemv then uses the general kernel).
cudaError_t launch_gemv_stream(const GemvArgs& a, cudaStream_t st, bool pdl);
// The direct-load tensor-core GEMV for 1..4 FP8 activation rows (k_gemv_fp8tc.cu); cudaErrorNotSupported when the
// call does not fit it.
cudaError_t launch_gemv_fp8_tc(const GemvArgs& a, cudaStream_t st, bool pdl);
// The tensor-core kernel for 5+ activation rows (k_mma.cu); cudaErrorNotSupported when the call does not fit.
cudaError_t launch_gemm_tc(const GemvArgs& a, cudaStream_t st, bool pdl);
// The warp-specialised tcgen05 kernel (k_umma_ws.cu) for 1..64 rows on activations split into f16 hi / lo
// ([M][K] each, 16-byte aligned): the weights as the UMMA's 128-row M side; cudaErrorNotSupported when the call
// does not fit.
bool gemm_ws_fits(const GemvArgs& a);
cudaError_t launch_gemm_ws(const GemvArgs& a, const __half* xh, const __half* xl, cudaStream_t st, bool pdl);
// The tcgen05 kernel (k_umma.cu) for 128+ rows on activations split into f16 hi / lo ([M][K] each);
// cudaErrorNotSupported when the call does not fit.
cudaError_t launch_gemm_umma(const GemvArgs& a, const __half* xh, const __half* xl, cudaStream_t st, bool pdl);
// 256+ rows: the weights dequantised once into hi / lo f16 rows in a.ws (after M x K floats of split activations;
// needs (M + matrix rows) x K floats), then a TMA-fed tcgen05 GEMM. cudaErrorNotSupported when it does not apply.
cudaError_t launch_gemm_umma_dq(const GemvArgs& a, const __half* xh, const __half* xl, cudaStream_t st, bool pdl);
constexpr int kGemmDqMinRows = 256;
// Workspace (floats, tickets) with which launch_gemm_tc splits this matmul's activations once (norm: with the
// norm prologue applied); 0, 0 when it needs none or the tensor-core path does not apply.
void gemm_tc_scratch(int fmt, int rows, int K, int M, bool pair, bool norm, int64_t* floats, int64_t* tickets);
// Kernel launches of such a matmul with that workspace (the activation split or norm, and the GEMM), 0 when the
// tensor-core path does not apply.
int gemm_tc_launches(int fmt, int rows, int K, int M, bool pair, bool norm);
int gemv_launch_count();  // number of launches launch_gemv issues per call (1)

// ------------------------------------------------------------------ other ops (k_ops.cu)
cudaError_t launch_norm(const float* x, int64_t x_stride, float* y, int64_t y_stride, const float* gamma,
                        const float* beta, int rows, int C, float eps, bool rms, cudaStream_t st, bool pdl);
cudaError_t launch_softmax(const float* x, float* y, int rows, int C, cudaStream_t st);
// Token sampling (k_sample.cu): Sampler::sample per row with caller-supplied uniform draws; top-k at most kMaxTopK
// (cudaErrorNotSupported beyond, unless greedy).
constexpr int kMaxTopK = NEKO_MAX_TOP_K;
// FP8 (E4M3) checkpoint codes times their block scales, to f32 (tensor_store.cpp:543-571)
int64_t fp8_block_of(int64_t n, int64_t parts);
cudaError_t launch_fp8_block_dequant(const uint8_t* codes, int64_t rows, int64_t cols, const float* scales,
                                     int64_t sR, int64_t sC, float* out, cudaStream_t st);
cudaError_t launch_sample(float* logits, int rows, int V, const int* hist, const int* hist_len, int hist_stride,
                          const double* u, const neko_sampling& sp, int* out, cudaStream_t st);
// Wide rows, fewer than the SMs (RMSNorm or softmax): chunks per row for launch_wide_rows, 0 when one CTA per row
// is the better plan. launch_wide_rows needs rows x S x 2 doubles of scratch in part.
constexpr int kWideRowMinC = 16384;
int wide_row_chunks(int rows, int C);
cudaError_t launch_wide_rows(const float* x, int64_t x_stride, float* y, int64_t y_stride, const float* gamma,
                             int rows, int C, float eps, bool softmax, double* part, int S, cudaStream_t st);
cudaError_t launch_argmax(const float* x, int64_t stride, int rows, int C, int* out, cudaStream_t st, bool pdl);
cudaError_t launch_silu_mul(const float* h, float* g, int T, int I, cudaStream_t st);
// Embedding gather (embed.comp semantics + the native runner's f32 position table):
// x[t][c] = deq(table[tok[t] - row_base])[c] (+ wpe[pos][c]); tokens outside [row_base, row_base + nrows) are
// skipped. wpe16 is an f16 table (the reference GPU path), wpe32 an f32 one (the CPU path); pos per row from
// pos_arr when not NULL, else pos0 + t.
cudaError_t launch_embed(const int* tokens, int T, int C, int fmt, const uint8_t* table, int64_t rb, int row_base,
                         int nrows, const uint16_t* wpe16, const float* wpe32, int pos0, const int* pos_arr, float* x,
                         cudaStream_t st, bool pdl);

// QK-norm + RoPE + KV-cache store for rows of a fused qkv buffer (rope.comp + kv_store.comp semantics).
struct QkvPostArgs {
    float* qkv = nullptr;
    int64_t qkv_stride = 0;          // floats between rows
    int rows = 0;
    int n_head = 0, n_kv = 0, hd = 0;
    int do_norm = 0;                 // per-head RMSNorm with wn (q: wn[0..hd), k: wn[hd..2hd))
    const float* wn = nullptr;
    float eps = 0.0f;
    int do_rope = 0;                 // NeoX rotation from cs [pos][hd/2](cos, sin)
    const float* cs = nullptr;
    int rope_kv_heads = 1;           // 1: rotate the key heads too (always, in the models)
    int store_kv = 0;                // write K, V (f16) to the caches
    uint16_t* kc = nullptr;
    uint16_t* vc = nullptr;
    int64_t slot_stride = 0, pos_stride = 0, head_stride = 0;  // cache element strides
    const int* row_slot = nullptr;   // per-row slot (NULL: slot0)
    const int* row_pos = nullptr;    // per-row position (NULL: pos0 + row)
    int slot0 = 0, pos0 = 0;
    int k_off = 0, v_off = 0;        // column offsets of K and V inside a qkv row
    int pos_limit = 0x7fffffff;      // positions >= limit are not stored (device error kErrBadIndex)
    int write_back_k = 0;            // also write the rotated keys back into qkv (debug dumps)
};
cudaError_t launch_qkv_post(const QkvPostArgs& a, cudaStream_t st, bool pdl);

// ------------------------------------------------------------------ attention (k_attention.cu)
struct AttnArgs {
    const float* q = nullptr;        // row r, head h at q + r * q_stride + h * hd
    int64_t q_stride = 0;
    const uint16_t* kc = nullptr;    // element (slot, pos, kvh, d) at kc + slot*slot_stride + pos*pos_stride
    const uint16_t* vc = nullptr;    //                                    + kvh*head_stride + d
    int64_t slot_stride = 0, pos_stride = 0, head_stride = 0;
    const int* row_slot = nullptr;
    const int* row_pos = nullptr;
    int slot0 = 0, pos0 = 0;
    int rows = 0, n_head = 0, n_kv = 0, hd = 0;
    float scale = 0.0f;
    float* out = nullptr;            // row r, head h at out + r * out_stride + h * hd
    int64_t out_stride = 0;
    int max_pos = 0;                 // upper bound of any row's position (sizes the split-KV grid)
    int pos_limit = 0x7fffffff;      // rows whose position is >= limit or > the planned max_pos are skipped
    // split-KV scratch: partial (max, sum, acc[hd]) per (row, q head, split) and one ticket per (row, kv head)
    float* part = nullptr;
    unsigned* tickets = nullptr;
    int64_t part_capacity = 0;       // floats available in part
    int64_t ticket_capacity = 0;
    // rows of hd elements in each of kc and vc (0: unknown). Known, with positions hd apart, it lets the kernel
    // stage key / value chunks with 2D tensor copies bounded by the arrays.
    int64_t cache_rows = 0;
    // optional: the output also as f16 hi + lo (row r, head h at out_hi + r * out_hl_stride + h * hd), the next
    // matmul's split activations (tensor-core kernel only)
    __half* out_hi = nullptr;
    __half* out_lo = nullptr;
    int64_t out_hl_stride = 0;
    // Qwen3 decode steps (every row a different slot, one new position each; TMA variant only): q, k, v arrive
    // raw in the qkv rows (q at q, k at q + k_off, v at q + v_off, per row q_stride) and the kernel applies the
    // per-head RMSNorm (post_wn: q gains [hd], then k gains [hd]; post_eps) and the NeoX rotation (post_cs
    // [pos][hd] cos / sin pairs) itself, stores the new key / value rows into the caches and uses them in place
    // of the cache rows it reads (which qkv_post would otherwise have written before the launch)
    int fuse_post = 0;
    const float* post_wn = nullptr;
    const float* post_cs = nullptr;
    float post_eps = 0.0f;
    int k_off = 0, v_off = 0;
};
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st, bool pdl);
// Scratch the split-KV attention needs for rows x n_head heads up to position max_pos (tma: the caller may pass
// cache_rows, so the TMA variant's plan is covered too).
void attention_scratch(int rows, int n_head, int n_kv, int hd, int max_pos, int64_t* part_floats,
                       int64_t* tickets, bool tma = false);
// Head counts and head dim the attention kernels take: n_head a multiple of n_kv, at most 8 query heads per
// KV head, hd a multiple of 8 up to 256.
bool attention_shape_ok(int n_head, int n_kv, int hd);

// ------------------------------------------------------------------ decode-step kernel (k_decode.cu)
// One whole decode step (embedding, every layer, final norm, LM head, greedy argmax) of 1..4 sequences in a
// single persistent launch. Weight pointers per layer; matrices use the packed rows of one format.
constexpr int kDecodeMaxLayers = 64;
constexpr int kDecodeMaxSeqs = 4;
struct DecodeLayer {
    const uint8_t *wqkv = nullptr, *wo = nullptr, *wup = nullptr, *wdown = nullptr;
    const float *ln1 = nullptr, *ln2 = nullptr, *ln1b = nullptr, *ln2b = nullptr, *qknorm = nullptr;
    const float *bqkv = nullptr, *bo = nullptr, *bup = nullptr, *bdown = nullptr;
    uint16_t *kc = nullptr, *vc = nullptr;  // this layer's caches [slot][kv head][pos][hd]
};
struct DecodeParams {
    int M = 0;          // sequences (activation rows), <= kDecodeMaxSeqs
    int grid = 0;       // CTAs (one per SM, all co-resident)
    int qwen = 0;       // 1: Qwen3 (RMSNorm, QK-norm, RoPE, SwiGLU); 0: GPT-2 (LayerNorm, biases, GELU, wpe)
    int fmt = 0;        // weight format of every matrix
    int layers = 0;
    int C = 0, H = 0, KV = 0, hd = 0, F = 0, V = 0, QW = 0, context = 0;
    int64_t rb_c = 0, rb_att = 0, rb_f = 0;  // row bytes of matrices with C, H * hd and F columns
    float eps = 0.0f, scale = 0.0f;
    const uint8_t* embed = nullptr;  // [V] rows, also the tied LM head
    const float *normf = nullptr, *normfb = nullptr, *rope = nullptr, *wpe = nullptr;
    int64_t kv_slot = 0, kv_head = 0;  // cache element strides (positions are hd apart)
    // Exchange buffers of tagged words (float bits | tag << 32), one per hand-off: x [M][C], q|k|v [M][QW],
    // attention output [M][H * hd], SwiGLU / GELU output [M][F], split-KV partials
    // [M][KV][max_splits][group][hd + 2] (max, sum, unnormalised P.V). Any initial content whose tags the epoch
    // never produces (zeros with the epoch starting at 1).
    uint64_t *x_tw = nullptr, *qkv_tw = nullptr, *att_tw = nullptr, *h_tw = nullptr, *part_tw = nullptr;
    unsigned* epoch = nullptr;           // tag base of the next step; the kernel advances it by the stride
    float* logits = nullptr;
    float* x_final = nullptr;            // non-null: no LM head phase; the last layer's residual rows go here as
                                         // plain floats [M][C] for a separate LM-head launch (and no argmax)
    int *tokens = nullptr, *slots = nullptr, *pos = nullptr, *argmax = nullptr;
    unsigned long long* keys = nullptr;  // greedy argmax keys (zero between steps)
    int advance = 0;                     // device greedy loop: next token = argmax, position + 1
    unsigned* sync = nullptr;            // one counter: CTAs done with the step (zero between steps)
    int span = 0, max_splits = 0;        // keys per attention split; splits per (seq, kv head) at most
    uint64_t wait_ns = 2000000000ull;    // a wait of the kernel gives up after this long (device error)
    int stall_test = 0;                  // 1: a wait that nothing satisfies (exercises the timeout path)
    // shared-memory plan (filled by plan_decode)
    int slot_bytes = 0, nslot = 0, xs_bytes = 0, kv_bytes = 0;
    DecodeLayer layer[kDecodeMaxLayers];
};
// Checks that the step fits the kernel and plans its shared memory; false (with a reason) when it does not.
bool plan_decode(DecodeParams& p, std::string* why);
// Exchange-buffer sizes (64-bit words) for p.M sequences.
struct DecodeScratch {
    int64_t part_words = 0, x_words = 0, qkv_words = 0, att_words = 0, h_words = 0;
};
void decode_scratch(const DecodeParams& p, DecodeScratch* s);
// Tag values one step uses: the epoch advances by this much per step.
__host__ __device__ inline unsigned decode_epoch_stride(int layers) { return unsigned(layers + 2) * 8u; }
cudaError_t launch_decode(const DecodeParams& p, cudaStream_t st);  // p planned by plan_decode
cudaError_t decode_clear_abort();  // after a wait of the kernel gave up (device error reported)

// ------------------------------------------------------------------ errors
std::string cuda_msg(cudaError_t e, const char* what);
void set_last_error(const std::string& msg);  // the thread-local message behind neko_last_error()
unsigned read_device_error(bool clear);
// Copies the device error flag into `host` (pinned) on `st`: read after the stream's own synchronisation
cudaError_t enqueue_device_error_read(unsigned* host, cudaStream_t st);

}  // namespace neko
