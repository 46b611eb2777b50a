// Native GPT-2 / Qwen3 runner on the sm_100a kernels (the neko_model_* ABI of include/neko_cuda.h).
//
// It computes what Gpt2Model::forwardCpu / Qwen3Model::forwardCpu compute (app/architecture/gpt2/cpp/
// gpt2_model.cpp:179-218, qwen3/cpp/qwen3_model.cpp:232-276), with the fusions the reference's one-dispatch-
// per-op sequence (forwardGpu, qwen3_model.cpp:278-341) leaves on the table:
//   Qwen3 layer = [RMSNorm -> qkv GEMV] [QK-norm + RoPE + KV store] [attention] [o_proj GEMV + residual]
//                 [RMSNorm -> gate|up GEMV -> SiLU*up] [down GEMV + residual]            6 launches (ref: 11)
//   GPT-2 layer = [LayerNorm -> qkv GEMV + bias] [KV store] [attention] [proj GEMV + bias + residual]
//                 [LayerNorm -> fc GEMV + bias + GELU] [fc2 GEMV + bias + residual]       6 launches (ref: 9)
// Final norm + LM head (+ greedy argmax) close the step. All launches after the first use programmatic
// dependent launch, so each GEMV streams its weights while its predecessor finishes, and a step is captured
// once as a CUDA graph per (rows, outputs, context bucket) and replayed.
//
// Rows: a step processes R activation rows; row r belongs to KV slot slot[r] at position pos[r]. A prefill
// chunk is R consecutive positions of one slot (Model::forward); a batched decode step is one row per
// sequence. Logits are produced for `nout` rows given by out_rows.
//
// Device memory: one arena for the packed weights (engine row format, quantized on the GPU from f32 with the
// byte-identical quantizer), one for the KV cache laid out [layer][slot][kv head][position][head dim] f16 (a
// head's keys are contiguous), and a workspace sized for max_rows.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <new>
#include <set>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/neko_cuda.h"
#include "neko_common.cuh"
#include "neko_internal.h"

using namespace neko;

namespace {

thread_local std::string t_model_err;

struct Mat {
    uint8_t* w = nullptr;
    int rows = 0, cols = 0, fmt = 0;
    int64_t rb = 0;
};

struct Layer {
    Mat wqkv, wo, wup, wdown;  // Qwen3: wup = gate|up (2F rows); GPT-2: wup = c_fc (4C rows)
    float *ln1 = nullptr, *ln2 = nullptr, *ln1b = nullptr, *ln2b = nullptr;
    float *qknorm = nullptr;  // Qwen3: q_norm | k_norm (2 hd)
    float *bqkv = nullptr, *bo = nullptr, *bup = nullptr, *bdown = nullptr;  // GPT-2 biases
};

// Greedy argmax finalize: the LM head's fused argmax left one (value, ~index) key per sequence; turn it into the
// token id, clear the key for the next step and, for the device-side greedy loop, make it the next input token
// with position + 1 (a sequence at the end of its context stays there and reports kErrBadIndex).
__global__ void argmax_finalize_kernel(unsigned long long* keys, int* argmax, int* tokens, int* pos, int n,
                                       int context, int advance) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    pdl_wait();
    if (i >= n) return;
    const int idx = int(0xFFFFFFFFu - unsigned(keys[i] & 0xFFFFFFFFull));
    keys[i] = 0ull;
    argmax[i] = idx;
    if (advance) {
        tokens[i] = idx;
        if (pos[i] + 1 < context) pos[i] += 1;
        else set_device_error(kErrBadIndex);
    }
}

// Device-side greedy loop past 64 sequences (argmax by its own kernel): the token becomes the next input token
// with position + 1, as argmax_finalize_kernel does.
__global__ void advance_kernel(const int* argmax, int* tokens, int* pos, int n, int context) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    pdl_wait();
    if (i >= n) return;
    tokens[i] = argmax[i];
    if (pos[i] + 1 < context) pos[i] += 1;
    else set_device_error(kErrBadIndex);
}

// Engine::generate's per-token bookkeeping (engine.cpp:120-134) after a device greedy step: the token each
// sequence just sampled ends it when it is a stop id (reason 1, not logged), else it is logged and ends it when
// max_new tokens are logged (reason 0). A finished sequence is frozen: its token and position are put back after
// every later step, so those steps re-run the same row at the same position (no KV beyond it is written).
// state: -1 running, else the stop reason; frozen: (token, position) pairs; log: [max_new][S].
__global__ void track_kernel(int* tokens, int* pos, int n, const int* stop_ids, int n_stop, int* counts, int* state,
                             int* frozen, int* log, int max_new, int S) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    pdl_wait();
    if (i >= n) return;
    if (state[i] >= 0) {
        tokens[i] = frozen[2 * i];
        pos[i] = frozen[2 * i + 1];
        return;
    }
    const int t = tokens[i];
    bool stop = false;
    for (int s = 0; s < n_stop; s++) stop = stop || stop_ids[s] == t;
    if (!stop) {
        const int c = counts[i];
        log[int64_t(c) * S + i] = t;
        counts[i] = c + 1;
        if (c + 1 < max_new) return;
    }
    state[i] = stop ? 1 : 0;
    frozen[2 * i] = t;
    frozen[2 * i + 1] = pos[i];
}

__global__ void gather_rows_kernel(const float* x, int C, const int* rows, int n, float* out) {
    pdl_wait();
    const int r = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < n && c < C) out[int64_t(r) * C + c] = x[int64_t(rows[r]) * C + c];
}

}  // namespace

struct neko_model {
    neko_model_config cfg{};
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    bool qwen = false;
    int C = 0, H = 0, KV = 0, hd = 0, F = 0, V = 0, QW = 0, UPW = 0;
    int fmt = 0;

    // arenas
    uint8_t* warena = nullptr;
    size_t wbytes = 0, wused = 0;
    uint16_t *kc = nullptr, *vc = nullptr;
    size_t kv_bytes = 0;
    int64_t kv_layer = 0, kv_slot = 0, kv_head = 0;  // element strides
    // workspace
    float *x = nullptr, *xn = nullptr, *qkv = nullptr, *att = nullptr, *h = nullptr, *hx = nullptr, *logits = nullptr;
    int *d_tokens = nullptr, *d_slots = nullptr, *d_pos = nullptr, *d_argmax = nullptr, *d_outrows = nullptr;
    unsigned long long* d_keys = nullptr;  // fused greedy argmax keys, one per output row (zero between steps)
    float* part = nullptr;
    unsigned* tickets = nullptr;
    int64_t part_cap = 0, tick_cap = 0;
    // matmul chaining at 5..127 rows (Qwen3): split activations in two ping-pong buffers, A [2][rows][C] (the
    // normed residual stream times gamma) and B [2][rows][max(H * hd, F)] (attention output, SwiGLU product), and
    // the residual stream's per-tile sums of squares [C / 64][rows]
    __half *ch_a = nullptr, *ch_b = nullptr;
    float* ch_ss = nullptr;
    int ch_rows = 0;
    float* mm_ws = nullptr;          // tensor-core matmul workspace (K splits, split activations)
    unsigned* mm_tickets = nullptr;
    int64_t mm_ws_floats = 0, mm_tickets_n = 0;
    size_t work_bytes = 0;
    // host pinned staging for the synchronous API
    int* h_in = nullptr;     // tokens | slots | pos | outrows  (4 * max_rows)
    float* h_logits = nullptr;
    size_t h_logits_floats = 0;
    int* h_argmax = nullptr;
    unsigned* h_err = nullptr;  // the device error flag, read with each synchronous step
    // weights
    Mat embed;               // also the tied LM head
    float* normf = nullptr;  // Qwen3 final RMSNorm / GPT-2 ln_f gamma
    float* normfb = nullptr; // GPT-2 ln_f beta
    float* rope = nullptr;   // Qwen3 [context][hd]
    float* wpe = nullptr;    // GPT-2 [max_pos][C] f32 (the CPU path keeps positions in f32)
    std::vector<Layer> layers;
    std::set<std::string> have;
    std::set<std::string> need;
    float* staging = nullptr;  // f32 upload buffer for matrices
    size_t staging_floats = 0;
    uint8_t* staging8 = nullptr;  // FP8 checkpoint codes + their f32 block scales
    // stop ids for the device greedy loop (neko_model_set_stop): ids | counts [S] | state [S] | frozen [2 S] |
    // log [max_new][S], S = max_seqs
    int track_steps = 0;
    std::vector<int> stop_ids;
    int* d_track = nullptr;
    size_t staging8_bytes = 0;
    bool final_ok = false;
    int debug_layers = -1;  // Model::setDebugLayers: stop after this many layers and output the hidden states
    int debug_stage = 0;    // > 0: stop inside layer debug_layers after this stage (debugStages numbering)
    // graphs keyed by (rows, nout, bucket, mode)
    std::map<std::tuple<int, int, int, int>, cudaGraphExec_t> graphs;
    int graph_kernels = 0;  // kernel nodes of the most recently captured step graph
    // single-kernel decode steps (k_decode.cu)
    bool dec_enabled = true;
    int dec_stall_test = 0;    // the next single-kernel step waits for a CTA that does not exist (50 ms limit)
    int dec_seqs = 0;          // most sequences one launch serves
    int dec_max_splits = 0;    // attention splits per (sequence, KV head) at the smallest span
    // single-kernel decode step: tagged-word exchange buffers (one allocation), tag epoch and the step counter
    uint64_t* dec_tw = nullptr;
    DecodeScratch dec_sz;
    int64_t dec_tw_words = 0;
    unsigned* dec_sync = nullptr;  // [0] CTAs done with the step, [1] the tag epoch, [2] LM-head CTAs done
    int dec_ok[kDecodeMaxSeqs + 1] = {-1, -1, -1, -1, -1};  // per sequence count: -1 not planned yet
};

namespace {

int fail(neko_model* m, int code, const std::string& msg) {
    if (m) m->err = msg;
    t_model_err = msg;
    return code;
}

#define CK(expr, what)                                                              \
    do {                                                                            \
        cudaError_t e_ = (expr);                                                    \
        if (e_ != cudaSuccess) return fail(m, NEKO_ERR_CUDA, cuda_msg(e_, what)); \
    } while (0)

struct Guard {
    int prev = -1;
    explicit Guard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~Guard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

int fmt_for(int cols, int f) { return cols % kQuantBlock == 0 ? f : int(kF16); }  // Model::formatFor (model.h:164)

// Carves the weight arena (two passes: size, then assign).
struct Carver {
    neko_model* m;
    bool assign;
    size_t off = 0;
    uint8_t* take(size_t n) {
        uint8_t* p = assign ? m->warena + off : nullptr;
        off += align256(n);
        return p;
    }
    float* vec(size_t n) { return reinterpret_cast<float*>(take(n * 4)); }
    Mat mat(int rows, int cols) {
        Mat t;
        t.rows = rows;
        t.cols = cols;
        t.fmt = fmt_for(cols, m->fmt);
        t.rb = row_bytes(t.fmt, cols);
        t.w = take(size_t(rows) * t.rb);
        return t;
    }
};

void carve(neko_model* m, Carver& cv) {
    const int C = m->C, V = m->V;
    m->embed = cv.mat(V, C);
    m->normf = cv.vec(C);
    if (!m->qwen) {
        m->normfb = cv.vec(C);
        m->wpe = cv.vec(size_t(m->cfg.max_pos) * C);
    } else {
        m->rope = cv.vec(size_t(m->cfg.context) * m->hd);
    }
    for (auto& L : m->layers) {
        L.wqkv = cv.mat(m->QW, C);
        L.wo = cv.mat(C, m->H * m->hd);
        L.wup = cv.mat(m->UPW, C);
        L.wdown = cv.mat(C, m->F);
        L.ln1 = cv.vec(C);
        L.ln2 = cv.vec(C);
        if (m->qwen) {
            L.qknorm = cv.vec(2 * size_t(m->hd));
        } else {
            L.ln1b = cv.vec(C);
            L.ln2b = cv.vec(C);
            L.bqkv = cv.vec(m->QW);
            L.bo = cv.vec(C);
            L.bup = cv.vec(m->UPW);
            L.bdown = cv.vec(C);
        }
    }
}

// Qwen3 rotary table [pos][hd/2](cos, sin), computed in double like Qwen3Model::ropeTable
// (qwen3_model.cpp:102-114) so the device rotates with the same table the CPU does.
std::vector<float> rope_table(int ctx, int hd, double theta) {
    std::vector<float> t(size_t(ctx) * hd);
    for (int i = 0; i < hd / 2; i++) {
        const double inv = std::pow(theta, -2.0 * i / hd);
        for (int p = 0; p < ctx; p++) {
            const double a = p * inv;
            t[size_t(p) * hd + 2 * i] = float(std::cos(a));
            t[size_t(p) * hd + 2 * i + 1] = float(std::sin(a));
        }
    }
    return t;
}

// Matmul chaining: activation rows, the column tile of the per-tile sums of squares (the tensor-core kernel's
// 64-column CTA tile), and the inputs / outputs of one chained matmul.
constexpr int kChainMaxRows = 127;
constexpr int kChainTile = 64;
struct ChainIO {
    const __half *xh, *xl;  // split input activations
    const float* in_ss;     // RMSNorm row scale from these sums of squares (null: none)
    __half *oh, *ol;        // split output * og for the next matmul (null: none)
    int64_t old;
    const float* og;
    float* oss;             // per-tile sums of squares of the output (null: none)
};
// Whether a step of R rows chains its matmuls: Qwen3, every layer matmul on the tensor-core kernel, attention
// on its tensor-core kernel.
bool chain_ok(const neko_model* m, int R);
bool chain_head_ok(const neko_model* m, int R);

int bucket_for(neko_model* m, int max_pos) {
    int b = 256;
    while (b < max_pos + 1) b *= 2;
    return std::min(b, m->cfg.context);
}

// Enqueues one step: R rows (tokens/slots/pos already in the device arrays), logits for nout rows listed in
// d_outrows (or the last row when nout == 1 and rows are one prefill chunk), optional argmax and advance.
int enqueue_step(neko_model* m, int R, int nout, bool outrows_identity, int max_pos, bool do_argmax, bool advance,
                 cudaStream_t st) {
    cudaError_t dumped = cudaSuccess;
    const int C = m->C, H = m->H, KV = m->KV, hd = m->hd;
    const float eps = m->cfg.eps;
    bool first = true;
    auto pdl = [&]() {
        const bool p = !first;
        first = false;
        return p;
    };
    // embedding rows (+ f32 positions for GPT-2)
    CK(launch_embed(m->d_tokens, R, C, m->embed.fmt, m->embed.w, m->embed.rb, 0, m->V, nullptr,
                    m->qwen ? nullptr : m->wpe, 0, m->d_pos, m->x, st, pdl()),
       "embed");

    const bool x_fits = gemv_norm_fusable(fmt_for(C, m->fmt), R, C);
    auto gemv = [&](const Mat& W, int nrows, const float* x, int64_t xs, int M, int norm, const float* g,
                    const float* b, const float* bias, int flags, float* y, int64_t ys, int64_t pair,
                    unsigned long long* keys = nullptr, const ChainIO* io = nullptr) -> cudaError_t {
        GemvArgs a;
        a.W = W.w;
        a.row_bytes = W.rb;
        a.rows = nrows;
        a.K = W.cols;
        a.fmt = W.fmt;
        a.x = x;
        a.x_stride = xs;
        a.M = M;
        a.norm = norm;
        a.gamma = g;
        a.beta = b;
        a.eps = eps;
        a.bias = bias;
        a.flags = flags;
        a.y = y;
        a.y_stride = ys;
        a.pair_off = pair;
        a.argmax = keys;
        a.ws = m->mm_ws;
        a.ws_floats = m->mm_ws_floats;
        a.ws_tickets = m->mm_tickets;
        a.ws_ntickets = int(m->mm_tickets_n);
        if (io) {
            a.x_hi = io->xh;
            a.x_lo = io->xl;
            a.in_ss = io->in_ss;
            a.in_ss_tiles = io->in_ss ? m->C / kChainTile : 0;
            a.out_hi = io->oh;
            a.out_lo = io->ol;
            a.out_ld = io->old;
            a.out_gamma = io->og;
            a.out_ss = io->oss;
        }
        return launch_gemv(a, st, pdl());
    };
    const bool staged = m->debug_layers >= 0 && m->debug_stage > 0;
    // matmul chaining (5..127 rows): A holds the next normed matmul's input (x * gamma, hi / lo), B the attention
    // output and the SwiGLU product; the RMSNorms are row scales from the per-tile sums of squares
    const bool chain = !staged && chain_ok(m, R);
    // decode steps (decode and stage refuse a slot twice; a prompt runs one slot with nout = 1) of a chained
    // Qwen3 step: the attention kernel does qkv_post's work itself
    const bool fuse_post = chain && outrows_identity && nout == R;
    const int64_t BW = std::max<int64_t>(int64_t(H) * hd, m->F);
    __half *a_hi = m->ch_a, *a_lo = m->ch_a + int64_t(R) * C;
    __half *b_hi = m->ch_b, *b_lo = m->ch_b + int64_t(R) * BW;
    // norm: applied by the matmul call (the GEMV prologue when the activations fit in shared memory, or the
    // tensor-core path's activation split) or by a separate kernel
    auto normed = [&](const Mat& W, int rows, bool pair, const float* g, const float* b, int& norm_kind,
                      const float*& src) -> cudaError_t {
        const int kind = m->qwen ? kNormRms : kNormLayer;
        if (x_fits || (!staged && gemm_tc_launches(W.fmt, rows, W.cols, R, pair, true) > 0)) {
            norm_kind = kind;
            src = m->x;
            return cudaSuccess;
        }
        norm_kind = kNormNone;
        src = m->xn;
        return launch_norm(m->x, C, m->xn, C, g, b, R, C, eps, m->qwen, st, pdl());
    };

    const size_t nlayers = m->debug_layers >= 0
                               ? std::min(m->layers.size(), size_t(m->debug_layers) + (staged ? 1 : 0))
                               : m->layers.size();
    // Model::setDebugLayers(n, stage) (model.h:93-104): inside layer n, stop after `stage` and dump that buffer.
    auto dump = [&](size_t l, int stage, const float* buf, int width) -> bool {
        if (!staged || int(l) != m->debug_layers || m->debug_stage != stage) return false;
        dumped = cudaMemcpyAsync(m->logits, buf, size_t(R) * width * 4, cudaMemcpyDeviceToDevice, st);
        return true;
    };
    for (size_t l = 0; l < nlayers; l++) {
        const Layer& L = m->layers[l];
        uint16_t* kc = m->kc + int64_t(l) * m->kv_layer;
        uint16_t* vc = m->vc + int64_t(l) * m->kv_layer;
        int nk;
        const float* src;
        if (chain && l > 0) {  // the previous layer's down projection wrote x * ln1 and the sums of squares
            const ChainIO io{a_hi, a_lo, m->ch_ss, nullptr, nullptr, 0, nullptr, nullptr};
            CK(gemv(L.wqkv, m->QW, m->x, C, R, kNormNone, nullptr, nullptr, L.bqkv, m->qwen ? 0 : kBias, m->qkv,
                    m->QW, 0, nullptr, &io),
               "qkv");
        } else {
            CK(normed(L.wqkv, m->QW, false, L.ln1, L.ln1b, nk, src), "norm1");
            CK(gemv(L.wqkv, m->QW, src, C, R, nk, L.ln1, L.ln1b, L.bqkv, m->qwen ? 0 : kBias, m->qkv, m->QW, 0),
               "qkv");
        }
        if (dump(l, 2, m->qkv, m->QW)) return dumped == cudaSuccess ? NEKO_OK : fail(m, NEKO_ERR_CUDA, "dump");
        QkvPostArgs q;
        q.qkv = m->qkv;
        q.qkv_stride = m->QW;
        q.rows = R;
        q.n_head = H;
        q.n_kv = KV;
        q.hd = hd;
        q.do_norm = m->qwen;
        q.wn = L.qknorm;
        q.eps = eps;
        q.do_rope = m->qwen;
        q.cs = m->rope;
        q.store_kv = 1;
        q.kc = kc;
        q.vc = vc;
        q.slot_stride = m->kv_slot;
        q.pos_stride = hd;
        q.head_stride = m->kv_head;
        q.row_slot = m->d_slots;
        q.row_pos = m->d_pos;
        q.k_off = H * hd;
        q.v_off = (H + KV) * hd;
        q.pos_limit = m->cfg.context;
        q.write_back_k = staged ? 1 : 0;
        if (!fuse_post) CK(launch_qkv_post(q, st, pdl()), "qkv_post");
        if (m->qwen && dump(l, 3, m->qkv, m->QW)) return dumped == cudaSuccess ? NEKO_OK : fail(m, NEKO_ERR_CUDA, "dump");
        AttnArgs a;
        a.q = m->qkv;
        a.q_stride = m->QW;
        a.kc = kc;
        a.vc = vc;
        a.slot_stride = m->kv_slot;
        a.pos_stride = hd;
        a.head_stride = m->kv_head;
        a.row_slot = m->d_slots;
        a.row_pos = m->d_pos;
        a.rows = R;
        a.n_head = H;
        a.n_kv = KV;
        a.hd = hd;
        a.scale = 1.0f / std::sqrt(float(hd));
        a.out = m->att;
        a.out_stride = int64_t(H) * hd;
        a.max_pos = max_pos;
        a.pos_limit = m->cfg.context;
        a.part = m->part;
        a.tickets = m->tickets;
        a.part_capacity = m->part_cap;
        a.ticket_capacity = m->tick_cap;
        a.cache_rows = m->kv_layer / hd;
        if (chain) {
            a.out_hi = b_hi;
            a.out_lo = b_lo;
            a.out_hl_stride = int64_t(H) * hd;
        }
        if (fuse_post) {  // QK-norm, rotation and the cache store inside the attention kernel
            a.fuse_post = 1;
            a.post_wn = L.qknorm;
            a.post_cs = m->rope;
            a.post_eps = eps;
            a.k_off = H * hd;
            a.v_off = (H + KV) * hd;
        }
        CK(launch_attention(a, st, pdl()), "attention");
        if (dump(l, m->qwen ? 4 : 3, m->att, H * hd)) return dumped == cudaSuccess ? NEKO_OK : fail(m, NEKO_ERR_CUDA, "dump");
        if (chain) {
            // o_proj reads the attention's split output and writes x * ln2 + sums of squares for gate / up, whose
            // SwiGLU product (split) feeds down, which writes x * (next ln1 or the final norm) + sums of squares
            const ChainIO io_o{b_hi, b_lo, nullptr, a_hi, a_lo, C, L.ln2, m->ch_ss};
            CK(gemv(L.wo, C, m->att, int64_t(H) * hd, R, kNormNone, nullptr, nullptr, nullptr, kAccumulate, m->x, C,
                    0, nullptr, &io_o),
               "o_proj");
            const ChainIO io_gu{a_hi, a_lo, m->ch_ss, b_hi, b_lo, m->F, nullptr, nullptr};
            CK(gemv(L.wup, m->F, m->x, C, R, kNormNone, nullptr, nullptr, nullptr, 0, m->h, m->F, m->F, nullptr,
                    &io_gu),
               "gate_up");
            const float* g_next = l + 1 < m->layers.size() ? m->layers[l + 1].ln1 : m->normf;
            const ChainIO io_d{b_hi, b_lo, nullptr, a_hi, a_lo, C, g_next, m->ch_ss};
            CK(gemv(L.wdown, C, m->h, m->F, R, kNormNone, nullptr, nullptr, nullptr, kAccumulate, m->x, C, 0,
                    nullptr, &io_d),
               "down");
            continue;
        }
        CK(gemv(L.wo, C, m->att, int64_t(H) * hd, R, kNormNone, nullptr, nullptr, L.bo,
                kAccumulate | (m->qwen ? 0 : kBias), m->x, C, 0),
           "o_proj");
        if (dump(l, m->qwen ? 5 : 4, m->x, C)) return dumped == cudaSuccess ? NEKO_OK : fail(m, NEKO_ERR_CUDA, "dump");
        CK(normed(L.wup, m->qwen ? m->F : m->UPW, m->qwen, L.ln2, L.ln2b, nk, src), "norm2");
        if (m->qwen) {
            CK(gemv(L.wup, m->F, src, C, R, nk, L.ln2, nullptr, nullptr, 0, m->h, m->F, m->F), "gate_up");
        } else {
            CK(gemv(L.wup, m->UPW, src, C, R, nk, L.ln2, L.ln2b, L.bup, kBias | kGelu, m->h, m->UPW, 0), "fc");
        }
        if (dump(l, m->qwen ? 8 : 6, m->h, m->F)) return dumped == cudaSuccess ? NEKO_OK : fail(m, NEKO_ERR_CUDA, "dump");
        CK(gemv(L.wdown, C, m->h, m->F, R, kNormNone, nullptr, nullptr, L.bdown, kAccumulate | (m->qwen ? 0 : kBias),
                m->x, C, 0),
           "down");
        if (dump(l, m->qwen ? 9 : 7, m->x, C)) return dumped == cudaSuccess ? NEKO_OK : fail(m, NEKO_ERR_CUDA, "dump");
    }
    if (m->debug_layers >= 0) {  // hidden states of every row instead of logits
        CK(cudaMemcpyAsync(m->logits, m->x, size_t(R) * C * 4, cudaMemcpyDeviceToDevice, st), "debug copy");
        return NEKO_OK;
    }
    // final norm + LM head on the output rows
    const float* hx;
    if (outrows_identity && nout == R) {
        hx = m->x;
    } else if (outrows_identity && nout == 1) {
        hx = m->x + int64_t(R - 1) * C;
    } else {
        gather_rows_kernel<<<dim3((C + 255) / 256, nout), 256, 0, st>>>(m->x, C, m->d_outrows, nout, m->hx);
        first = false;
        CK(cudaGetLastError(), "gather");
        hx = m->hx;
    }
    const bool head_fits = gemv_norm_fusable(m->embed.fmt, nout, C) ||
                           gemm_tc_launches(m->embed.fmt, m->V, C, nout, false, true) > 0;
    const bool fused_argmax = do_argmax && nout <= 64;
    unsigned long long* keys = fused_argmax ? m->d_keys : nullptr;
    if (chain && outrows_identity && nout == R && chain_head_ok(m, R)) {  // x * normf split by the last down
        const ChainIO io{a_hi, a_lo, m->ch_ss, nullptr, nullptr, 0, nullptr, nullptr};
        CK(gemv(m->embed, m->V, m->x, C, nout, kNormNone, nullptr, nullptr, nullptr, 0, m->logits, m->V, 0, keys, &io),
           "lm_head");
    } else if (head_fits) {
        CK(gemv(m->embed, m->V, hx, C, nout, m->qwen ? kNormRms : kNormLayer, m->normf, m->normfb, nullptr, 0,
                m->logits, m->V, 0, keys),
           "lm_head");
    } else {
        CK(launch_norm(hx, C, m->xn, C, m->normf, m->normfb, nout, C, eps, m->qwen, st, pdl()), "final norm");
        CK(gemv(m->embed, m->V, m->xn, C, nout, kNormNone, nullptr, nullptr, nullptr, 0, m->logits, m->V, 0, keys),
           "lm_head");
    }
    if (do_argmax && !fused_argmax) CK(launch_argmax(m->logits, m->V, nout, m->V, m->d_argmax, st, pdl()), "argmax");
    if (fused_argmax)
        CK(launch_ex(argmax_finalize_kernel, dim3((nout + 127) / 128), dim3(128), 0, st, pdl(), m->d_keys,
                     m->d_argmax, m->d_tokens, m->d_pos, nout, m->cfg.context, advance ? 1 : 0),
           "argmax finalize");
    else if (advance)
        CK(launch_ex(advance_kernel, dim3((nout + 127) / 128), dim3(128), 0, st, pdl(), m->d_argmax, m->d_tokens,
                     m->d_pos, nout, m->cfg.context),
           "advance");
    return NEKO_OK;
}

bool fill_decode(neko_model* m, int R, int bucket, bool advance, DecodeParams& p, std::string* why);
bool head_split_ok(const neko_model* m, int R);

// Whether decode steps of R sequences can run as the single kernel (planned once per R).
bool decode_ok(neko_model* m, int R) {
    if (R < 1 || R > kDecodeMaxSeqs) return false;
    if (m->dec_ok[R] < 0) {
        DecodeParams dp;
        std::string why;
        m->dec_ok[R] = fill_decode(m, R, bucket_for(m, 0), false, dp, &why) ? 1 : 0;
        if (!m->dec_ok[R]) m->err = "decode kernel not used for " + std::to_string(R) + " sequences: " + why;
    }
    return m->dec_ok[R] == 1;
}

// The matmuls of a step (format, output rows, K, SwiGLU pair), the LM head last.
struct MatShape {
    int fmt, rows, K;
    bool pair, norm, lm_head;
};
std::vector<MatShape> mat_shapes(const neko_model* m) {
    const int K_att = m->H * m->hd;
    std::vector<MatShape> v = {{fmt_for(m->C, m->fmt), m->QW, m->C, false, true, false},
                               {fmt_for(K_att, m->fmt), m->C, K_att, false, false, false},
                               {fmt_for(m->C, m->fmt), m->qwen ? m->F : m->UPW, m->C, m->qwen, true, false},
                               {fmt_for(m->F, m->fmt), m->C, m->F, false, false, false},
                               {m->embed.fmt, m->V, m->C, false, true, true}};
    return v;
}

// Launches of one matmul of the step and of its norm: into the matmul call (GEMV prologue or the tensor-core
// path's split) when x_fits or the tensor-core path takes it, else a norm kernel first.
int matmul_launches(const MatShape& ms, int M, bool x_fits) {
    if (ms.norm) {
        const int tcn = gemm_tc_launches(ms.fmt, ms.rows, ms.K, M, ms.pair, true);
        if (tcn > 0) return tcn;
        if (x_fits) return 1;
        const int tc = gemm_tc_launches(ms.fmt, ms.rows, ms.K, M, ms.pair, false);
        return 1 + (tc > 0 ? tc : 1);
    }
    const int tc = gemm_tc_launches(ms.fmt, ms.rows, ms.K, M, ms.pair, false);
    return tc > 0 ? tc : 1;
}

bool chain_ok(const neko_model* m, int R) {
    if (!m->qwen || !m->ch_a || R < 5 || R > std::min(kChainMaxRows, m->ch_rows) || m->C % kChainTile) return false;
    if ((m->hd != 64 && m->hd != 128) || m->KV <= 0 || m->H % m->KV || m->H / m->KV > 8) return false;
    for (const MatShape& ms : mat_shapes(m))
        if (!ms.lm_head && gemm_tc_launches(ms.fmt, ms.rows, ms.K, R, ms.pair, false) <= 0) return false;
    return true;
}

bool chain_head_ok(const neko_model* m, int R) {
    return gemm_tc_launches(m->embed.fmt, m->V, m->C, R, false, false) > 0;
}

int step_launches(neko_model* m, int R, int nout, bool gather, bool do_argmax, bool advance) {
    if (!gather && nout == R && m->debug_layers < 0 && m->dec_enabled && R <= m->dec_seqs && decode_ok(m, R))
        return head_split_ok(m, R) ? 2 : 1;  // the decode kernel (+ the LM head, which finalizes the tokens)
    if (m->debug_layers < 0 && chain_ok(m, R)) {
        // embedding, the first layer's norm split + qkv, then per layer qkv_post, attention, o_proj, gate / up,
        // down and (after the first) qkv
        const MatShape q = mat_shapes(m)[0];
        const int nl = int(m->layers.size());
        // (qkv_post folded into attention on decode steps: every row its own slot, all rows output)
        const bool fused = !gather && nout == R;
        int n = 1 + gemm_tc_launches(q.fmt, q.rows, q.K, R, false, true) + (fused ? 4 : 5) * nl + (nl - 1) +
                (gather ? 1 : 0);
        if (!gather && nout == R && chain_head_ok(m, R)) n += 1;
        else n += matmul_launches(mat_shapes(m).back(), nout, gemv_norm_fusable(m->embed.fmt, nout, m->C));
        return n + (do_argmax ? 1 : 0) + (advance && nout > 64 ? 1 : 0);
    }
    const bool x_fits = gemv_norm_fusable(fmt_for(m->C, m->fmt), R, m->C);
    int per_layer = 2;  // qkv_post, attention
    for (const MatShape& ms : mat_shapes(m))
        if (!ms.lm_head) per_layer += matmul_launches(ms, R, x_fits);
    int n = 1 + int(m->layers.size()) * per_layer + (gather ? 1 : 0);
    for (const MatShape& ms : mat_shapes(m))
        if (ms.lm_head) n += matmul_launches(ms, nout, gemv_norm_fusable(m->embed.fmt, nout, m->C));
    return n + (do_argmax ? 1 : 0) + (advance && nout > 64 ? 1 : 0);
}

// Parameters of the single-kernel decode step for R sequences (tokens / slots / positions in the device arrays);
// false when the model or the step does not fit that kernel.
// The LM head of a single-kernel decode step as a launch of its own: the direct-load tensor-core GEMV streams the
// head at about twice the rate of the in-kernel phase (FP8 heads that it takes: C a multiple of 128).
bool head_split_ok(const neko_model* m, int R) {
    return m->embed.fmt == kFP8 && R <= kDecodeMaxSeqs && m->C % 128 == 0 && m->embed.rb % 16 == 0;
}

bool fill_decode(neko_model* m, int R, int bucket, bool advance, DecodeParams& p, std::string* why) {
    if (!m->dec_enabled || R < 1 || R > m->dec_seqs || size_t(m->layers.size()) > size_t(kDecodeMaxLayers)) {
        if (why) *why = "disabled or too many sequences / layers";
        return false;
    }
    const Layer& L0 = m->layers[0];
    const int f = m->fmt;
    if (m->embed.fmt != f || L0.wqkv.fmt != f || L0.wo.fmt != f || L0.wup.fmt != f || L0.wdown.fmt != f) {
        if (why) *why = "f16 matrices";
        return false;
    }
    p.M = R;
    p.qwen = m->qwen ? 1 : 0;
    p.fmt = f;
    p.layers = int(m->layers.size());
    p.C = m->C;
    p.H = m->H;
    p.KV = m->KV;
    p.hd = m->hd;
    p.F = m->F;
    p.V = m->V;
    p.QW = m->QW;
    p.context = m->cfg.context;
    p.rb_c = L0.wqkv.rb;
    p.rb_att = L0.wo.rb;
    p.rb_f = L0.wdown.rb;
    p.eps = m->cfg.eps;
    p.scale = 1.0f / std::sqrt(float(m->hd));
    p.embed = m->embed.w;
    p.normf = m->normf;
    p.normfb = m->normfb;
    p.rope = m->rope;
    p.wpe = m->wpe;
    p.kv_slot = m->kv_slot;
    p.kv_head = m->kv_head;
    {
        auto pad = [](int64_t w) { return (w + 31) / 32 * 32; };
        const DecodeScratch& z = m->dec_sz;
        uint64_t* b = m->dec_tw;
        p.x_tw = b;
        p.qkv_tw = b += pad(z.x_words);
        p.att_tw = b += pad(z.qkv_words);
        p.h_tw = b += pad(z.att_words);
        p.part_tw = b += pad(z.h_words);
    }
    p.epoch = m->dec_sync + 1;
    p.logits = m->logits;
    p.x_final = head_split_ok(m, R) ? m->x : nullptr;  // m->x is free during single-kernel steps
    p.tokens = m->d_tokens;
    p.slots = m->d_slots;
    p.pos = m->d_pos;
    p.argmax = m->d_argmax;
    p.keys = m->d_keys;
    p.advance = advance ? 1 : 0;
    p.sync = m->dec_sync;
    // keys per attention item: the bound the kernel's buffers are sized for; each step the kernel takes the
    // smallest multiple of 32 up to it whose items fit one per CTA (bucket unused)
    (void)bucket;
    p.span = 64;
    p.max_splits = m->dec_max_splits;
    if (m->dec_stall_test) {
        p.stall_test = 1;
        p.wait_ns = 50000000ull;
    }
    for (size_t l = 0; l < m->layers.size(); l++) {
        const Layer& L = m->layers[l];
        DecodeLayer& d = p.layer[l];
        d.wqkv = L.wqkv.w;
        d.wo = L.wo.w;
        d.wup = L.wup.w;
        d.wdown = L.wdown.w;
        d.ln1 = L.ln1;
        d.ln2 = L.ln2;
        d.ln1b = L.ln1b;
        d.ln2b = L.ln2b;
        d.qknorm = L.qknorm;
        d.bqkv = L.bqkv;
        d.bo = L.bo;
        d.bup = L.bup;
        d.bdown = L.bdown;
        d.kc = m->kc + int64_t(l) * m->kv_layer;
        d.vc = m->vc + int64_t(l) * m->kv_layer;
    }
    return plan_decode(p, why);
}

// Runs (capturing on first use) the graph of one step shape.
int run_step(neko_model* m, int R, int nout, bool identity, int max_pos, bool do_argmax, bool advance, cudaStream_t st) {
    const int bucket = bucket_for(m, max_pos);
    const bool single = m->dec_enabled && m->debug_layers < 0 && identity && nout == R && R <= m->dec_seqs &&
                        decode_ok(m, R);
    const int mode = (identity ? 1 : 0) | (do_argmax ? 2 : 0) | (advance ? 4 : 0) | (single ? 1 << 24 : 0) |
                     (single && m->dec_stall_test ? 1 << 25 : 0) |
                     (m->debug_layers >= 0 ? (8 + (m->debug_layers << 4) + (m->debug_stage << 12)) : 0);
    auto key = std::make_tuple(R, nout, bucket, mode);
    auto it = m->graphs.find(key);
    if (it == m->graphs.end()) {
        cudaStream_t cap = nullptr;
        CK(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking), "capture stream");
        cudaGraph_t g = nullptr;
        cudaError_t e = cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) {
            cudaStreamDestroy(cap);
            return fail(m, NEKO_ERR_CUDA, cuda_msg(e, "begin capture"));
        }
        int rc = NEKO_OK;
        DecodeParams dp;
        std::string why;
        if (single && !fill_decode(m, R, bucket, advance, dp, &why))
            rc = fail(m, NEKO_ERR_CUDA, "decode kernel plan: " + why);
        else if (single) {
            cudaError_t le = launch_decode(dp, cap);
            if (le == cudaSuccess && dp.x_final) {  // final norm + LM head + greedy argmax, then the token / position
                GemvArgs a;
                a.W = m->embed.w;
                a.row_bytes = m->embed.rb;
                a.rows = m->V;
                a.K = m->C;
                a.fmt = m->embed.fmt;
                a.x = dp.x_final;
                a.x_stride = m->C;
                a.M = R;
                a.norm = m->qwen ? kNormRms : kNormLayer;
                a.gamma = m->normf;
                a.beta = m->normfb;
                a.eps = m->cfg.eps;
                a.y = m->logits;
                a.y_stride = m->V;
                a.argmax = m->d_keys;
                a.fin_count = m->dec_sync + 2;  // its last CTA finalizes the greedy tokens
                a.fin_argmax = m->d_argmax;
                a.fin_tokens = m->d_tokens;
                a.fin_pos = m->d_pos;
                a.fin_context = m->cfg.context;
                a.fin_advance = advance ? 1 : 0;
                le = launch_gemv(a, cap, true);
            }
            if (le != cudaSuccess) rc = fail(m, NEKO_ERR_CUDA, cuda_msg(le, "decode kernel"));
        } else {
            rc = enqueue_step(m, R, nout, identity, bucket - 1, do_argmax, advance, cap);
        }
        e = cudaStreamEndCapture(cap, &g);
        cudaStreamDestroy(cap);
        if (rc != NEKO_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (e != cudaSuccess) return fail(m, NEKO_ERR_CUDA, cuda_msg(e, "end capture"));
        // kernel nodes of the step (checked against neko_model_step_launches by the tests)
        size_t nn = 0;
        m->graph_kernels = 0;
        if (cudaGraphGetNodes(g, nullptr, &nn) == cudaSuccess && nn > 0) {
            std::vector<cudaGraphNode_t> nodes(nn);
            if (cudaGraphGetNodes(g, nodes.data(), &nn) == cudaSuccess)
                for (size_t i = 0; i < nn; i++) {
                    cudaGraphNodeType t;
                    if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel)
                        m->graph_kernels++;
                }
        }
        cudaGraphExec_t ex = nullptr;
        e = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return fail(m, NEKO_ERR_CUDA, cuda_msg(e, "instantiate"));
        it = m->graphs.emplace(key, ex).first;
    }
    CK(cudaGraphLaunch(it->second, st), "graph launch");
    return NEKO_OK;
}

// floats per row that a debug dump holds (debugStages widths, qwen3_model.cpp:80-85, gpt2_model.cpp:61-64)
int debug_width(const neko_model* m) {
    switch (m->debug_stage) {
        case 2: case 3: return m->qwen || m->debug_stage == 2 ? m->QW : m->H * m->hd;
        case 4: return m->qwen ? m->H * m->hd : m->C;
        case 6: return m->qwen ? m->C : m->F;
        case 8: return m->F;
        default: return m->C;
    }
}

// After a device error the single-kernel step may have stopped between its phases (its epoch not advanced, some
// exchange words written under its tags): clear the exchange buffers, the step counter, the argmax keys and the
// abort flag, and restart the epoch, so the next step starts clean.
void decode_reset(neko_model* m) {
    if (m->dec_tw) cudaMemset(m->dec_tw, 0, size_t(m->dec_tw_words) * 8);
    if (m->dec_sync) {
        const unsigned init[4] = {0u, 1u, 0u, 0u};
        cudaMemcpy(m->dec_sync, init, sizeof(init), cudaMemcpyHostToDevice);
    }
    cudaMemset(m->d_keys, 0, size_t(std::max(m->cfg.max_rows, m->cfg.max_seqs)) * sizeof(unsigned long long));
    decode_clear_abort();
    cudaDeviceSynchronize();
}

int wait_model(neko_model* m) {
    // the error flag rides on the step's own stream and synchronisation (no second blocking copy per step)
    *m->h_err = 0;
    cudaError_t e = enqueue_device_error_read(m->h_err, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return fail(m, NEKO_ERR_CUDA, cuda_msg(e, "step"));
    if (*reinterpret_cast<volatile unsigned*>(m->h_err) == 0) return NEKO_OK;
    if (unsigned d = read_device_error(true)) {
        decode_reset(m);
        return fail(m, NEKO_ERR_DEVICE, "kernel reported device error " + std::to_string(d));
    }
    return NEKO_OK;
}

bool parse_layer(const std::string& n, const char* prefix, int& layer, std::string& leaf) {
    const size_t pl = std::strlen(prefix);
    if (n.compare(0, pl, prefix) != 0) return false;
    size_t dot = n.find('.', pl);
    if (dot == std::string::npos) return false;
    try {
        layer = std::stoi(n.substr(pl, dot - pl));
    } catch (...) {
        return false;
    }
    leaf = n.substr(dot + 1);
    return true;
}

}  // namespace

extern "C" {

const char* neko_model_last_error(neko_model* m) { return m ? m->err.c_str() : t_model_err.c_str(); }

neko_model* neko_model_create(int device, const neko_model_config* cfg, char* err, size_t err_len) {
    auto bail = [&](neko_model* m, const std::string& msg) -> neko_model* {
        t_model_err = msg;
        if (err && err_len) std::snprintf(err, err_len, "%s", msg.c_str());
        if (m) neko_model_destroy(m);
        return nullptr;
    };
    if (!cfg) return bail(nullptr, "null config");
    const neko_model_config& c = *cfg;
    if (c.arch != NEKO_ARCH_GPT2 && c.arch != NEKO_ARCH_QWEN3) return bail(nullptr, "unknown architecture");
    if (c.vocab <= 0 || c.embd <= 0 || c.layers <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.heads % c.kv_heads ||
        c.head_dim <= 0 || c.head_dim > 256 || (c.head_dim & 7) || c.ff <= 0 || c.context <= 0 || c.max_seqs <= 0 ||
        c.max_rows <= 0 || c.context > c.max_pos || c.weight_format < 0 || c.weight_format > 2)
        return bail(nullptr, "invalid model config");
    if (c.heads / c.kv_heads > 8) return bail(nullptr, "at most 8 query heads per KV head");
    if (c.embd % 8 || c.ff % 8) return bail(nullptr, "embd and ff must be multiples of 8");
    auto* m = new (std::nothrow) neko_model;
    if (!m) return bail(nullptr, "out of host memory");
    m->cfg = c;
    m->device = device;
    m->qwen = c.arch == NEKO_ARCH_QWEN3;
    m->C = c.embd;
    m->H = c.heads;
    m->KV = m->qwen ? c.kv_heads : c.heads;
    m->hd = m->qwen ? c.head_dim : c.embd / c.heads;
    if (!m->qwen && m->hd * c.heads != c.embd) return bail(m, "GPT-2 embd must equal heads * head_dim");
    m->F = c.ff;
    m->V = c.vocab;
    m->fmt = c.weight_format;
    m->QW = (m->H + 2 * m->KV) * m->hd;
    m->UPW = m->qwen ? 2 * c.ff : c.ff;
    m->layers.resize(size_t(c.layers));
    Guard g(device);
    cudaError_t e;
    if ((e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking)) != cudaSuccess)
        return bail(m, cuda_msg(e, "stream"));
    Carver size_pass{m, false};
    carve(m, size_pass);
    m->wbytes = size_pass.off;
    if ((e = cudaMalloc(&m->warena, m->wbytes)) != cudaSuccess) return bail(m, cuda_msg(e, "weights"));
    Carver assign{m, true};
    carve(m, assign);
    // KV cache [layer][slot][kv head][pos][hd]
    m->kv_head = int64_t(c.context) * m->hd;
    m->kv_slot = m->kv_head * m->KV;
    m->kv_layer = m->kv_slot * c.max_seqs;
    m->kv_bytes = size_t(m->kv_layer) * c.layers * 2;
    if ((e = cudaMalloc(&m->kc, m->kv_bytes)) != cudaSuccess) return bail(m, cuda_msg(e, "k cache"));
    if ((e = cudaMalloc(&m->vc, m->kv_bytes)) != cudaSuccess) return bail(m, cuda_msg(e, "v cache"));
    cudaMemset(m->kc, 0, m->kv_bytes);
    cudaMemset(m->vc, 0, m->kv_bytes);
    // workspace
    const size_t R = size_t(c.max_rows), nout = std::max<size_t>(R, size_t(c.max_seqs));
    auto falloc = [&](float** p, size_t n) {
        m->work_bytes += n * 4;
        return cudaMalloc(p, std::max<size_t>(n, 1) * 4);
    };
    auto ialloc = [&](int** p, size_t n) {
        m->work_bytes += n * 4;
        return cudaMalloc(p, std::max<size_t>(n, 1) * 4);
    };
    if (falloc(&m->x, R * m->C) || falloc(&m->xn, nout * m->C) || falloc(&m->qkv, R * m->QW) ||
        falloc(&m->att, R * m->H * m->hd) || falloc(&m->h, R * std::max(m->F, m->UPW)) || falloc(&m->hx, nout * m->C) ||
        falloc(&m->logits, nout * size_t(m->V)) || ialloc(&m->d_tokens, 3 * nout) ||
        ialloc(&m->d_argmax, nout) || ialloc(&m->d_outrows, nout) ||
        cudaMalloc(&m->d_keys, nout * sizeof(unsigned long long)) != cudaSuccess)
        return bail(m, "workspace allocation failed");
    cudaMemset(m->d_keys, 0, nout * sizeof(unsigned long long));
    // tokens | slots | positions in one block (nout apart), so a decode step's inputs arrive in one copy
    m->d_slots = m->d_tokens + nout;
    m->d_pos = m->d_tokens + 2 * nout;
    int64_t pf = 0, tk = 0;
    attention_scratch(int(R), m->H, m->KV, m->hd, c.context - 1, &pf, &tk, true);
    // fewer rows split more: size for the worst case over every row count 1..R
    for (int r = 1; r <= int(R); r++) {
        int64_t p2 = 0, t2 = 0;
        attention_scratch(r, m->H, m->KV, m->hd, c.context - 1, &p2, &t2, true);
        pf = std::max(pf, p2);
        tk = std::max(tk, t2);
    }
    m->part_cap = std::max<int64_t>(pf, 1);
    m->tick_cap = std::max<int64_t>(tk, 1);
    if (falloc(&m->part, size_t(m->part_cap)) || cudaMalloc(&m->tickets, size_t(m->tick_cap) * 4))
        return bail(m, "attention scratch allocation failed");
    cudaMemset(m->tickets, 0, size_t(m->tick_cap) * 4);
    // tensor-core matmul workspace: the largest any matmul asks for at any row count 5..max(R, seqs)
    {
        int64_t wf = 0, wt = 0;
        for (int r = 5; r <= int(nout); r++)
            for (const MatShape& ms : mat_shapes(m)) {
                if (!ms.lm_head && r > int(R)) continue;
                int64_t f = 0, t = 0;
                gemm_tc_scratch(ms.fmt, ms.rows, ms.K, r, ms.pair, ms.norm, &f, &t);
                wf = std::max(wf, f);
                wt = std::max(wt, t);
            }
        m->mm_ws_floats = wf;
        m->mm_tickets_n = wt;
        if (wf > 0 && (falloc(&m->mm_ws, size_t(wf)) || cudaMalloc(&m->mm_tickets, size_t(std::max<int64_t>(wt, 1)) * 4)))
            return bail(m, "matmul workspace allocation failed");
        if (m->mm_tickets) cudaMemset(m->mm_tickets, 0, size_t(std::max<int64_t>(wt, 1)) * 4);
        m->work_bytes += size_t(wt) * 4;
    }
    // matmul chaining buffers (Qwen3)
    if (m->qwen) {
        m->ch_rows = int(std::min<size_t>(R, size_t(kChainMaxRows)));
        const int64_t bw = std::max<int64_t>(int64_t(m->H) * m->hd, m->F);
        const size_t na = size_t(2) * m->ch_rows * m->C, nb = size_t(2) * m->ch_rows * bw;
        const size_t nss = size_t(m->ch_rows) * ((m->C + kChainTile - 1) / kChainTile);
        if (cudaMalloc(&m->ch_a, na * 2) != cudaSuccess || cudaMalloc(&m->ch_b, nb * 2) != cudaSuccess ||
            falloc(&m->ch_ss, nss))
            return bail(m, "matmul chaining buffers allocation failed");
        m->work_bytes += (na + nb) * 2;
    }
    // single-kernel decode steps: exchange buffers sized for the most sequences a launch serves and split-KV
    // partials at the smallest span (32 keys); the step counter and the tag epoch (starting at 1, so the zeroed
    // buffers hold no tag a step waits for)
    m->dec_seqs = std::min({kDecodeMaxSeqs, c.max_rows, c.max_seqs});
    m->dec_max_splits = (c.context + 31) / 32;
    {
        DecodeParams dp;
        dp.M = m->dec_seqs;
        dp.C = m->C;
        dp.QW = m->QW;
        dp.F = m->qwen ? m->F : m->UPW;
        dp.H = m->H;
        dp.KV = m->KV;
        dp.hd = m->hd;
        dp.layers = c.layers;
        dp.max_splits = m->dec_max_splits;
        decode_scratch(dp, &m->dec_sz);
        const DecodeScratch& z = m->dec_sz;
        auto pad = [](int64_t w) { return (w + 31) / 32 * 32; };  // 256-byte aligned sections
        m->dec_tw_words = pad(z.x_words) + pad(z.qkv_words) + pad(z.att_words) + pad(z.h_words) + pad(z.part_words);
        if (cudaMalloc(&m->dec_tw, size_t(m->dec_tw_words) * 8) != cudaSuccess ||
            cudaMalloc(&m->dec_sync, 4 * sizeof(unsigned)) != cudaSuccess)
            return bail(m, "decode exchange buffers allocation failed");
        m->work_bytes += size_t(m->dec_tw_words) * 8 + 16;
        cudaMemset(m->dec_tw, 0, size_t(m->dec_tw_words) * 8);
        const unsigned init[4] = {0u, 1u, 0u, 0u};
        cudaMemcpy(m->dec_sync, init, sizeof(init), cudaMemcpyHostToDevice);
    }
    m->h_logits_floats = nout * size_t(m->V);
    if (cudaMallocHost(&m->h_in, 4 * nout * sizeof(int)) || cudaMallocHost(&m->h_logits, nout * size_t(m->V) * 4) ||
        cudaMallocHost(&m->h_argmax, nout * sizeof(int)) || cudaMallocHost(&m->h_err, sizeof(unsigned)))
        return bail(m, "pinned host allocation failed");
    if (m->qwen) {
        std::vector<float> t = rope_table(c.context, m->hd, c.rope_theta);
        if ((e = cudaMemcpy(m->rope, t.data(), t.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess)
            return bail(m, cuda_msg(e, "rope table"));
    }
    // names every tensor must provide
    if (m->qwen) {
        m->need = {"embed_tokens.weight", "norm.weight"};
        for (int l = 0; l < c.layers; l++)
            for (const char* leaf : {"input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_norm.weight",
                                     "self_attn.k_norm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
                                     "self_attn.v_proj.weight", "self_attn.o_proj.weight", "mlp.gate_proj.weight",
                                     "mlp.up_proj.weight", "mlp.down_proj.weight"})
                m->need.insert("layers." + std::to_string(l) + "." + leaf);
    } else {
        m->need = {"wte.weight", "wpe.weight", "ln_f.weight", "ln_f.bias"};
        for (int l = 0; l < c.layers; l++)
            for (const char* leaf : {"ln_1.weight", "ln_1.bias", "ln_2.weight", "ln_2.bias", "attn.c_attn.weight",
                                     "attn.c_attn.bias", "attn.c_proj.weight", "attn.c_proj.bias", "mlp.c_fc.weight",
                                     "mlp.c_fc.bias", "mlp.c_proj.weight", "mlp.c_proj.bias"})
                m->need.insert("h." + std::to_string(l) + "." + leaf);
    }
    if ((e = cudaDeviceSynchronize()) != cudaSuccess) return bail(m, cuda_msg(e, "init"));
    return m;
}

void neko_model_destroy(neko_model* m) {
    if (!m) return;
    Guard g(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
    for (void* p : {(void*)m->warena, (void*)m->kc, (void*)m->vc, (void*)m->x, (void*)m->xn, (void*)m->qkv,
                    (void*)m->att, (void*)m->h, (void*)m->hx, (void*)m->logits, (void*)m->d_tokens,
                    (void*)m->d_argmax, (void*)m->d_outrows, (void*)m->d_keys, (void*)m->part,
                    (void*)m->tickets, (void*)m->mm_ws, (void*)m->mm_tickets, (void*)m->dec_tw, (void*)m->dec_sync,
                    (void*)m->ch_a, (void*)m->ch_b, (void*)m->ch_ss,
                    (void*)m->staging, (void*)m->staging8, (void*)m->d_track})
        if (p) cudaFree(p);
    if (m->h_in) cudaFreeHost(m->h_in);
    if (m->h_logits) cudaFreeHost(m->h_logits);
    if (m->h_argmax) cudaFreeHost(m->h_argmax);
    if (m->h_err) cudaFreeHost(m->h_err);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

static int set_tensor(neko_model* m, const char* cname, const float* data, int64_t rows, int64_t cols, bool on_device) {
    if (!m || !cname || !data || rows <= 0 || cols <= 0) return fail(m, NEKO_ERR_ARG, "set_tensor: bad arguments");
    Guard g(m->device);
    std::string name(cname);
    for (const char* pre : {"model.", "transformer."})
        if (name.compare(0, std::strlen(pre), pre) == 0) name = name.substr(std::strlen(pre));
    const int C = m->C, hd = m->hd;
    // destination: a matrix row range (quantized) or an f32 vector
    Mat* mat = nullptr;
    int row0 = 0, exp_rows = 0, exp_cols = 0;
    bool transpose = false;
    float* vec = nullptr;
    size_t vec_n = 0;
    int layer = -1;
    std::string leaf;
    if (m->qwen) {
        if (name == "embed_tokens.weight") {
            mat = &m->embed, exp_rows = m->V, exp_cols = C;
        } else if (name == "norm.weight") {
            vec = m->normf, vec_n = C;
        } else if (parse_layer(name, "layers.", layer, leaf) && layer < int(m->layers.size())) {
            Layer& L = m->layers[size_t(layer)];
            const int qh = m->H * hd, kvw = m->KV * hd;
            if (leaf == "input_layernorm.weight") vec = L.ln1, vec_n = C;
            else if (leaf == "post_attention_layernorm.weight") vec = L.ln2, vec_n = C;
            else if (leaf == "self_attn.q_norm.weight") vec = L.qknorm, vec_n = hd;
            else if (leaf == "self_attn.k_norm.weight") vec = L.qknorm + hd, vec_n = hd;
            else if (leaf == "self_attn.q_proj.weight") mat = &L.wqkv, row0 = 0, exp_rows = qh, exp_cols = C;
            else if (leaf == "self_attn.k_proj.weight") mat = &L.wqkv, row0 = qh, exp_rows = kvw, exp_cols = C;
            else if (leaf == "self_attn.v_proj.weight") mat = &L.wqkv, row0 = qh + kvw, exp_rows = kvw, exp_cols = C;
            else if (leaf == "self_attn.o_proj.weight") mat = &L.wo, exp_rows = C, exp_cols = qh;
            else if (leaf == "mlp.gate_proj.weight") mat = &L.wup, row0 = 0, exp_rows = m->F, exp_cols = C;
            else if (leaf == "mlp.up_proj.weight") mat = &L.wup, row0 = m->F, exp_rows = m->F, exp_cols = C;
            else if (leaf == "mlp.down_proj.weight") mat = &L.wdown, exp_rows = C, exp_cols = m->F;
        }
    } else {
        if (name == "wte.weight") {
            mat = &m->embed, exp_rows = m->V, exp_cols = C;
        } else if (name == "wpe.weight") {
            vec = m->wpe, vec_n = size_t(m->cfg.max_pos) * C;
        } else if (name == "ln_f.weight") {
            vec = m->normf, vec_n = C;
        } else if (name == "ln_f.bias") {
            vec = m->normfb, vec_n = C;
        } else if (parse_layer(name, "h.", layer, leaf) && layer < int(m->layers.size())) {
            Layer& L = m->layers[size_t(layer)];
            // Conv1D weights are stored [in][out]; the engine transposes them and rounds to f16 first.
            if (leaf == "ln_1.weight") vec = L.ln1, vec_n = C;
            else if (leaf == "ln_1.bias") vec = L.ln1b, vec_n = C;
            else if (leaf == "ln_2.weight") vec = L.ln2, vec_n = C;
            else if (leaf == "ln_2.bias") vec = L.ln2b, vec_n = C;
            else if (leaf == "attn.c_attn.weight") mat = &L.wqkv, exp_rows = C, exp_cols = 3 * C, transpose = true;
            else if (leaf == "attn.c_attn.bias") vec = L.bqkv, vec_n = 3 * size_t(C);
            else if (leaf == "attn.c_proj.weight") mat = &L.wo, exp_rows = C, exp_cols = C, transpose = true;
            else if (leaf == "attn.c_proj.bias") vec = L.bo, vec_n = C;
            else if (leaf == "mlp.c_fc.weight") mat = &L.wup, exp_rows = C, exp_cols = m->UPW, transpose = true;
            else if (leaf == "mlp.c_fc.bias") vec = L.bup, vec_n = size_t(m->UPW);
            else if (leaf == "mlp.c_proj.weight") mat = &L.wdown, exp_rows = m->F, exp_cols = C, transpose = true;
            else if (leaf == "mlp.c_proj.bias") vec = L.bdown, vec_n = C;
            else if (leaf == "attn.bias" || leaf == "attn.masked_bias") return NEKO_OK;  // causal-mask buffers
        }
    }
    if (!mat && !vec) return fail(m, NEKO_ERR_ARG, "set_tensor: unknown tensor " + name);
    if (vec) {
        if (size_t(rows * cols) != vec_n) return fail(m, NEKO_ERR_ARG, "set_tensor: wrong size for " + name);
        // Stream-ordered copies only: a pageable cudaMemcpy may return before its DMA lands, and the model's
        // stream does not order itself after the legacy default stream.
        CK(cudaMemcpyAsync(vec, data, vec_n * 4, on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                           m->stream),
           "upload vector");
        CK(cudaStreamSynchronize(m->stream), "upload vector");
    } else {
        if (rows != exp_rows || cols != exp_cols)
            return fail(m, NEKO_ERR_ARG, "set_tensor: wrong shape for " + name + " (" + std::to_string(rows) + "x" +
                                             std::to_string(cols) + ")");
        const size_t n = size_t(rows) * size_t(cols);
        const float* src = data;
        if (!on_device) {
            if (n > m->staging_floats) {
                cudaFree(m->staging);
                m->staging = nullptr;
                CK(cudaMalloc(&m->staging, n * 4), "staging");
                m->staging_floats = n;
            }
            CK(cudaMemcpyAsync(m->staging, data, n * 4, cudaMemcpyHostToDevice, m->stream), "upload matrix");
            src = m->staging;
        }
        // out rows / in cols of the packed matrix
        const int orows = transpose ? int(cols) : int(rows);
        const int icols = transpose ? int(rows) : int(cols);
        CK(launch_quantize(mat->fmt, src, orows, icols, cols, transpose ? 1 : 0,
                           mat->w + int64_t(row0) * mat->rb, m->stream),
           "quantize");
        CK(cudaStreamSynchronize(m->stream), "quantize");
    }
    m->have.insert(name);
    m->final_ok = false;
    return NEKO_OK;
}

}  // extern "C"

static int set_tensor_entry(neko_model* m, const char* name, const float* data, int64_t rows, int64_t cols,
                            bool on_device) {
    if (!m) return NEKO_ERR_ARG;
    Guard g(m->device);
    if (on_device) {
        // the runner's kernels read the tensor on its own device: memory of another device is refused here
        // (a kernel would fault on it without peer access)
        cudaPointerAttributes pa{};
        if (cudaPointerGetAttributes(&pa, data) != cudaSuccess || pa.type != cudaMemoryTypeDevice ||
            pa.device != m->device) {
            cudaGetLastError();
            return fail(m, NEKO_ERR_ARG, "set_tensor_device: the data is not device memory of the model's device " +
                                             std::to_string(m->device));
        }
        // device data may come from work on another stream (e.g. a framework's generator): let it finish first
        CK(cudaDeviceSynchronize(), "set_tensor_device");
    }
    return set_tensor(m, name, data, rows, cols, on_device);
}

extern "C" {

int neko_model_set_tensor(neko_model* m, const char* name, const float* data, int64_t rows, int64_t cols) {
    return set_tensor_entry(m, name, data, rows, cols, false);
}

int neko_model_set_tensor_device(neko_model* m, const char* name, const float* d_data, int64_t rows, int64_t cols) {
    return set_tensor_entry(m, name, d_data, rows, cols, true);
}

int neko_model_set_tensor_fp8(neko_model* m, const char* name, const uint8_t* codes, int64_t rows, int64_t cols,
                              const float* scales, int64_t scale_rows, int64_t scale_cols) {
    if (!m) return NEKO_ERR_ARG;
    if (!name || !codes || !scales || rows <= 0 || cols <= 0 || scale_rows < 1 || scale_cols < 1)
        return fail(m, NEKO_ERR_ARG, "set_tensor_fp8: bad argument");
    Guard g(m->device);
    const size_t n = size_t(rows) * size_t(cols), ns = size_t(scale_rows) * size_t(scale_cols);
    const size_t scale_off = (n + 255) & ~size_t(255);
    if (scale_off + ns * 4 > m->staging8_bytes) {
        CK(cudaStreamSynchronize(m->stream), "staging8");
        cudaFree(m->staging8);
        m->staging8 = nullptr;
        m->staging8_bytes = 0;
        CK(cudaMalloc(&m->staging8, scale_off + ns * 4), "staging8");
        m->staging8_bytes = scale_off + ns * 4;
    }
    if (n > m->staging_floats) {
        CK(cudaStreamSynchronize(m->stream), "staging");
        cudaFree(m->staging);
        m->staging = nullptr;
        m->staging_floats = 0;
        CK(cudaMalloc(&m->staging, n * 4), "staging");
        m->staging_floats = n;
    }
    float* d_scales = reinterpret_cast<float*>(m->staging8 + scale_off);
    CK(cudaMemcpyAsync(m->staging8, codes, n, cudaMemcpyHostToDevice, m->stream), "upload fp8 codes");
    CK(cudaMemcpyAsync(d_scales, scales, ns * 4, cudaMemcpyHostToDevice, m->stream), "upload fp8 scales");
    CK(launch_fp8_block_dequant(m->staging8, rows, cols, d_scales, scale_rows, scale_cols, m->staging, m->stream),
       "fp8 dequant");
    // the f32 tensor is device memory of the model's device, ordered on its stream: the device-data path
    return set_tensor(m, name, m->staging, rows, cols, true);
}

int neko_model_finalize(neko_model* m) {
    if (!m) return NEKO_ERR_ARG;
    for (const auto& n : m->need)
        if (!m->have.count(n)) return fail(m, NEKO_ERR_ARG, "finalize: missing tensor " + n);
    m->final_ok = true;
    return NEKO_OK;
}

int neko_model_forward(neko_model* m, int slot, const int* tokens, int T, int pos0, float* logits) {
    if (!m || !tokens || !logits) return fail(m, NEKO_ERR_ARG, "forward: null argument");
    if (!m->final_ok) return fail(m, NEKO_ERR_ARG, "forward: call neko_model_finalize first");
    // Model::checkBatch (model.cpp:127-132)
    if (T <= 0 || T > m->cfg.max_rows) return fail(m, NEKO_ERR_ARG, "forward: bad batch size");
    if (pos0 < 0 || pos0 + T > m->cfg.context) return fail(m, NEKO_ERR_ARG, "forward: context overflow");
    if (slot < 0 || slot >= m->cfg.max_seqs) return fail(m, NEKO_ERR_ARG, "forward: bad slot");
    for (int t = 0; t < T; t++)
        if (tokens[t] < 0 || tokens[t] >= m->V) return fail(m, NEKO_ERR_ARG, "forward: token id out of range");
    Guard g(m->device);
    int* hi = m->h_in;
    for (int t = 0; t < T; t++) {
        hi[t] = tokens[t];
        hi[T + t] = slot;
        hi[2 * T + t] = pos0 + t;
    }
    CK(cudaMemcpyAsync(m->d_tokens, hi, size_t(T) * 4, cudaMemcpyHostToDevice, m->stream), "h2d");
    CK(cudaMemcpyAsync(m->d_slots, hi + T, size_t(T) * 4, cudaMemcpyHostToDevice, m->stream), "h2d");
    CK(cudaMemcpyAsync(m->d_pos, hi + 2 * T, size_t(T) * 4, cudaMemcpyHostToDevice, m->stream), "h2d");
    if (int rc = run_step(m, T, 1, true, pos0 + T - 1, false, false, m->stream); rc != NEKO_OK) return rc;
    const size_t nout = m->debug_layers >= 0 ? size_t(T) * size_t(debug_width(m)) : size_t(m->V);
    CK(cudaMemcpyAsync(m->h_logits, m->logits, nout * 4, cudaMemcpyDeviceToHost, m->stream), "d2h");
    if (int rc = wait_model(m); rc != NEKO_OK) return rc;
    if (logits != m->h_logits) std::memcpy(logits, m->h_logits, nout * 4);
    return NEKO_OK;
}

int neko_model_decode(neko_model* m, int n, const int* slots, const int* tokens, const int* pos, float* logits,
                      int* argmax) {
    if (!m || !slots || !tokens || !pos) return fail(m, NEKO_ERR_ARG, "decode: null argument");
    if (!m->final_ok) return fail(m, NEKO_ERR_ARG, "decode: call neko_model_finalize first");
    if (n <= 0 || n > m->cfg.max_rows || n > m->cfg.max_seqs) return fail(m, NEKO_ERR_ARG, "decode: bad count");
    int max_pos = 0;
    for (int i = 0; i < n; i++) {
        if (slots[i] < 0 || slots[i] >= m->cfg.max_seqs) return fail(m, NEKO_ERR_ARG, "decode: bad slot");
        if (pos[i] < 0 || pos[i] >= m->cfg.context) return fail(m, NEKO_ERR_ARG, "decode: context overflow");
        if (tokens[i] < 0 || tokens[i] >= m->V) return fail(m, NEKO_ERR_ARG, "decode: token id out of range");
        for (int j = 0; j < i; j++)
            if (slots[j] == slots[i]) return fail(m, NEKO_ERR_ARG, "decode: a slot appears twice in one step");
        max_pos = std::max(max_pos, pos[i]);
    }
    Guard g(m->device);
    // the device block's layout (tokens | slots | positions, nout apart) in the pinned staging: one copy
    const size_t nout = size_t(m->d_slots - m->d_tokens);
    int* hi = m->h_in;
    std::memcpy(hi, tokens, size_t(n) * 4);
    std::memcpy(hi + nout, slots, size_t(n) * 4);
    std::memcpy(hi + 2 * nout, pos, size_t(n) * 4);
    CK(cudaMemcpyAsync(m->d_tokens, hi, (2 * nout + size_t(n)) * 4, cudaMemcpyHostToDevice, m->stream), "h2d");
    if (int rc = run_step(m, n, n, true, max_pos, argmax != nullptr, false, m->stream); rc != NEKO_OK) return rc;
    if (logits)
        CK(cudaMemcpyAsync(m->h_logits, m->logits, size_t(n) * m->V * 4, cudaMemcpyDeviceToHost, m->stream), "d2h");
    if (argmax) CK(cudaMemcpyAsync(m->h_argmax, m->d_argmax, size_t(n) * 4, cudaMemcpyDeviceToHost, m->stream), "d2h");
    if (int rc = wait_model(m); rc != NEKO_OK) return rc;
    if (logits && logits != m->h_logits) std::memcpy(logits, m->h_logits, size_t(n) * m->V * 4);
    if (argmax) std::memcpy(argmax, m->h_argmax, size_t(n) * 4);
    return NEKO_OK;
}

int neko_model_stage(neko_model* m, int n, const int* slots, const int* tokens, const int* pos) {
    if (!m || !slots || !tokens || !pos) return fail(m, NEKO_ERR_ARG, "stage: null argument");
    if (n <= 0 || n > m->cfg.max_rows || n > m->cfg.max_seqs) return fail(m, NEKO_ERR_ARG, "stage: bad count");
    for (int i = 0; i < n; i++) {
        if (slots[i] < 0 || slots[i] >= m->cfg.max_seqs) return fail(m, NEKO_ERR_ARG, "stage: bad slot");
        if (pos[i] < 0 || pos[i] >= m->cfg.context) return fail(m, NEKO_ERR_ARG, "stage: context overflow");
        if (tokens[i] < 0 || tokens[i] >= m->V) return fail(m, NEKO_ERR_ARG, "stage: token id out of range");
        for (int j = 0; j < i; j++)
            if (slots[j] == slots[i]) return fail(m, NEKO_ERR_ARG, "stage: a slot appears twice");
    }
    Guard g(m->device);
    CK(cudaDeviceSynchronize(), "stage");  // no step may still be reading the arrays
    std::memcpy(m->h_in, tokens, size_t(n) * 4);
    std::memcpy(m->h_in + n, slots, size_t(n) * 4);
    std::memcpy(m->h_in + 2 * n, pos, size_t(n) * 4);
    CK(cudaMemcpyAsync(m->d_tokens, m->h_in, size_t(n) * 4, cudaMemcpyHostToDevice, m->stream), "stage");
    CK(cudaMemcpyAsync(m->d_slots, m->h_in + n, size_t(n) * 4, cudaMemcpyHostToDevice, m->stream), "stage");
    CK(cudaMemcpyAsync(m->d_pos, m->h_in + 2 * n, size_t(n) * 4, cudaMemcpyHostToDevice, m->stream), "stage");
    if (m->track_steps) {
        // the staged token is the engine's first sample (engine.cpp:121-124): a stop id ends the sequence before
        // any step, else it is the first logged token
        const size_t S = size_t(m->cfg.max_seqs);
        std::vector<int> cnt(S, 0), state(S, 0), frozen(2 * S, 0), first(S, 0);
        for (int i = 0; i < n; i++) {
            const bool stop = std::find(m->stop_ids.begin(), m->stop_ids.end(), tokens[i]) != m->stop_ids.end();
            cnt[i] = stop ? 0 : 1;
            state[i] = stop ? 1 : (m->track_steps <= 1 ? 0 : -1);
            frozen[2 * i] = tokens[i];
            frozen[2 * i + 1] = pos[i];
            first[i] = tokens[i];
        }
        int* t = m->d_track + NEKO_MAX_STOP_IDS;
        CK(cudaMemcpyAsync(t, cnt.data(), S * 4, cudaMemcpyHostToDevice, m->stream), "stage");
        CK(cudaMemcpyAsync(t + S, state.data(), S * 4, cudaMemcpyHostToDevice, m->stream), "stage");
        CK(cudaMemcpyAsync(t + 2 * S, frozen.data(), 2 * S * 4, cudaMemcpyHostToDevice, m->stream), "stage");
        CK(cudaMemcpyAsync(t + 4 * S, first.data(), S * 4, cudaMemcpyHostToDevice, m->stream), "stage");
    }
    CK(cudaStreamSynchronize(m->stream), "stage");
    return NEKO_OK;
}

int neko_model_step(neko_model* m, int n, int max_pos, void* stream) {
    if (!m) return NEKO_ERR_ARG;
    if (!m->final_ok) return fail(m, NEKO_ERR_ARG, "step: call neko_model_finalize first");
    if (n <= 0 || n > m->cfg.max_rows || n > m->cfg.max_seqs) return fail(m, NEKO_ERR_ARG, "step: bad count");
    if (max_pos < 0 || max_pos >= m->cfg.context) return fail(m, NEKO_ERR_ARG, "step: context overflow");
    Guard g(m->device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (const int rc = run_step(m, n, n, true, max_pos, true, true, st); rc != NEKO_OK || !m->track_steps) return rc;
    const int S = m->cfg.max_seqs;
    int* t = m->d_track;
    CK(launch_ex(track_kernel, dim3((n + 127) / 128), dim3(128), 0, st, false, m->d_tokens, m->d_pos, n, t,
                 int(m->stop_ids.size()), t + NEKO_MAX_STOP_IDS, t + NEKO_MAX_STOP_IDS + S,
                 t + NEKO_MAX_STOP_IDS + 2 * S, t + NEKO_MAX_STOP_IDS + 4 * S, m->track_steps, S),
       "track");
    return NEKO_OK;
}

float* neko_model_host_logits(neko_model* m, size_t* floats) {
    if (!m) return nullptr;
    if (floats) *floats = m->h_logits_floats;
    return m->h_logits;
}

int neko_model_set_stop(neko_model* m, const int* stop_ids, int n_stop, int max_new) {
    if (!m) return NEKO_ERR_ARG;
    if (n_stop < 0 || n_stop > NEKO_MAX_STOP_IDS || max_new < 0 || (n_stop > 0 && !stop_ids))
        return fail(m, NEKO_ERR_ARG, "set_stop: bad argument");
    for (int i = 0; i < n_stop; i++)
        if (stop_ids[i] < 0 || stop_ids[i] >= m->V) return fail(m, NEKO_ERR_ARG, "set_stop: stop id out of range");
    Guard g(m->device);
    CK(cudaDeviceSynchronize(), "set_stop");  // no step may still use the old arrays
    cudaFree(m->d_track);
    m->d_track = nullptr;
    m->track_steps = 0;
    m->stop_ids.clear();
    if (max_new == 0) return NEKO_OK;
    const size_t S = size_t(m->cfg.max_seqs);
    CK(cudaMalloc(&m->d_track, (NEKO_MAX_STOP_IDS + 4 * S + size_t(max_new) * S) * sizeof(int)), "set_stop");
    CK(cudaMemset(m->d_track, 0, (NEKO_MAX_STOP_IDS + 2 * S) * sizeof(int)), "set_stop");
    // every sequence counts as finished (reason 0, nothing logged, frozen at token 0 position 0) until staged
    CK(cudaMemset(m->d_track + NEKO_MAX_STOP_IDS + 2 * S, 0, 2 * S * sizeof(int)), "set_stop");
    m->stop_ids.assign(stop_ids, stop_ids + n_stop);
    if (n_stop)
        CK(cudaMemcpy(m->d_track, stop_ids, size_t(n_stop) * sizeof(int), cudaMemcpyHostToDevice), "set_stop");
    m->track_steps = max_new;
    return NEKO_OK;
}

int neko_model_generated(neko_model* m, int n, int* tokens, int* counts, int* reasons) {
    if (!m || n <= 0 || n > m->cfg.max_seqs) return NEKO_ERR_ARG;
    if (!m->track_steps) return fail(m, NEKO_ERR_ARG, "generated: call neko_model_set_stop first");
    Guard g(m->device);
    CK(cudaDeviceSynchronize(), "generated");
    if (unsigned d = read_device_error(true)) {
        decode_reset(m);
        return fail(m, NEKO_ERR_DEVICE, "kernel reported device error " + std::to_string(d));
    }
    const size_t S = size_t(m->cfg.max_seqs), L = size_t(m->track_steps);
    std::vector<int> h(4 * S + L * S);
    CK(cudaMemcpy(h.data(), m->d_track + NEKO_MAX_STOP_IDS, h.size() * sizeof(int), cudaMemcpyDeviceToHost),
       "generated");
    for (int i = 0; i < n; i++) {
        const int c = h[size_t(i)];
        if (counts) counts[i] = c;
        if (reasons) reasons[i] = h[S + size_t(i)];
        if (tokens)
            for (size_t j = 0; j < L; j++) tokens[size_t(i) * L + j] = int(j) < c ? h[4 * S + j * S + size_t(i)] : -1;
    }
    return NEKO_OK;
}

int neko_model_tokens(neko_model* m, int n, int* tokens, int* pos) {
    if (!m || n <= 0 || n > m->cfg.max_seqs) return NEKO_ERR_ARG;
    Guard g(m->device);
    CK(cudaDeviceSynchronize(), "tokens");
    if (unsigned d = read_device_error(true)) {
        decode_reset(m);
        return fail(m, NEKO_ERR_DEVICE, "kernel reported device error " + std::to_string(d));
    }
    if (tokens) CK(cudaMemcpyAsync(tokens, m->d_tokens, size_t(n) * 4, cudaMemcpyDeviceToHost, m->stream), "tokens");
    if (pos) CK(cudaMemcpyAsync(pos, m->d_pos, size_t(n) * 4, cudaMemcpyDeviceToHost, m->stream), "tokens");
    CK(cudaStreamSynchronize(m->stream), "tokens");
    return NEKO_OK;
}

int neko_model_set_debug(neko_model* m, int layers, int stage) {
    if (!m) return NEKO_ERR_ARG;
    // stages with a buffer of their own in the fused step (the others are fused into a neighbour)
    static const int qwen_ok[] = {2, 3, 4, 5, 8, 9}, gpt2_ok[] = {2, 3, 4, 6, 7};
    bool ok = stage == 0;
    for (int s : m->qwen ? std::vector<int>(qwen_ok, qwen_ok + 6) : std::vector<int>(gpt2_ok, gpt2_ok + 5))
        ok = ok || s == stage;
    if (!ok) return fail(m, NEKO_ERR_UNSUPPORTED, "set_debug: stage " + std::to_string(stage) + " is fused away");
    m->debug_layers = layers;
    m->debug_stage = layers >= 0 ? stage : 0;
    if (layers >= 0 && size_t(m->cfg.max_rows) * debug_width(m) > size_t(std::max(m->cfg.max_rows, m->cfg.max_seqs)) * m->V)
        return fail(m, NEKO_ERR_UNSUPPORTED, "set_debug: the dump does not fit the logits workspace");
    return NEKO_OK;
}

int neko_model_memory(neko_model* m, int64_t* weights, int64_t* kv, int64_t* workspace) {
    if (!m) return NEKO_ERR_ARG;
    if (weights) *weights = int64_t(m->wbytes);
    if (kv) *kv = int64_t(m->kv_bytes) * 2;
    if (workspace) *workspace = int64_t(m->work_bytes);
    return NEKO_OK;
}

int neko_model_set_decode_kernel(neko_model* m, int enable) {
    if (!m) return NEKO_ERR_ARG;
    Guard g(m->device);
    m->dec_enabled = enable != 0;
    m->dec_stall_test = enable == 2 ? 1 : 0;
    if (!m->dec_enabled) return 0;
    return decode_ok(m, 1) ? 1 : 0;
}

int neko_model_step_launches(neko_model* m, int n) {
    if (!m) return NEKO_ERR_ARG;
    return step_launches(m, n, n, false, true, true);
}

int neko_model_graph_kernels(neko_model* m) {
    if (!m) return NEKO_ERR_ARG;
    return m->graph_kernels;
}

int neko_model_matrix(neko_model* m, const char* which, const uint8_t** ptr, int* rows, int* cols) {
    if (!m || !which) return NEKO_ERR_ARG;
    std::string w(which);
    const Mat* t = nullptr;
    int layer = -1;
    std::string leaf;
    if (w == "head" || w == "embed") t = &m->embed;
    else if (parse_layer(w, "layers.", layer, leaf) && layer < int(m->layers.size())) {
        const Layer& L = m->layers[size_t(layer)];
        if (leaf == "wqkv") t = &L.wqkv;
        else if (leaf == "wo") t = &L.wo;
        else if (leaf == "wgu" || leaf == "wup") t = &L.wup;
        else if (leaf == "wdown") t = &L.wdown;
    }
    if (!t) return fail(m, NEKO_ERR_ARG, "matrix: unknown name " + w);
    if (ptr) *ptr = t->w;
    if (rows) *rows = t->rows;
    if (cols) *cols = t->cols;
    return t->fmt;
}

}  // extern "C"
