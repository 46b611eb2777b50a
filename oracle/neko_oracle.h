/* CPU restatement of NekoChat's hot-path arithmetic: the weight codec and the transformer ops.
 *
 * TEST INFRASTRUCTURE ONLY. The oracle is the checker for the B200 kernels (tests/, the smoke check and
 * the bench's CPU-baseline leg load it); no product code path may call it.
 *
 * Parity is pinned two ways: against golden vectors that the reference engine itself produced
 * (tests/golden/, made by tests/golden/make_golden.py from oracle/_ref/libneko_ref.so), and live against
 * that compiled reference in the CPU test suite. Each function names the reference code it restates
 * (paths relative to app/architecture/shared/cpp). Floating-point expressions keep the reference's
 * evaluation order and are compiled with -ffp-contract=off, so results are bit-identical to the
 * reference built the same way.
 */
#ifndef NEKO_ORACLE_H
#define NEKO_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { NO_F16 = 0, NO_FP8 = 1, NO_FP4 = 2 };  /* quant.h:19 WeightFormat */
enum { NO_GELU = 1, NO_ACCUMULATE = 2 };     /* cpu_ops.h:15 MatmulFlags */

uint16_t no_f32_to_f16(float f);  /* common.h:58-80, round to nearest even */
float no_f16_to_f32(uint16_t h);  /* common.h:33-55 */

size_t no_row_bytes(int fmt, int cols);                                   /* quant.cpp:199-208 */
void no_quantize_rows(int fmt, int rows, int cols, const float* w, uint8_t* out); /* quant.cpp:255-279 */
void no_dequantize_rows(int fmt, int rows, int cols, const uint8_t* data, float* out); /* quant.cpp:230-253 */

/* y[t][n] (+)= act(x[t] . W[n] + bias[n]); yStride is the row stride of y. cpu_ops.cpp:108-128, 442-458 */
void no_matmul(int fmt, const float* x, int T, int K, const uint8_t* W, int rows, const float* bias, float* y,
               int yStride, int flags);
void no_layer_norm(const float* x, float* y, const float* g, const float* b, int T, int C, float eps); /* :483-500 */
void no_rms_norm(const float* x, float* y, const float* w, int rows, int C, float eps);               /* :502-511 */
void no_rope(float* x, int nHeads, int hd, const float* cs);                                         /* :513-524 */
void no_silu_mul(const float* h, float* out, int T, int I);                                          /* :526-533 */
float no_gelu(float x);                                                                              /* :20-23 */
void no_store_kv(const float* k, const float* v, int srcStride, uint16_t* kc, uint16_t* vc, int width, int T,
                 int pos0);                                                                          /* :535-542 */
void no_attention(const float* q, int qStride, const uint16_t* kc, const uint16_t* vc, float* out, int T, int nHead,
                  int nKv, int hd, int pos0);                                                        /* :544-575 */
/* Row softmax: the reference has no kernel for it; this restates the softmax inside cpu::attention
 * (cpu_ops.cpp:556-572): max, exp(x - max), float sum, multiply by 1 / sum. */
void no_softmax_rows(const float* x, float* y, int rows, int C);
/* Qwen3 rotary table [pos][hd/2](cos, sin): qwen3/cpp/qwen3_model.cpp:102-114 */
void no_rope_table(int ctx, int hd, double theta, float* out);
/* Embedding rows: QMatrix::dequantizeRow of each token (qwen3_model.cpp:236), plus the f32 position row
 * for GPT-2 (gpt2_model.cpp:182-187) when wpe is not NULL. */
void no_embed(int fmt, const uint8_t* table, int cols, const int* tokens, int T, const float* wpe, int pos0, float* x);
/* Greedy sampling: index of the first maximum (sampler.cpp:24, std::max_element). */
int no_argmax(const float* x, int n);

#ifdef __cplusplus
}
#endif
#endif
