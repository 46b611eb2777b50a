/* CPU restatement of NekoChat's hot-path arithmetic. TEST INFRASTRUCTURE ONLY (see neko_oracle.h).
 * Compiled with -ffp-contract=off: each float expression below is rounded exactly as written, in the
 * reference's order. Paths are relative to app/architecture/shared/cpp. */
#include "neko_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define QBLOCK 32 /* quant.h:23 kQuantBlock */

static float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* IEEE binary16 -> binary32. Exact for every input (common.h:33-55). */
float no_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    int e = (h >> 10) & 31;
    uint32_t m = h & 1023u;
    if (e == 31) return bits_f(sign | 0x7f800000u | (m << 13));
    if (e == 0) {
        /* zero or subnormal: m * 2^-24, exact in binary32 */
        float v = (float)m * 5.9604644775390625e-08f;
        return (h >> 15) ? -v : v;
    }
    return bits_f(sign | ((uint32_t)(e + 112) << 23) | (m << 13));
}

/* binary32 -> binary16, round to nearest, ties to even, overflow to infinity (common.h:58-80). */
uint16_t no_f32_to_f16(float f) {
    uint32_t x = f_bits(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ebits = (x >> 23) & 0xffu;
    uint32_t m = x & 0x7fffffu;
    if (ebits == 0xff) return (uint16_t)(sign | 0x7c00u | (m ? 0x200u : 0));
    int e = (int)ebits - 112; /* binary16 biased exponent */
    uint32_t sig, shift;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e >= 1) {
        /* normal: keep 10 of 23 mantissa bits; a carry out of the mantissa bumps the exponent */
        sig = ((uint32_t)e << 10) | (m >> 13);
        shift = 13;
        uint32_t rem = m & 0x1fffu, half = 0x1000u;
        if (rem > half || (rem == half && (sig & 1u))) sig++;
        (void)shift;
        return (uint16_t)(sign | sig);
    }
    if (e < -10) return sign;
    /* subnormal result: value = (1.m) * 2^(e-15), expressed in units of 2^-24 */
    m |= 0x800000u;
    shift = (uint32_t)(14 - e);
    sig = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (sig & 1u))) sig++;
    return (uint16_t)(sign | sig);
}

size_t no_row_bytes(int fmt, int cols) {
    size_t c = (size_t)cols;
    size_t scales = (c / QBLOCK * 2 + 15) / 16 * 16; /* f16 scales, padded to 16 bytes */
    if (fmt == NO_F16) return c * 2;
    if (fmt == NO_FP8) return c + scales;
    return c / 2 + scales;
}

/* ---------------------------------------------------------------- codecs (quant.cpp:41-65) */

/* E4M3 by way of binary16: scale by 1/256 (exact), round to binary16, then round the binary16 pattern's
 * low 7 mantissa bits away (ties to even) and clamp to 0x7E = 448. The two roundings are the format's
 * definition and are kept. */
static uint8_t enc_fp8(float y) {
    uint16_t h = no_f32_to_f16(y * (1.0f / 256.0f));
    uint32_t mag = h & 0x7fffu;
    uint32_t c = (mag + 0x3fu + ((mag >> 7) & 1u)) >> 7;
    if (c > 0x7eu) c = 0x7eu;
    return (uint8_t)(c | ((h >> 8) & 0x80u));
}

static float dec_fp8(uint8_t c) {
    return no_f16_to_f32((uint16_t)(((c & 0x80u) << 8) | ((c & 0x7fu) << 7))) * 256.0f;
}

/* E2M1 magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6 chosen by midpoint thresholds; -0 encodes as 0. */
static uint8_t enc_fp4(float y) {
    float a = fabsf(y);
    int c = (a > 0.25f) + (a > 0.75f) + (a > 1.25f) + (a > 1.75f) + (a > 2.5f) + (a > 3.5f) + (a > 5.0f);
    return (uint8_t)(c == 0 ? 0 : (c | (y < 0 ? 8 : 0)));
}

static float dec_fp4(uint8_t c) {
    return no_f16_to_f32((uint16_t)(((c & 8u) << 12) | ((c & 7u) << 9))) * 16384.0f;
}

/* ---------------------------------------------------------------- scales (quant.cpp:72-178) */

static float block_amax(const float* x) {
    float a = 0;
    for (int i = 0; i < QBLOCK; i++) {
        float v = fabsf(x[i]);
        if (a < v) a = v; /* std::max(a, v) keeps a unless a < v */
    }
    return a;
}

/* f16 scale so the largest magnitude maps to maxCode; zero for an all-zero block (quant.cpp:72-79) */
static uint16_t block_scale(const float* x, float maxCode, float* inv) {
    uint16_t s = no_f32_to_f16(block_amax(x) / maxCode);
    float sv = no_f16_to_f32(s);
    *inv = sv > 0 ? 1.0f / sv : 0.0f;
    return sv > 0 ? s : 0;
}

static float fp4_round(float a) { /* quant.cpp:93-97; nearbyintf rounds half to even */
    if (a < 1.75f) return nearbyintf(a * 2.0f) * 0.5f;
    if (a < 3.5f) return nearbyintf(a);
    return a < 5.0f ? 4.0f : 6.0f;
}

typedef struct { float err, xr, rr; } fit_t;

static fit_t fit_fp4(const float* ax, float s) { /* scalar fitFp4, quant.cpp:126-136 */
    fit_t f = {0, 0, 0};
    const float inv = 1.0f / s;
    for (int i = 0; i < QBLOCK; i++) {
        float r = fp4_round(ax[i] * inv);
        float d = ax[i] - r * s;
        f.err += d * d;
        f.xr += ax[i] * r;
        f.rr += r * r;
    }
    return f;
}

/* Start at amax/6, then up to two least-squares refits s = sum(|x| r) / sum(r^2); keep the best
 * (quant.cpp:142-165). */
static uint16_t fp4_scale(const float* xb) {
    uint16_t best = no_f32_to_f16(block_amax(xb) / 6.0f);
    if (no_f16_to_f32(best) <= 0) return 0;
    float ax[QBLOCK];
    for (int i = 0; i < QBLOCK; i++) ax[i] = fabsf(xb[i]);
    fit_t fit = fit_fp4(ax, no_f16_to_f32(best));
    float bestErr = fit.err;
    for (int it = 0; it < 2 && fit.rr > 0; it++) {
        uint16_t s = no_f32_to_f16(fit.xr / fit.rr);
        if (no_f16_to_f32(s) <= 0 || s == best) break;
        fit = fit_fp4(ax, no_f16_to_f32(s));
        if (fit.err >= bestErr) break;
        bestErr = fit.err;
        best = s;
    }
    return best;
}

static void quant_row(int fmt, const float* x, int cols, uint8_t* out) {
    int nb = cols / QBLOCK;
    if (fmt == NO_F16) {
        for (int c = 0; c < cols; c++) {
            uint16_t h = no_f32_to_f16(x[c]);
            memcpy(out + 2 * c, &h, 2);
        }
        return;
    }
    uint8_t* sc = out + (fmt == NO_FP8 ? cols : cols / 2);
    for (int b = 0; b < nb; b++) {
        const float* xb = x + b * QBLOCK;
        uint16_t s;
        float inv;
        if (fmt == NO_FP8) {
            s = block_scale(xb, 448.0f, &inv);
            for (int i = 0; i < QBLOCK; i++) out[b * QBLOCK + i] = enc_fp8(xb[i] * inv);
        } else {
            s = fp4_scale(xb);
            inv = s ? 1.0f / no_f16_to_f32(s) : 0.0f;
            for (int j = 0; j < 16; j++)
                out[b * 16 + j] = (uint8_t)(enc_fp4(xb[j] * inv) | (enc_fp4(xb[16 + j] * inv) << 4));
        }
        memcpy(sc + 2 * b, &s, 2);
    }
}

void no_quantize_rows(int fmt, int rows, int cols, const float* w, uint8_t* out) {
    size_t rb = no_row_bytes(fmt, cols);
    memset(out, 0, rb * (size_t)rows); /* zero scale padding */
    for (int r = 0; r < rows; r++) quant_row(fmt, w + (size_t)r * cols, cols, out + (size_t)r * rb);
}

static void dequant_row(int fmt, const uint8_t* p, int cols, float* out) {
    if (fmt == NO_F16) {
        for (int c = 0; c < cols; c++) {
            uint16_t h;
            memcpy(&h, p + 2 * c, 2);
            out[c] = no_f16_to_f32(h);
        }
        return;
    }
    const uint8_t* sc = p + (fmt == NO_FP8 ? cols : cols / 2);
    for (int c = 0; c < cols; c++) {
        int b = c / QBLOCK, j = c % QBLOCK;
        uint16_t s;
        memcpy(&s, sc + 2 * b, 2);
        float sv = no_f16_to_f32(s);
        if (fmt == NO_FP8) {
            out[c] = dec_fp8(p[c]) * sv;
        } else {
            uint8_t byte = p[b * 16 + (j & 15)];
            out[c] = dec_fp4(j < 16 ? (uint8_t)(byte & 15u) : (uint8_t)(byte >> 4)) * sv;
        }
    }
}

void no_dequantize_rows(int fmt, int rows, int cols, const uint8_t* data, float* out) {
    size_t rb = no_row_bytes(fmt, cols);
    for (int r = 0; r < rows; r++) dequant_row(fmt, data + (size_t)r * rb, cols, out + (size_t)r * cols);
}

/* ---------------------------------------------------------------- ops (cpu_ops.cpp) */

float no_gelu(float x) { return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x))); }

void no_matmul(int fmt, const float* x, int T, int K, const uint8_t* W, int rows, const float* bias, float* y,
               int yStride, int flags) {
    size_t rb = no_row_bytes(fmt, K);
    float* w = (float*)malloc(sizeof(float) * (size_t)K);
    for (int n = 0; n < rows; n++) {
        dequant_row(fmt, W + (size_t)n * rb, K, w);
        for (int t = 0; t < T; t++) {
            const float* xt = x + (size_t)t * K;
            float v;
            if (fmt == NO_F16) {
                /* matmulF16 (x86 tail loop of dotRow4): sum from zero, bias added after */
                float acc = 0;
                for (int k = 0; k < K; k++) acc += w[k] * xt[k];
                v = acc + (bias ? bias[n] : 0.0f);
            } else {
                /* matmulGeneric: sum starts at the bias */
                v = bias ? bias[n] : 0.0f;
                for (int k = 0; k < K; k++) v += xt[k] * w[k];
            }
            if (flags & NO_GELU) v = no_gelu(v);
            float* dst = y + (size_t)t * yStride + n;
            *dst = (flags & NO_ACCUMULATE) ? *dst + v : v;
        }
    }
    free(w);
}

void no_layer_norm(const float* x, float* y, const float* g, const float* b, int T, int C, float eps) {
    for (int t = 0; t < T; t++) {
        const float* xr = x + (size_t)t * C;
        float* yr = y + (size_t)t * C;
        double mean = 0, var = 0;
        for (int c = 0; c < C; c++) mean += xr[c];
        mean /= C;
        for (int c = 0; c < C; c++) {
            double d = xr[c] - mean;
            var += d * d;
        }
        var /= C;
        float r = (float)(1.0 / sqrt(var + eps));
        float m = (float)mean;
        for (int c = 0; c < C; c++) yr[c] = (xr[c] - m) * r * g[c] + b[c];
    }
}

void no_rms_norm(const float* x, float* y, const float* w, int rows, int C, float eps) {
    for (int r = 0; r < rows; r++) {
        const float* xr = x + (size_t)r * C;
        float* yr = y + (size_t)r * C;
        double ss = 0;
        for (int c = 0; c < C; c++) ss += (double)xr[c] * xr[c];
        float s = (float)(1.0 / sqrt(ss / C + eps));
        for (int c = 0; c < C; c++) yr[c] = xr[c] * s * w[c];
    }
}

void no_rope(float* x, int nHeads, int hd, const float* cs) {
    int half = hd / 2;
    for (int h = 0; h < nHeads; h++) {
        float* v = x + (size_t)h * hd;
        for (int i = 0; i < half; i++) {
            float c = cs[2 * i], s = cs[2 * i + 1];
            float a = v[i], b = v[i + half];
            v[i] = a * c - b * s;
            v[i + half] = a * s + b * c;
        }
    }
}

void no_silu_mul(const float* h, float* out, int T, int I) {
    for (int t = 0; t < T; t++) {
        const float* gate = h + (size_t)t * 2 * I;
        const float* up = gate + I;
        float* o = out + (size_t)t * I;
        for (int i = 0; i < I; i++) o[i] = gate[i] / (1.0f + expf(-gate[i])) * up[i];
    }
}

void no_store_kv(const float* k, const float* v, int srcStride, uint16_t* kc, uint16_t* vc, int width, int T,
                 int pos0) {
    for (int t = 0; t < T; t++) {
        size_t dst = (size_t)(pos0 + t) * width;
        for (int i = 0; i < width; i++) {
            kc[dst + i] = no_f32_to_f16(k[(size_t)t * srcStride + i]);
            vc[dst + i] = no_f32_to_f16(v[(size_t)t * srcStride + i]);
        }
    }
}

void no_attention(const float* q, int qStride, const uint16_t* kc, const uint16_t* vc, float* out, int T, int nHead,
                  int nKv, int hd, int pos0) {
    int kvW = nKv * hd, group = nHead / nKv;
    float scale = 1.0f / sqrtf((float)hd);
    float* scores = (float*)malloc(sizeof(float) * (size_t)(pos0 + T));
    float* acc = (float*)malloc(sizeof(float) * (size_t)hd);
    for (int i = 0; i < nHead * T; i++) {
        int h = i % nHead, t = i / nHead, L = pos0 + t + 1;
        const float* qh = q + (size_t)t * qStride + (size_t)h * hd;
        size_t off = (size_t)(h / group) * hd;
        float mx = -INFINITY;
        for (int j = 0; j < L; j++) {
            const uint16_t* kr = kc + (size_t)j * kvW + off;
            float s = 0;
            for (int d = 0; d < hd; d++) s += qh[d] * no_f16_to_f32(kr[d]);
            s = s * scale;
            scores[j] = s;
            if (mx < s) mx = s;
        }
        float sum = 0;
        for (int j = 0; j < L; j++) {
            float e = expf(scores[j] - mx);
            scores[j] = e;
            sum += e;
        }
        for (int d = 0; d < hd; d++) acc[d] = 0;
        for (int j = 0; j < L; j++) {
            const uint16_t* vr = vc + (size_t)j * kvW + off;
            for (int d = 0; d < hd; d++) acc[d] += scores[j] * no_f16_to_f32(vr[d]);
        }
        float inv = 1.0f / sum;
        float* o = out + (size_t)t * nHead * hd + (size_t)h * hd;
        for (int d = 0; d < hd; d++) o[d] = acc[d] * inv;
    }
    free(scores);
    free(acc);
}

void no_softmax_rows(const float* x, float* y, int rows, int C) {
    for (int r = 0; r < rows; r++) {
        const float* xr = x + (size_t)r * C;
        float* yr = y + (size_t)r * C;
        float mx = -INFINITY, sum = 0;
        for (int j = 0; j < C; j++)
            if (mx < xr[j]) mx = xr[j];
        for (int j = 0; j < C; j++) {
            float e = expf(xr[j] - mx);
            yr[j] = e;
            sum += e;
        }
        float inv = 1.0f / sum;
        for (int j = 0; j < C; j++) yr[j] = yr[j] * inv;
    }
}

void no_rope_table(int ctx, int hd, double theta, float* out) {
    for (int i = 0; i < hd / 2; i++) {
        double inv = pow(theta, -2.0 * i / hd);
        for (int p = 0; p < ctx; p++) {
            double a = p * inv;
            out[(size_t)p * hd + 2 * i] = (float)cos(a);
            out[(size_t)p * hd + 2 * i + 1] = (float)sin(a);
        }
    }
}

void no_embed(int fmt, const uint8_t* table, int cols, const int* tokens, int T, const float* wpe, int pos0, float* x) {
    size_t rb = no_row_bytes(fmt, cols);
    for (int t = 0; t < T; t++) {
        float* xr = x + (size_t)t * cols;
        dequant_row(fmt, table + (size_t)tokens[t] * rb, cols, xr);
        if (wpe) {
            const float* pe = wpe + (size_t)(pos0 + t) * cols;
            for (int c = 0; c < cols; c++) xr[c] += pe[c];
        }
    }
}

int no_argmax(const float* x, int n) {
    int best = 0;
    for (int i = 1; i < n; i++)
        if (x[best] < x[i]) best = i;
    return best;
}
