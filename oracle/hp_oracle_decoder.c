/*
 * hp_oracle_decoder.c -- CPU restatement of the per-layer decoder math that
 * surrounds the quantized matmuls in the WASM provider.
 *
 * TEST INFRASTRUCTURE ONLY (see hp_oracle.c).
 *
 * Source: packages/engine/src/runner/wasm/layers.ts.  That code runs in
 * JavaScript numbers (f64) and rounds to f32 only where it stores into a
 * Float32Array or calls Math.fround; each function below keeps those rounding
 * points, doing the rest in double.
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>

float hpo_round_f16_ts(float v);

/* layers.ts:871-885 rmsNormVector: f64 sum of squares, f64 scale, the
 * product x*scale*w in f64, stored as f32. */
static void rms_vec(const float *x, const float *w, size_t n, double eps, float *o) {
    double ss = 0.0;
    for (size_t i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    double scale = 1.0 / sqrt(ss / (double)n + eps);
    for (size_t i = 0; i < n; i++) o[i] = (float)(((double)x[i] * scale) * (double)w[i]);
}

/* layers.ts:824-831 rmsNormRows and layers.ts:861-869 normHeads (same math,
 * rows of weight-length). */
void hpo_rms_norm_rows(const float *x, size_t rows, size_t dim, const float *w, double eps, float *o) {
    for (size_t r = 0; r < rows; r++) rms_vec(x + r * dim, w, dim, eps, o + r * dim);
}

/* layers.ts:833-848 rmsNormRowsNoWeight. */
void hpo_rms_norm_rows_noweight(const float *x, size_t rows, size_t dim, double eps, float *o) {
    for (size_t r = 0; r < rows; r++) {
        const float *xr = x + r * dim;
        double ss = 0.0;
        for (size_t i = 0; i < dim; i++) ss += (double)xr[i] * (double)xr[i];
        double scale = 1.0 / sqrt(ss / (double)dim + eps);
        for (size_t i = 0; i < dim; i++) o[r * dim + i] = (float)((double)xr[i] * scale);
    }
}

/* layers.ts:850-859 residualAdd. */
void hpo_residual_add(const float *a, const float *b, size_t n, float *o) {
    for (size_t i = 0; i < n; i++) o[i] = a[i] + b[i];
}

/* layers.ts:990-1033 ropeNeox: pairs (i, i + ndims/2); theta starts at the
 * position, is divided by the optional frequency factor, and is advanced as
 * fround(theta * base^(-2/ndims)); cos/sin in f64; each product rounded to
 * f32 before the f32 add/subtract. */
void hpo_rope_neox(const float *x, size_t head, size_t nheads, size_t ntok, const int32_t *pos,
                   size_t ndims, double freq_base, const float *factors, float *o) {
    size_t n = head * nheads * ntok;
    memcpy(o, x, n * sizeof(float));
    double theta_scale = pow(freq_base, -2.0 / (double)ndims);
    size_t half = ndims / 2;
    for (size_t t = 0; t < ntok; t++) {
        for (size_t h = 0; h < nheads; h++) {
            size_t row = (t * nheads + h) * head;
            double theta = (double)pos[t];
            for (size_t i = 0; i < half; i++) {
                double x0 = x[row + i], x1 = x[row + half + i];
                double th = theta / (factors ? (double)factors[i] : 1.0);
                double c = cos(th), s = sin(th);
                float a = (float)(x0 * c), b = (float)(x1 * s);
                float e = (float)(x0 * s), f = (float)(x1 * c);
                o[row + i] = a - b;
                o[row + half + i] = e + f;
                theta = (double)(float)(theta * theta_scale);
            }
        }
    }
}

/* layers.ts:982-988 castF16Rows (TS codec: ties to even, clamp to 65504). */
void hpo_cast_f16_rows(const float *x, size_t n, float *o) {
    for (size_t i = 0; i < n; i++) o[i] = hpo_round_f16_ts(x[i]);
}

/* layers.ts:1062-1076 gelu (tanh form) with f16 round trips of its input and
 * output; |x| >= 10 short-circuits. */
double hpo_gelu(float v) {
    if (v <= -10.0f) return 0.0;
    if (v >= 10.0f) return (double)v;
    double x = (double)hpo_round_f16_ts(v);
    float xx = (float)(x * x);
    float poly = (float)(1.0 + (double)(float)(0.044715 * (double)xx));
    float lin = (float)(sqrt(2.0 / M_PI) * x);
    float inner = (float)((double)lin * (double)poly);
    float half = (float)(0.5 * x);
    float act = (float)((double)half * (double)(float)(1.0 + tanh((double)inner)));
    return (double)hpo_round_f16_ts(act);
}

/* layers.ts:450-456 GeGLU: fround(gelu(gate) * up). */
void hpo_geglu(const float *gate, const float *up, size_t n, float *o) {
    for (size_t i = 0; i < n; i++) o[i] = (float)(hpo_gelu(gate[i]) * (double)up[i]);
}

/* layers.ts:407-412 final logit softcap: fround(tanh(x / c) * c). */
void hpo_softcap(float *v, size_t n, double cap) {
    for (size_t i = 0; i < n; i++) v[i] = (float)(tanh((double)v[i] / cap) * cap);
}

/* layers.ts:887-911 updateFullAttentionCache: K stored [slot][kv_head][dim],
 * V stored [dim][kv_head][slot]; slot = position mod capacity. */
void hpo_kv_update(float *kc, float *vc, size_t cap, size_t nkv, size_t klen, size_t vlen, const float *k,
                   const float *v, const int32_t *pos, size_t ntok) {
    for (size_t t = 0; t < ntok; t++) {
        size_t slot = (size_t)pos[t] % cap;
        for (size_t h = 0; h < nkv; h++) {
            for (size_t d = 0; d < klen; d++) kc[(slot * nkv + h) * klen + d] = k[(t * nkv + h) * klen + d];
            for (size_t d = 0; d < vlen; d++) vc[(d * nkv + h) * cap + slot] = v[(t * nkv + h) * vlen + d];
        }
    }
}

/* layers.ts:54-67 prepareInput embedding scale: fround(row * sqrt(d)). */
void hpo_scale_embedding(float *x, size_t n, double dim) {
    double s = sqrt(dim);
    for (size_t i = 0; i < n; i++) x[i] = (float)((double)x[i] * s);
}

/* ---- MTP draft head ("assistant") math --------------------------------- */

/* packages/engine/src/runner/wasm/mtp-assistant-runner.ts:275-290 rmsNorm and
 * runner/webgpu/mtp-target-runner.ts:225-244 normalizedHiddenSlice: unlike the
 * decoder's rmsNormVector the sum of squares is accumulated in f32 (each square
 * and each partial sum rounded); scale in f64; fround(fround(x * scale) * w). */
void hpo_rms_norm_f32sum_rows(const float *x, size_t rows, size_t dim, const float *w, double eps, float *o) {
    for (size_t r = 0; r < rows; r++) {
        const float *xr = x + r * dim;
        float ss = 0.0f;
        for (size_t i = 0; i < dim; i++) ss = ss + xr[i] * xr[i];
        double scale = 1.0 / sqrt((double)ss / (double)dim + eps);
        for (size_t i = 0; i < dim; i++) o[r * dim + i] = (float)((double)(float)((double)xr[i] * scale) * (double)w[i]);
    }
}

/* mtp-assistant-runner.ts:361-387 ropeNeox with activePairCount: only the first
 * `pairs` pairs (i, i + ndims/2) of each head rotate; theta starts at the
 * position and advances as fround(theta * base^(-2/ndims)). */
void hpo_rope_neox_pairs(const float *x, size_t head, size_t nheads, int32_t pos, size_t ndims, size_t pairs,
                         double freq_base, float *o) {
    memcpy(o, x, head * nheads * sizeof(float));
    double theta_scale = pow(freq_base, -2.0 / (double)ndims);
    size_t half = ndims / 2;
    for (size_t h = 0; h < nheads; h++) {
        size_t row = h * head;
        double theta = (double)pos;
        for (size_t i = 0; i < pairs; i++) {
            double x0 = x[row + i], x1 = x[row + half + i];
            double c = cos(theta), s = sin(theta);
            float a = (float)(x0 * c), b = (float)(x1 * s);
            float e = (float)(x0 * s), f = (float)(x1 * c);
            o[row + i] = a - b;
            o[row + half + i] = e + f;
            theta = (double)(float)(theta * theta_scale);
        }
    }
}

/* mtp-assistant-runner.ts:399-411 gelu (tanh form, no f16 round trips) and
 * :150-153 the gated product fround(gelu(gate) * up). */
static double gelu_f32points(float v) {
    double x = v;
    if (x <= -10.0) return 0.0;
    if (x >= 10.0) return x;
    float a = (float)(sqrt(2.0 / M_PI) * x);
    float xx = (float)(x * x);
    float b = (float)(0.044715 * (double)xx);
    float c = (float)(1.0 + (double)b);
    float inner = (float)((double)a * (double)c);
    float h = (float)(0.5 * x);
    float t = (float)(1.0 + tanh((double)inner));
    return (double)(float)((double)h * (double)t);
}

void hpo_gelu_mul_f32(const float *gate, const float *up, size_t n, float *o) {
    for (size_t i = 0; i < n; i++) o[i] = (float)(gelu_f32points(gate[i]) * (double)up[i]);
}
