/*
 * hp_oracle.c -- CPU restatement of the Heliopause decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle and the timed CPU
 * baseline.  Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may
 * load it; the CUDA product path never links or calls it.
 *
 * What it restates (paths are relative to the Heliopause source tree):
 *   packages/engine/wasm-kernels/src/lib.rs           (Rust kernels compiled to WASM)
 *   packages/engine/src/runner/wasm/layers.ts         (decoder math around the matmuls)
 *   packages/engine/src/runner/wasm/thread-pool.ts    (row sharding, splitRows)
 *   packages/engine/src/runtime.ts                    (topK)
 *   packages/engine/src/quant.ts                      (TS float16 codec used by layers.ts)
 *
 * Numeric contract: compiled with -O2 -ffp-contract=off and no fast-math, so
 * every f32 multiply and add rounds exactly like the Rust/WASM code (which
 * never contracts to FMA).  The lib.rs SIMD and scalar accumulators produce the
 * same integers (integer addition is exact), so the scalar lane order used here
 * (lane = element index mod 8) gives bit-identical f32 results.
 *
 * Status codes and validation order follow lib.rs:7-10 and the drivers at
 * lib.rs:41-536.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define HPO_OK 0
#define HPO_ERR_SHAPE 1
#define HPO_ERR_HEADS 2
#define HPO_ERR_TYPE 3

/* Type ids: lib.rs:12-17. */
#define HPO_Q4_K 1
#define HPO_Q5_K 2
#define HPO_Q6_K 3
#define HPO_IQ4_XS 4
#define HPO_Q8_0 5
#define HPO_Q4_0 6
#define QK 256

/* IQ4_NL code book, lib.rs:19-21 (a format table: must be identical). */
static const int8_t iq4nl_values[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                        1,    13,   25,  38,  53,  69,  89,  113};

/* ---------------------------------------------------------------- halves -- */

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* lib.rs:2507-2532 -- exact f16 -> f32 (subnormals normalised by shifting). */
float hpo_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)(h & 0x8000u)) << 16;
    int exp = (h >> 10) & 0x1f;
    uint32_t frac = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (frac == 0) {
            bits = sign;
        } else {
            int e = -14;
            while ((frac & 0x400u) == 0) {
                frac <<= 1;
                e -= 1;
            }
            frac &= 0x3ffu;
            bits = sign | ((uint32_t)(e + 127) << 23) | (frac << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (frac << 13);
    } else {
        bits = sign | ((uint32_t)(exp + 112) << 23) | (frac << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

/* lib.rs:2534-2568 -- the Rust f32 -> f16: round half UP on the 13 dropped
 * bits (not ties-to-even), overflow clamps to 0x7bff, NaN -> 0x7e00. */
uint16_t hpo_f32_to_f16_rust(float v) {
    uint32_t bits;
    memcpy(&bits, &v, 4);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    int exp = (int)((bits >> 23) & 0xff);
    uint32_t mant = bits & 0x7fffffu;
    if (exp == 0xff) return mant == 0 ? (uint16_t)(sign | 0x7c00u) : (uint16_t)0x7e00u;
    int he = exp - 127 + 15;
    if (he >= 31) return (uint16_t)(sign | 0x7bffu);
    if (he <= 0) {
        if (he < -10) return sign;
        uint32_t m = mant | 0x800000u;
        uint32_t shift = (uint32_t)(14 - he);
        uint32_t r = (m + (1u << (shift - 1))) >> shift;
        return (uint16_t)(sign | r);
    }
    uint32_t rm = mant + 0x1000u;
    if (rm & 0x800000u) {
        int re = he + 1;
        if (re >= 31) return (uint16_t)(sign | 0x7bffu);
        return (uint16_t)(sign | (uint16_t)(re << 10));
    }
    return (uint16_t)(sign | (uint16_t)(he << 10) | (uint16_t)(rm >> 13));
}

/* quant.ts:632-669 -- the TS f32 -> f16 used by layers.ts (castF16Rows, gelu):
 * ties-to-even, |x| >= 65504 clamps to 0x7bff, |x| < 2^-24 flushes to +-0.
 * Written with exact double arithmetic (frexp) instead of log2, which gives the
 * same exponent for every finite f32. */
static double rte(double x) {
    double f = floor(x);
    double frac = x - f;
    if (frac < 0.5) return f;
    if (frac > 0.5) return f + 1.0;
    return fmod(f, 2.0) == 0.0 ? f : f + 1.0;
}
uint16_t hpo_f32_to_f16_ts(float v) {
    if (isnan(v)) return 0x7e00u;
    if (isinf(v)) return v > 0 ? 0x7c00u : 0xfc00u;
    uint16_t sign = signbit(v) ? 0x8000u : 0;
    double a = fabs((double)v);
    if (a == 0.0) return sign;
    if (a >= 65504.0) return (uint16_t)(sign | 0x7bffu);
    if (a < ldexp(1.0, -24)) return sign;
    int e2;
    double m2 = frexp(a, &e2); /* a = m2 * 2^e2, m2 in [0.5,1) */
    int exponent = e2 - 1;      /* floor(log2(a)) */
    if (exponent < -14) {
        double sub = rte(a / ldexp(1.0, -24));
        return (uint16_t)(sign | (uint16_t)sub);
    }
    double mantissa = m2 * 2.0 - 1.0;
    double hm = rte(mantissa * 1024.0);
    if (hm == 1024.0) {
        exponent += 1;
        hm = 0.0;
    }
    return (uint16_t)(sign | (uint16_t)((exponent + 15) << 10) | (uint16_t)hm);
}

float hpo_round_f16_ts(float v) { return hpo_f16_to_f32(hpo_f32_to_f16_ts(v)); }
float hpo_round_f16_rust(float v) { return hpo_f16_to_f32(hpo_f32_to_f16_rust(v)); }

/* --------------------------------------------------------- block layouts -- */

/* lib.rs:1551-1561 */
static int row_bytes(int type, size_t k, size_t *out) {
    switch (type) {
    case HPO_Q4_K: if (k % QK) return 0; *out = k / QK * 144; return 1;
    case HPO_Q5_K: if (k % QK) return 0; *out = k / QK * 176; return 1;
    case HPO_Q6_K: if (k % QK) return 0; *out = k / QK * 210; return 1;
    case HPO_IQ4_XS: if (k % QK) return 0; *out = k / QK * 136; return 1;
    case HPO_Q8_0: if (k % 32) return 0; *out = k / 32 * 34; return 1;
    case HPO_Q4_0: if (k % 32) return 0; *out = k / 32 * 18; return 1;
    default: return 0;
    }
}

/* lib.rs:1563-1571 */
static int scale_values_per_row(int type, size_t k, size_t *out) {
    switch (type) {
    case HPO_Q4_K: case HPO_Q5_K: if (k % QK) return 0; *out = k / QK * 2; return 1;
    case HPO_Q6_K: case HPO_IQ4_XS: if (k % QK) return 0; *out = k / QK; return 1;
    case HPO_Q8_0: case HPO_Q4_0: if (k % 32) return 0; *out = k / 32; return 1;
    default: return 0;
    }
}

int hpo_row_bytes(int type, size_t k, size_t *out) { return row_bytes(type, k, out); }
int hpo_scale_values_per_row(int type, size_t k, size_t *out) { return scale_values_per_row(type, k, out); }

static inline int uses_q8_0(int type) { return type == HPO_Q4_0 || type == HPO_Q8_0; }

/* lib.rs:2250-2259 -- 6-bit scale/min unpack of the 12 packed bytes. */
static inline void scale_min_k4(int j, const uint8_t *q, uint8_t *sc, uint8_t *mn) {
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4));
        *mn = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* ----------------------------------------------------------- dequantize -- */

/* lib.rs:1592-1610 */
static void dq_q4_0(const uint8_t *b, size_t n, float *o) {
    for (size_t blk = 0; blk < n / 32; blk++, b += 18, o += 32) {
        float d = hpo_f16_to_f32(rd16(b));
        for (int i = 0; i < 16; i++) {
            o[i] = (float)((int)(b[2 + i] & 0x0f) - 8) * d;
            o[i + 16] = (float)((int)(b[2 + i] >> 4) - 8) * d;
        }
    }
}

/* lib.rs:1612-1628 */
static void dq_q8_0(const uint8_t *b, size_t n, float *o) {
    for (size_t blk = 0; blk < n / 32; blk++, b += 34, o += 32) {
        float d = hpo_f16_to_f32(rd16(b));
        for (int i = 0; i < 32; i++) o[i] = (float)(int8_t)b[2 + i] * d;
    }
}

/* lib.rs:1630-1664 -- y = (d*sc)*q - dmin*m, every step an f32 rounding. */
static void dq_q4_k(const uint8_t *b, size_t n, float *o) {
    for (size_t blk = 0; blk < n / QK; blk++, b += 144) {
        float d = hpo_f16_to_f32(rd16(b));
        float dmin = hpo_f16_to_f32(rd16(b + 2));
        const uint8_t *sc = b + 4, *qs = b + 16;
        for (int g = 0; g < 4; g++) {
            uint8_t s1, m1, s2, m2;
            scale_min_k4(2 * g, sc, &s1, &m1);
            scale_min_k4(2 * g + 1, sc, &s2, &m2);
            float d1 = d * (float)s1, d2 = d * (float)s2;
            float mm1 = dmin * (float)m1, mm2 = dmin * (float)m2;
            for (int l = 0; l < 32; l++) *o++ = d1 * (float)(qs[32 * g + l] & 0x0f) - mm1;
            for (int l = 0; l < 32; l++) *o++ = d2 * (float)(qs[32 * g + l] >> 4) - mm2;
        }
    }
}

/* lib.rs:1666-1707 */
static void dq_q5_k(const uint8_t *b, size_t n, float *o) {
    for (size_t blk = 0; blk < n / QK; blk++, b += 176) {
        float d = hpo_f16_to_f32(rd16(b));
        float dmin = hpo_f16_to_f32(rd16(b + 2));
        const uint8_t *sc = b + 4, *qh = b + 16, *qs = b + 48;
        uint8_t lowmask = 1, highmask = 2;
        for (int g = 0; g < 4; g++) {
            uint8_t s1, m1, s2, m2;
            scale_min_k4(2 * g, sc, &s1, &m1);
            scale_min_k4(2 * g + 1, sc, &s2, &m2);
            float d1 = d * (float)s1, d2 = d * (float)s2;
            float mm1 = dmin * (float)m1, mm2 = dmin * (float)m2;
            for (int l = 0; l < 32; l++) {
                int hi = (qh[l] & lowmask) ? 16 : 0;
                *o++ = d1 * (float)((qs[32 * g + l] & 0x0f) + hi) - mm1;
            }
            for (int l = 0; l < 32; l++) {
                int hi = (qh[l] & highmask) ? 16 : 0;
                *o++ = d2 * (float)((qs[32 * g + l] >> 4) + hi) - mm2;
            }
            lowmask = (uint8_t)(lowmask << 2);
            highmask = (uint8_t)(highmask << 2);
        }
    }
}

/* lib.rs:1709-1744 -- y = (d*sc)*q evaluated left to right as d*sc*q. */
static void dq_q6_k(const uint8_t *b, size_t n, float *o) {
    for (size_t blk = 0; blk < n / QK; blk++, b += 210, o += QK) {
        const uint8_t *ql = b, *qh = b + 128, *sc = b + 192;
        float d = hpo_f16_to_f32(rd16(b + 208));
        for (int half = 0; half < 2; half++) {
            const uint8_t *l8 = ql + 64 * half, *h8 = qh + 32 * half;
            const int8_t *s8 = (const int8_t *)(sc + 8 * half);
            float *oo = o + 128 * half;
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                uint8_t h = h8[l];
                int q1 = (int)((l8[l] & 0x0f) | (((h >> 0) & 3) << 4)) - 32;
                int q2 = (int)((l8[l + 32] & 0x0f) | (((h >> 2) & 3) << 4)) - 32;
                int q3 = (int)((l8[l] >> 4) | (((h >> 4) & 3) << 4)) - 32;
                int q4 = (int)((l8[l + 32] >> 4) | (((h >> 6) & 3) << 4)) - 32;
                oo[l] = d * (float)s8[is] * (float)q1;
                oo[l + 32] = d * (float)s8[is + 2] * (float)q2;
                oo[l + 64] = d * (float)s8[is + 4] * (float)q3;
                oo[l + 96] = d * (float)s8[is + 6] * (float)q4;
            }
        }
    }
}

/* lib.rs:1746-1772 */
static void dq_iq4_xs(const uint8_t *b, size_t n, float *o) {
    for (size_t blk = 0; blk < n / QK; blk++, b += 136) {
        float d = hpo_f16_to_f32(rd16(b));
        uint16_t sh = rd16(b + 2);
        const uint8_t *sl = b + 4, *qs = b + 8;
        for (int ib = 0; ib < 8; ib++) {
            int ls = (int)((((sl[ib / 2] >> (4 * (ib % 2))) & 0x0f)) | (((sh >> (2 * ib)) & 3) << 4));
            float dl = d * (float)(ls - 32);
            for (int j = 0; j < 16; j++) {
                o[j] = dl * (float)iq4nl_values[qs[16 * ib + j] & 0x0f];
                o[j + 16] = dl * (float)iq4nl_values[qs[16 * ib + j] >> 4];
            }
            o += 32;
        }
    }
}

/* lib.rs:1573-1586: returns 1 on success. */
int hpo_dequantize_row(int type, const uint8_t *bytes, size_t byte_len, size_t elements, float *out) {
    size_t rb;
    if (!row_bytes(type, elements, &rb) || rb != byte_len) return 0;
    switch (type) {
    case HPO_Q4_K: dq_q4_k(bytes, elements, out); return 1;
    case HPO_Q5_K: dq_q5_k(bytes, elements, out); return 1;
    case HPO_Q6_K: dq_q6_k(bytes, elements, out); return 1;
    case HPO_IQ4_XS: dq_iq4_xs(bytes, elements, out); return 1;
    case HPO_Q8_0: dq_q8_0(bytes, elements, out); return 1;
    case HPO_Q4_0: dq_q4_0(bytes, elements, out); return 1;
    default: return 0;
    }
}

/* --------------------------------------------------- activation quantizers -- */

/* Rust `f32 as i8`: truncation toward zero with saturation, NaN -> 0. */
static inline int8_t sat_i8(float v) {
    if (isnan(v)) return 0;
    if (v >= 127.0f) return 127;
    if (v <= -128.0f) return -128;
    return (int8_t)(int)v;
}

/* lib.rs:1774-1811.  amax keeps the FIRST strictly larger |x| and its signed
 * value; inv = -127/max; q = min(127, round(inv*x)) (round = half away from
 * zero, i.e. C roundf); d = 1/inv; bsums32 are i16 sums of 32 consecutive qs.
 * An all-zero block leaves d = 0, q = 0, bsums = 0. */
void hpo_quantize_q8_k(const float *x, size_t n, float *d, int8_t *qs, int16_t *bsums32) {
    size_t nb = n / QK;
    memset(qs, 0, n);
    memset(bsums32, 0, nb * 8 * sizeof(int16_t));
    for (size_t b = 0; b < nb; b++) {
        const float *xb = x + b * QK;
        float amax = 0.0f, max = 0.0f;
        for (int i = 0; i < QK; i++) {
            float a = fabsf(xb[i]);
            if (a > amax) {
                amax = a;
                max = xb[i];
            }
        }
        d[b] = 0.0f;
        if (amax == 0.0f) continue;
        float inv = -127.0f / max;
        for (int i = 0; i < QK; i++) qs[b * QK + i] = sat_i8(fminf(roundf(inv * xb[i]), 127.0f));
        for (int g = 0; g < 8; g++) {
            int16_t s = 0;
            for (int i = 0; i < 32; i++) s = (int16_t)(s + qs[b * QK + g * 32 + i]);
            bsums32[b * 8 + g] = s;
        }
        d[b] = 1.0f / inv;
    }
}

/* lib.rs:1813-1833 */
void hpo_quantize_q8_0(const float *x, size_t n, float *d, int8_t *qs) {
    for (size_t b = 0; b < n / 32; b++) {
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[b * 32 + i]));
        float scale = hpo_f16_to_f32(hpo_f32_to_f16_rust(amax / 127.0f));
        float inv = scale != 0.0f ? 1.0f / scale : 0.0f;
        d[b] = scale;
        for (int i = 0; i < 32; i++) qs[b * 32 + i] = sat_i8(roundf(x[b * 32 + i] * inv));
    }
}

/* ---------------------------------------------------------- dot products -- */

typedef struct {
    size_t nb;         /* number of 256-blocks (Q8_K) or 32-blocks (Q8_0) */
    const float *d;
    const int8_t *qs;
    const int16_t *bsums32; /* Q8_K only */
} q8act;

/* lib.rs:2443-2466 scalar fallback: lane = index mod 8 over a 32-group. */
static inline void acc32(int32_t acc[8], int32_t scale, const int8_t *a, const int8_t *w) {
    for (int c = 0; c < 4; c++)
        for (int l = 0; l < 8; l++) acc[l] += scale * (int32_t)a[8 * c + l] * (int32_t)w[8 * c + l];
}
/* lib.rs:2265-2287 scalar fallback: lane = index mod 8 over a 16-group. */
static inline void acc16(int32_t acc[8], int32_t scale, const int8_t *a, const int8_t *w) {
    for (int c = 0; c < 2; c++)
        for (int l = 0; l < 8; l++) acc[l] += scale * (int32_t)a[8 * c + l] * (int32_t)w[8 * c + l];
}

static inline float lane_total(float sumf, const float sums[8]) {
    float t = 0.0f;
    for (int l = 0; l < 8; l++) t += sums[l];
    return sumf + t;
}

/* lib.rs:2059-2172.  `pre` is the prepared f32 (d, dmin) pair per block, or
 * NULL to decode the f16 halves in place (the two give identical values). */
static float dot_q4_k(const uint8_t *w, const q8act *a, const float *pre) {
    float sums[8] = {0}, sumf = 0.0f;
    int8_t aux8[QK];
    for (size_t b = 0; b < a->nb; b++, w += 144) {
        const uint8_t *scb = w + 4, *qs = w + 16;
        uint8_t sc[8], mn[8];
        for (int j = 0; j < 8; j++) scale_min_k4(j, scb, &sc[j], &mn[j]);
        for (int g = 0; g < 4; g++)
            for (int l = 0; l < 32; l++) {
                aux8[64 * g + l] = (int8_t)(qs[32 * g + l] & 0x0f);
                aux8[64 * g + 32 + l] = (int8_t)(qs[32 * g + l] >> 4);
            }
        int32_t sumi = 0;
        for (int g = 0; g < 8; g++) sumi += (int32_t)a->bsums32[b * 8 + g] * (int32_t)mn[g];
        int32_t aux32[8] = {0};
        for (int g = 0; g < 8; g++) acc32(aux32, sc[g], a->qs + b * QK + 32 * g, aux8 + 32 * g);
        float dw = pre ? pre[2 * b] : hpo_f16_to_f32(rd16(w));
        float mw = pre ? pre[2 * b + 1] : hpo_f16_to_f32(rd16(w + 2));
        float d = dw * a->d[b];
        for (int l = 0; l < 8; l++) sums[l] += d * (float)aux32[l];
        float dmin = mw * a->d[b];
        sumf -= dmin * (float)sumi;
    }
    return lane_total(sumf, sums);
}

/* lib.rs:1970-2057 */
static float dot_q5_k(const uint8_t *w, const q8act *a, const float *pre) {
    float sums[8] = {0}, sumf = 0.0f;
    int8_t aux8[QK];
    for (size_t b = 0; b < a->nb; b++, w += 176) {
        const uint8_t *scb = w + 4, *qh = w + 16, *qs = w + 48;
        for (int l = 0; l < 32; l++) {
            aux8[l] = (int8_t)((qs[l] & 0x0f) | ((qh[l] & 1) << 4));
            aux8[l + 32] = (int8_t)((qs[l] >> 4) | (((qh[l] >> 1) & 1) << 4));
            aux8[l + 64] = (int8_t)((qs[l + 32] & 0x0f) | (((qh[l] >> 2) & 1) << 4));
            aux8[l + 96] = (int8_t)((qs[l + 32] >> 4) | (((qh[l] >> 3) & 1) << 4));
            aux8[l + 128] = (int8_t)((qs[l + 64] & 0x0f) | (((qh[l] >> 4) & 1) << 4));
            aux8[l + 160] = (int8_t)((qs[l + 64] >> 4) | (((qh[l] >> 5) & 1) << 4));
            aux8[l + 192] = (int8_t)((qs[l + 96] & 0x0f) | (((qh[l] >> 6) & 1) << 4));
            aux8[l + 224] = (int8_t)((qs[l + 96] >> 4) | ((qh[l] >> 7) << 4));
        }
        int32_t aux32[8] = {0}, sumi = 0;
        for (int g = 0; g < 8; g++) {
            uint8_t sc, mn;
            scale_min_k4(g, scb, &sc, &mn);
            sumi += (int32_t)a->bsums32[b * 8 + g] * (int32_t)mn;
            acc32(aux32, sc, a->qs + b * QK + 32 * g, aux8 + 32 * g);
        }
        float dw = pre ? pre[2 * b] : hpo_f16_to_f32(rd16(w));
        float mw = pre ? pre[2 * b + 1] : hpo_f16_to_f32(rd16(w + 2));
        float d = dw * a->d[b];
        for (int l = 0; l < 8; l++) sums[l] += d * (float)aux32[l];
        float dmin = mw * a->d[b];
        sumf -= dmin * (float)sumi;
    }
    return lane_total(sumf, sums);
}

/* lib.rs:1877-1968 */
static float dot_q6_k(const uint8_t *w, const q8act *a, const float *pre) {
    float sums[8] = {0};
    int8_t aux8[QK];
    for (size_t b = 0; b < a->nb; b++, w += 210) {
        const uint8_t *ql = w, *qh = w + 128;
        const int8_t *sc = (const int8_t *)(w + 192);
        for (int half = 0; half < 2; half++) {
            const uint8_t *l8 = ql + 64 * half, *h8 = qh + 32 * half;
            int8_t *ax = aux8 + 128 * half;
            for (int l = 0; l < 32; l++) {
                uint8_t h = h8[l];
                ax[l] = (int8_t)((int)((l8[l] & 0x0f) | (((h >> 0) & 3) << 4)) - 32);
                ax[l + 32] = (int8_t)((int)((l8[l + 32] & 0x0f) | (((h >> 2) & 3) << 4)) - 32);
                ax[l + 64] = (int8_t)((int)((l8[l] >> 4) | (((h >> 4) & 3) << 4)) - 32);
                ax[l + 96] = (int8_t)((int)((l8[l + 32] >> 4) | (((h >> 6) & 3) << 4)) - 32);
            }
        }
        int32_t aux32[8] = {0};
        for (int g = 0; g < 16; g++) acc16(aux32, sc[g], a->qs + b * QK + 16 * g, aux8 + 16 * g);
        float dw = pre ? pre[b] : hpo_f16_to_f32(rd16(w + 208));
        float d = dw * a->d[b];
        for (int l = 0; l < 8; l++) sums[l] += d * (float)aux32[l];
    }
    float t = 0.0f;
    for (int l = 0; l < 8; l++) t += sums[l];
    return t;
}

/* lib.rs:2174-2247 (accumulate_iq4_nl_32_quads scalar path: lane = index/4). */
static float dot_iq4_xs(const uint8_t *w, const q8act *a, const float *pre) {
    float accum[8] = {0};
    for (size_t b = 0; b < a->nb; b++, w += 136) {
        float d4d8 = (pre ? pre[b] : hpo_f16_to_f32(rd16(w))) * a->d[b];
        uint16_t sh = rd16(w + 2);
        const uint8_t *sl = w + 4, *qs = w + 8;
        int32_t lane[8] = {0};
        const int8_t *q8 = a->qs + b * QK;
        for (int ib = 0; ib < 8; ib += 2) {
            uint8_t ps = sl[ib / 2];
            int32_t ls1 = (int32_t)((ps & 0x0f) | ((uint8_t)(sh << 4) & 0x30)) - 32;
            int32_t ls2 = (int32_t)((ps >> 4) | ((uint8_t)(sh << 2) & 0x30)) - 32;
            sh = (uint16_t)(sh >> 4);
            for (int half = 0; half < 2; half++) {
                int32_t ls = half ? ls2 : ls1;
                const uint8_t *p = qs + 16 * (ib + half);
                const int8_t *x = q8 + 32 * (ib + half);
                for (int j = 0; j < 32; j++) {
                    uint8_t byte = p[j & 15];
                    int32_t v = j < 16 ? iq4nl_values[byte & 0x0f] : iq4nl_values[byte >> 4];
                    lane[j >> 2] += ls * v * (int32_t)x[j];
                }
            }
        }
        for (int l = 0; l < 8; l++) accum[l] = d4d8 * (float)lane[l] + accum[l];
    }
    float t = 0.0f;
    for (int l = 0; l < 8; l++) t += accum[l];
    return t;
}

/* lib.rs:1835-1875 */
static float dot_q8_0(const uint8_t *w, const q8act *a, const float *pre) {
    float sum = 0.0f;
    for (size_t b = 0; b < a->nb; b++, w += 34) {
        int32_t isum = 0;
        for (int i = 0; i < 32; i++) isum += (int32_t)(int8_t)w[2 + i] * (int32_t)a->qs[b * 32 + i];
        float dw = pre ? pre[b] : hpo_f16_to_f32(rd16(w));
        sum += (float)isum * (dw * a->d[b]);
    }
    return sum;
}
static float dot_q4_0(const uint8_t *w, const q8act *a, const float *pre) {
    float sum = 0.0f;
    for (size_t b = 0; b < a->nb; b++, w += 18) {
        int32_t isum = 0;
        for (int i = 0; i < 16; i++) {
            uint8_t p = w[2 + i];
            isum += ((int32_t)(p & 0x0f) - 8) * (int32_t)a->qs[b * 32 + i];
            isum += ((int32_t)(p >> 4) - 8) * (int32_t)a->qs[b * 32 + i + 16];
        }
        float dw = pre ? pre[b] : hpo_f16_to_f32(rd16(w));
        sum += (float)isum * (dw * a->d[b]);
    }
    return sum;
}

typedef float (*dot_fn)(const uint8_t *, const q8act *, const float *);
static dot_fn dot_for(int type) {
    switch (type) {
    case HPO_Q4_K: return dot_q4_k;
    case HPO_Q5_K: return dot_q5_k;
    case HPO_Q6_K: return dot_q6_k;
    case HPO_IQ4_XS: return dot_iq4_xs;
    case HPO_Q8_0: return dot_q8_0;
    case HPO_Q4_0: return dot_q4_0;
    default: return NULL;
    }
}

/* Quantize one activation column into caller storage sized for k. */
typedef struct {
    float *d;
    int8_t *qs;
    int16_t *bs;
    q8act view;
} q8buf;

static int q8buf_init(q8buf *q, int type, const float *x, size_t k) {
    size_t nb = uses_q8_0(type) ? k / 32 : k / QK;
    q->d = (float *)malloc(nb * sizeof(float) + 1);
    q->qs = (int8_t *)malloc(k + 1);
    q->bs = (int16_t *)malloc((k / QK + 1) * 8 * sizeof(int16_t));
    if (!q->d || !q->qs || !q->bs) return 0;
    if (uses_q8_0(type)) hpo_quantize_q8_0(x, k, q->d, q->qs);
    else hpo_quantize_q8_k(x, k, q->d, q->qs, q->bs);
    q->view.nb = nb;
    q->view.d = q->d;
    q->view.qs = q->qs;
    q->view.bsums32 = q->bs;
    return 1;
}
static void q8buf_free(q8buf *q) {
    free(q->d);
    free(q->qs);
    free(q->bs);
}

/* -------------------------------------------------------------- drivers -- */

/* lib.rs:157-222 */
int hpo_prepare_quantized_scales_f32(int type, const uint8_t *w, size_t wlen, size_t k, size_t rows,
                                     float *scales, size_t slen) {
    size_t rb, spr;
    if (!row_bytes(type, k, &rb)) return HPO_ERR_TYPE;
    if (wlen != rb * rows) return HPO_ERR_SHAPE;
    if (!scale_values_per_row(type, k, &spr)) return HPO_ERR_TYPE;
    if (slen != spr * rows) return HPO_ERR_SHAPE;
    size_t nb = uses_q8_0(type) ? k / 32 : k / QK;
    for (size_t r = 0; r < rows; r++) {
        const uint8_t *row = w + r * rb;
        float *s = scales + r * spr;
        for (size_t b = 0; b < nb; b++) {
            switch (type) {
            case HPO_Q4_K: s[2 * b] = hpo_f16_to_f32(rd16(row + b * 144)); s[2 * b + 1] = hpo_f16_to_f32(rd16(row + b * 144 + 2)); break;
            case HPO_Q5_K: s[2 * b] = hpo_f16_to_f32(rd16(row + b * 176)); s[2 * b + 1] = hpo_f16_to_f32(rd16(row + b * 176 + 2)); break;
            case HPO_Q6_K: s[b] = hpo_f16_to_f32(rd16(row + b * 210 + 208)); break;
            case HPO_IQ4_XS: s[b] = hpo_f16_to_f32(rd16(row + b * 136)); break;
            case HPO_Q8_0: s[b] = hpo_f16_to_f32(rd16(row + b * 34)); break;
            case HPO_Q4_0: s[b] = hpo_f16_to_f32(rd16(row + b * 18)); break;
            default: return HPO_ERR_TYPE;
            }
        }
    }
    return HPO_OK;
}

/* Rows [r0, r1) of one column, shared by the direct, prepared and threaded
 * drivers (lib.rs:264-296 inner loop). */
static void rows_dot(int type, const uint8_t *w, size_t rb, const float *scales, size_t spr,
                     const q8act *a, size_t rows, size_t col, size_t r0, size_t r1, float *out) {
    dot_fn f = dot_for(type);
    for (size_t r = r0; r < r1; r++)
        out[col * rows + r] = f(w + r * rb, a, scales ? scales + r * spr : NULL);
}

/* lib.rs:41-100 (scales == NULL) and lib.rs:225-298 (prepared). */
static int matmul_common(int type, const uint8_t *w, size_t wlen, const float *scales, size_t slen,
                         int prepared, const float *in, size_t inlen, size_t k, size_t rows,
                         size_t cols, float *out, size_t outlen) {
    if (inlen != k * cols || outlen != rows * cols) return HPO_ERR_SHAPE;
    size_t rb, spr = 0;
    if (!row_bytes(type, k, &rb)) return HPO_ERR_TYPE;
    if (wlen != rb * rows) return HPO_ERR_SHAPE;
    if (prepared) {
        if (!scale_values_per_row(type, k, &spr)) return HPO_ERR_TYPE;
        if (slen != spr * rows) return HPO_ERR_SHAPE;
    }
    for (size_t c = 0; c < cols; c++) {
        q8buf q;
        if (!q8buf_init(&q, type, in + c * k, k)) return HPO_ERR_SHAPE;
        rows_dot(type, w, rb, prepared ? scales : NULL, spr, &q.view, rows, c, 0, rows, out);
        q8buf_free(&q);
    }
    return HPO_OK;
}

int hpo_matmul_quantized_f32(int type, const uint8_t *w, size_t wlen, const float *in, size_t inlen,
                             size_t k, size_t rows, size_t cols, float *out, size_t outlen) {
    return matmul_common(type, w, wlen, NULL, 0, 0, in, inlen, k, rows, cols, out, outlen);
}

int hpo_matmul_quantized_prepared_f32(int type, const uint8_t *w, size_t wlen, const float *scales,
                                      size_t slen, const float *in, size_t inlen, size_t k, size_t rows,
                                      size_t cols, float *out, size_t outlen) {
    return matmul_common(type, w, wlen, scales, slen, 1, in, inlen, k, rows, cols, out, outlen);
}

/* lib.rs:302-426 (prepared multi) and lib.rs:430-536 (direct multi): up to 4
 * weights share one input; the activation is quantized once per column. */
typedef struct {
    int type;
    const uint8_t *w;
    size_t wlen;
    const float *scales;
    size_t slen;
    size_t rows;
    float *out;
    size_t outlen;
} hpo_multi_spec;

int hpo_matmul_multi_f32(size_t count, const float *in, size_t inlen, size_t k, size_t cols,
                         const hpo_multi_spec *specs, int prepared) {
    if (count == 0 || count > 4 || inlen != k * cols) return HPO_ERR_SHAPE;
    for (size_t i = 0; i < count; i++) {
        size_t rb, spr;
        if (!row_bytes(specs[i].type, k, &rb)) return HPO_ERR_TYPE;
        if (prepared) {
            if (!scale_values_per_row(specs[i].type, k, &spr)) return HPO_ERR_TYPE;
            if (specs[i].wlen != rb * specs[i].rows || specs[i].slen != spr * specs[i].rows ||
                specs[i].outlen != specs[i].rows * cols)
                return HPO_ERR_SHAPE;
        } else if (specs[i].wlen != rb * specs[i].rows || specs[i].outlen != specs[i].rows * cols) {
            return HPO_ERR_SHAPE;
        }
    }
    for (size_t c = 0; c < cols; c++) {
        q8buf qk, q0;
        int have_k = 0, have_0 = 0;
        for (size_t i = 0; i < count; i++) {
            const hpo_multi_spec *s = &specs[i];
            size_t rb, spr = 0;
            row_bytes(s->type, k, &rb);
            scale_values_per_row(s->type, k, &spr);
            q8buf *q;
            if (uses_q8_0(s->type)) {
                if (!have_0) { q8buf_init(&q0, s->type, in + c * k, k); have_0 = 1; }
                q = &q0;
            } else {
                if (!have_k) { q8buf_init(&qk, s->type, in + c * k, k); have_k = 1; }
                q = &qk;
            }
            rows_dot(s->type, s->w, rb, prepared ? s->scales : NULL, spr, &q->view, s->rows, c, 0,
                     s->rows, s->out);
        }
        if (have_k) q8buf_free(&qk);
        if (have_0) q8buf_free(&q0);
    }
    return HPO_OK;
}

/* lib.rs:103-154 -- fp32 dequant row times f32 input, sequential f32 sum. */
int hpo_matmul_dequantized_f32(int type, const uint8_t *w, size_t wlen, const float *in, size_t inlen,
                               size_t k, size_t rows, size_t cols, float *out, size_t outlen) {
    if (inlen != k * cols || outlen != rows * cols) return HPO_ERR_SHAPE;
    size_t rb;
    if (!row_bytes(type, k, &rb)) return HPO_ERR_TYPE;
    if (wlen != rb * rows) return HPO_ERR_SHAPE;
    float *wr = (float *)malloc(k * sizeof(float));
    if (!wr) return HPO_ERR_SHAPE;
    for (size_t r = 0; r < rows; r++) {
        if (!hpo_dequantize_row(type, w + r * rb, rb, k, wr)) {
            free(wr);
            return HPO_ERR_TYPE;
        }
        for (size_t c = 0; c < cols; c++) {
            float s = 0.0f;
            for (size_t i = 0; i < k; i++) s = s + wr[i] * in[c * k + i];
            out[c * rows + r] = s;
        }
    }
    free(wr);
    return HPO_OK;
}

/* ---------------------------------------------- threaded (splitRows) path -- */

/* thread-pool.ts:410-424 -- contiguous shards, the first `rows % n` one row
 * larger; empty shards are dropped. */
size_t hpo_split_rows(size_t rows, size_t shards, size_t *starts, size_t *counts) {
    size_t base = rows / shards, extra = rows % shards, start = 0, n = 0;
    for (size_t i = 0; i < shards; i++) {
        size_t c = base + (extra > 0 ? 1 : 0);
        if (extra > 0) extra--;
        if (c > 0) {
            starts[n] = start;
            counts[n] = c;
            n++;
            start += c;
        }
    }
    return n;
}

typedef struct {
    int type;
    const uint8_t *w;
    size_t rb;
    const float *scales;
    size_t spr;
    const q8act *a;
    size_t rows, col, r0, r1;
    float *out;
} shard_job;

static void *shard_main(void *p) {
    shard_job *j = (shard_job *)p;
    rows_dot(j->type, j->w, j->rb, j->scales, j->spr, j->a, j->rows, j->col, j->r0, j->r1, j->out);
    return NULL;
}

/* Prepared single-weight matmul with the rows split across `threads` workers
 * (one worker per shard, as the WASM thread pool does). Same results as the
 * single-threaded driver: each row's dot is computed by exactly one worker. */
int hpo_matmul_prepared_threaded(int type, const uint8_t *w, size_t wlen, const float *scales,
                                 size_t slen, const float *in, size_t inlen, size_t k, size_t rows,
                                 size_t cols, float *out, size_t outlen, int threads) {
    if (inlen != k * cols || outlen != rows * cols) return HPO_ERR_SHAPE;
    size_t rb, spr;
    if (!row_bytes(type, k, &rb)) return HPO_ERR_TYPE;
    if (wlen != rb * rows) return HPO_ERR_SHAPE;
    if (!scale_values_per_row(type, k, &spr)) return HPO_ERR_TYPE;
    if (slen != spr * rows) return HPO_ERR_SHAPE;
    if (threads < 1) threads = 1;
    size_t starts[256], counts[256];
    if (threads > 256) threads = 256;
    size_t ns = hpo_split_rows(rows, (size_t)threads, starts, counts);
    pthread_t tid[256];
    shard_job jobs[256];
    for (size_t c = 0; c < cols; c++) {
        q8buf q;
        q8buf_init(&q, type, in + c * k, k);
        for (size_t s = 0; s < ns; s++) {
            jobs[s] = (shard_job){type, w, rb, scales, spr, &q.view, rows, c, starts[s], starts[s] + counts[s], out};
            pthread_create(&tid[s], NULL, shard_main, &jobs[s]);
        }
        for (size_t s = 0; s < ns; s++) pthread_join(tid[s], NULL);
        q8buf_free(&q);
    }
    return HPO_OK;
}

/* Exposed Q8_K helpers for tests: quantize and a single prepared row dot. */
float hpo_vec_dot_row(int type, const uint8_t *row, size_t k, const float *x) {
    q8buf q;
    q8buf_init(&q, type, x, k);
    float r = dot_for(type)(row, &q.view, NULL);
    q8buf_free(&q);
    return r;
}

/* ------------------------------------------------------------ attention -- */

/* lib.rs:539-654.  value_layout 1 = V stored [dim][kv_head][capacity slot]
 * ("dim-head-token"); 0 = [slot][kv_head][dim].  The query is rounded through
 * the Rust f16 codec when quantize_query_f16 != 0.  Softmax uses an f64 exp of
 * the f32 difference, as lib.rs:630 does. */
int hpo_gqa_attention_f32(const float *q, size_t qlen, const float *key, size_t klen, const float *val,
                          size_t vlen, const float *mask, size_t mlen, size_t head, size_t nq, size_t nkv,
                          size_t ntok, size_t nkvtok, size_t kvstart, size_t cap, float scale,
                          int value_layout, int quantize_query_f16, float *out, size_t outlen) {
    if (qlen != ntok * nq * head || klen != cap * nkv * head || vlen != cap * nkv * head ||
        outlen != ntok * nq * head || (mlen != 0 && mlen != ntok * nkvtok))
        return HPO_ERR_SHAPE;
    if (nkv == 0 || cap == 0 || nkvtok > cap || nq % nkv != 0) return HPO_ERR_HEADS;
    size_t group = nq / nkv;
    float *scores = (float *)malloc((nkvtok + 1) * sizeof(float));
    float *qq = (float *)malloc(head * sizeof(float));
    for (size_t t = 0; t < ntok; t++) {
        for (size_t h = 0; h < nq; h++) {
            size_t kvh = h / group;
            const float *qv = q + (t * nq + h) * head;
            for (size_t i = 0; i < head; i++) qq[i] = quantize_query_f16 ? hpo_round_f16_rust(qv[i]) : qv[i];
            float mx = -INFINITY;
            for (size_t j = 0; j < nkvtok; j++) {
                size_t slot = (kvstart + j) % cap;
                const float *kv = key + (slot * nkv + kvh) * head;
                float dot = 0.0f;
                for (size_t i = 0; i < head; i++) dot = dot + qq[i] * kv[i];
                float mv = mlen == 0 ? 0.0f : mask[t * nkvtok + j];
                float s = (mv == -INFINITY) ? -INFINITY : (dot * scale) + mv;
                scores[j] = s;
                if (s > mx) mx = s;
            }
            float sum = 0.0f;
            for (size_t j = 0; j < nkvtok; j++) {
                float p = scores[j] == -INFINITY ? 0.0f : (float)exp((double)(scores[j] - mx));
                scores[j] = p;
                sum += p;
            }
            float *o = out + (t * nq + h) * head;
            for (size_t i = 0; i < head; i++) {
                float acc = 0.0f;
                for (size_t j = 0; j < nkvtok; j++) {
                    size_t slot = (kvstart + j) % cap;
                    size_t vo = value_layout == 1 ? (i * nkv + kvh) * cap + slot : (slot * nkv + kvh) * head + i;
                    acc = acc + (scores[j] / sum) * val[vo];
                }
                o[i] = acc;
            }
        }
    }
    free(scores);
    free(qq);
    return HPO_OK;
}

/* ---------------------------------------------------------------- top-k -- */

/* runtime.ts:514-527: insertion into a list kept sorted by value descending;
 * a value enters only when the list is short or it is strictly greater than
 * the current last, so on ties the lower (earlier) id wins.  NaN never
 * enters a full list.  Returns the number of entries written (<= k). */
size_t hpo_topk(const float *v, size_t n, size_t k, int32_t *ids, float *vals) {
    size_t len = 0;
    if (k == 0) return 0;
    for (size_t i = 0; i < n; i++) {
        float x = v[i];
        if (len < k || x > vals[len - 1]) {
            size_t pos = len < k ? len : k - 1;
            /* stable insertion: move past every entry with value >= x */
            size_t at = 0;
            while (at < pos && !(x > vals[at])) at++;
            for (size_t s = pos; s > at; s--) {
                vals[s] = vals[s - 1];
                ids[s] = ids[s - 1];
            }
            vals[at] = x;
            ids[at] = (int32_t)i;
            if (len < k) len++;
        }
    }
    return len;
}
