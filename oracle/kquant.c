/*
 * CPU oracle, part 1: GGUF k-quant formats and the candle CPU QMatMul.
 * Test infrastructure only (see oracle.h for who may call it).
 *
 * Format semantics follow the reference's vendored k-quant code,
 * ferrite-os/crates/internal/ptx-kernels/kernels/candle/quantized.cu:
 *   block_q4_K :388-393, block_q6_K :419-424, block_q8_K :428-432,
 *   get_scale_min_k4 :925-933, dequantize_block_q4_K :936-1022,
 *   dequantize_block_q6_K :1024-1129.
 * The quantizers, the Q8_K activation quantizer, vec_dot and matmul restate
 * candle-core 0.8.4 src/quantized/k_quants.rs (crates.io, Cargo.lock:598-601,
 * not vendored): BlockQ4K/BlockQ6K/BlockQ8K::from_float, ::vec_dot (scalar
 * path — the reference build does not enable target-cpu=native,
 * .cargo/config.toml), and k_quants::matmul (rayon split over output
 * features, 128..512 per task).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

size_t or_block_bytes(int dtype) {
    switch (dtype) {
    case OR_Q4_K: return sizeof(or_block_q4k);
    case OR_Q6_K: return sizeof(or_block_q6k);
    case OR_Q8_K: return sizeof(or_block_q8k);
    case OR_F32: return 4;
    case OR_F16: return 2;
    default: return 0;
    }
}

/* ------------------------------------------------------------ fp16 ----- */
float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    float f;
    if (e == 0) {
        /* zero or subnormal: man * 2^-24, exact in f32 */
        f = (float)man * (1.0f / 16777216.0f);
        memcpy(&bits, &f, 4);
        bits |= sign;
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (man << 13);
    }
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t or_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t a = x & 0x7fffffffu;
    if (a >= 0x7f800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0u));
    if (a >= 0x477ff000u) /* >= 65520 rounds to inf */
        return (uint16_t)(sign | 0x7c00u);
    if (a < 0x38800000u) { /* below 2^-14: subnormal half or zero */
        if (a < 0x33000000u) /* <= 2^-25 (tie rounds to even 0) */
            return (uint16_t)sign;
        uint32_t e = a >> 23;
        uint32_t m = (a & 0x7fffffu) | 0x800000u;
        uint32_t sh = 126u - e; /* 14..24 */
        uint32_t r = m >> sh;
        uint32_t rem = m & ((1u << sh) - 1u);
        uint32_t half = 1u << (sh - 1u);
        if (rem > half || (rem == half && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = a - 0x38000000u;
    uint32_t h = r >> 13;
    uint32_t rem = r & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

/* Rust f32::round (half away from zero) or round-half-even. */
static inline int nearest_int(float v, int mode) {
    return mode ? (int)nearbyintf(v) : (int)roundf(v);
}

/* 6-bit scale j and min j of a Q4_K block (quantized.cu:925-933). */
static inline void q4k_scale_min(int j, const uint8_t *s, int *sc, int *mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* ------------------------------------------------------- quantizers ---- */
/* Iterative min/scale fit for one sub-block of asymmetric quants
 * (ggml make_qkx1_quants as used by candle's BlockQ4K::from_float with
 * nmax = 15, ntry = 5).  Returns the scale, writes the (positive) min. */
static float fit_scale_min(int n, int nmax, int ntry, const float *x,
                           float *min_out) {
    uint8_t lv[32];
    float lo = x[0], hi = x[0];
    for (int i = 1; i < n; i++) {
        if (x[i] < lo) lo = x[i];
        if (x[i] > hi) hi = x[i];
    }
    if (hi == lo) {
        *min_out = 0.f;
        return 0.f;
    }
    memset(lv, 0, sizeof lv);
    if (lo > 0.f) lo = 0.f;
    float iscale = (float)nmax / (hi - lo);
    float scale = 1.0f / iscale;
    for (int t = 0; t < ntry; t++) {
        float sumlx = 0.f;
        int suml2 = 0;
        int changed = 0;
        for (int i = 0; i < n; i++) {
            int l = nearest_int(iscale * (x[i] - lo), 0);
            if (l < 0) l = 0;
            if (l > nmax) l = nmax;
            if ((uint8_t)l != lv[i]) {
                lv[i] = (uint8_t)l;
                changed = 1;
            }
            sumlx += (x[i] - lo) * (float)l;
            suml2 += l * l;
        }
        scale = sumlx / (float)suml2;
        float acc = 0.f;
        for (int i = 0; i < n; i++) acc += x[i] - scale * (float)lv[i];
        lo = acc / (float)n;
        if (lo > 0.f) lo = 0.f;
        iscale = 1.0f / scale;
        if (!changed) break;
    }
    *min_out = -lo;
    return scale;
}

void or_quantize_q4k(const float *x, int64_t n, void *out) {
    or_block_q4k *blk = (or_block_q4k *)out;
    int64_t nb = n / OR_QK_K;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; b++) {
        const float *xb = x + b * OR_QK_K;
        or_block_q4k *y = blk + b;
        float scales[8], mins[8];
        for (int j = 0; j < 8; j++)
            scales[j] = fit_scale_min(32, 15, 5, xb + 32 * j, &mins[j]);
        float max_scale = 0.f, max_min = 0.f;
        for (int j = 0; j < 8; j++) {
            max_scale = scales[j] > max_scale ? scales[j] : max_scale;
            max_min = mins[j] > max_min ? mins[j] : max_min;
        }
        float inv_scale = max_scale > 0.f ? 63.f / max_scale : 0.f;
        float inv_min = max_min > 0.f ? 63.f / max_min : 0.f;
        memset(y->scales, 0, sizeof y->scales);
        for (int j = 0; j < 8; j++) {
            int ls = nearest_int(inv_scale * scales[j], 0);
            int lm = nearest_int(inv_min * mins[j], 0);
            if (ls > 63) ls = 63;
            if (lm > 63) lm = 63;
            uint8_t s8 = (uint8_t)ls, m8 = (uint8_t)lm;
            if (j < 4) {
                y->scales[j] = s8;
                y->scales[j + 4] = m8;
            } else {
                y->scales[j + 4] = (uint8_t)((s8 & 0x0F) | ((m8 & 0x0F) << 4));
                y->scales[j - 4] |= (uint8_t)((s8 >> 4) << 6);
                y->scales[j] |= (uint8_t)((m8 >> 4) << 6);
            }
        }
        y->d = or_f32_to_f16(max_scale / 63.f);
        y->dmin = or_f32_to_f16(max_min / 63.f);
        uint8_t lv[OR_QK_K];
        memset(lv, 0, sizeof lv);
        float dd = or_f16_to_f32(y->d), dm = or_f16_to_f32(y->dmin);
        for (int j = 0; j < 8; j++) {
            int sc, mn;
            q4k_scale_min(j, y->scales, &sc, &mn);
            float d = dd * (float)sc;
            if (d == 0.f) continue;
            float off = dm * (float)mn;
            for (int i = 0; i < 32; i++) {
                int l = nearest_int((xb[32 * j + i] + off) / d, 0);
                lv[32 * j + i] = (uint8_t)(l < 0 ? 0 : (l > 15 ? 15 : l));
            }
        }
        /* byte g*32+l: low nibble = weight 64g+l, high = weight 64g+32+l */
        for (int g = 0; g < 4; g++)
            for (int l = 0; l < 32; l++)
                y->qs[32 * g + l] =
                    (uint8_t)(lv[64 * g + l] | (lv[64 * g + 32 + l] << 4));
    }
}

/* Symmetric 6-bit fit of 16 weights with an x^2-weighted scale search
 * (ggml make_qx_quants with nmax = 32, rmse_type = 1, as used by candle's
 * BlockQ6K::from_float).  lv receives quants offset by +nmax. */
static float fit_symmetric(int n, int nmax, const float *x, int8_t *lv) {
    float mx = 0.f, amax = 0.f;
    for (int i = 0; i < n; i++) {
        float ax = fabsf(x[i]);
        if (ax > amax) {
            amax = ax;
            mx = x[i];
        }
    }
    if (amax < 1e-30f) {
        for (int i = 0; i < n; i++) lv[i] = 0;
        return 0.f;
    }
    float iscale = -(float)nmax / mx;
    float sumlx = 0.f, suml2 = 0.f;
    for (int i = 0; i < n; i++) {
        int l = nearest_int(iscale * x[i], 0);
        if (l < -nmax) l = -nmax;
        if (l > nmax - 1) l = nmax - 1;
        lv[i] = (int8_t)(l + nmax);
        float w = x[i] * x[i];
        sumlx += w * x[i] * (float)l;
        suml2 += w * (float)l * (float)l;
    }
    float scale = sumlx / suml2;
    float best = scale * sumlx;
    for (int s = -9; s <= 9; s++) {
        if (s == 0) continue;
        iscale = -((float)nmax + 0.1f * (float)s) / mx;
        sumlx = suml2 = 0.f;
        for (int i = 0; i < n; i++) {
            int l = nearest_int(iscale * x[i], 0);
            if (l < -nmax) l = -nmax;
            if (l > nmax - 1) l = nmax - 1;
            float w = x[i] * x[i];
            sumlx += w * x[i] * (float)l;
            suml2 += w * (float)l * (float)l;
        }
        if (suml2 > 0.f && sumlx * sumlx > best * suml2) {
            for (int i = 0; i < n; i++) {
                int l = nearest_int(iscale * x[i], 0);
                if (l < -nmax) l = -nmax;
                if (l > nmax - 1) l = nmax - 1;
                lv[i] = (int8_t)(l + nmax);
            }
            scale = sumlx / suml2;
            best = scale * sumlx;
        }
    }
    return scale;
}

void or_quantize_q6k(const float *x, int64_t n, void *out) {
    or_block_q6k *blk = (or_block_q6k *)out;
    int64_t nb = n / OR_QK_K;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; b++) {
        const float *xb = x + b * OR_QK_K;
        or_block_q6k *y = blk + b;
        int8_t lv[OR_QK_K];
        float scales[16];
        float max_scale = 0.f, max_abs = 0.f;
        for (int j = 0; j < 16; j++) {
            scales[j] = fit_symmetric(16, 32, xb + 16 * j, lv + 16 * j);
            float a = fabsf(scales[j]);
            if (a > max_abs) {
                max_abs = a;
                max_scale = scales[j];
            }
        }
        memset(y, 0, sizeof *y);
        if (max_abs == 0.f) continue; /* all-zero block */
        float iscale = -128.f / max_scale;
        y->d = or_f32_to_f16(1.0f / iscale);
        for (int j = 0; j < 16; j++) {
            int s = nearest_int(iscale * scales[j], 0);
            y->scales[j] = (int8_t)(s > 127 ? 127 : s);
        }
        float dd = or_f16_to_f32(y->d);
        for (int j = 0; j < 16; j++) {
            float d = dd * (float)y->scales[j];
            if (d == 0.f) continue;
            for (int i = 0; i < 16; i++) {
                int l = nearest_int(xb[16 * j + i] / d, 0);
                l = l < -32 ? -32 : (l > 31 ? 31 : l);
                lv[16 * j + i] = (int8_t)(l + 32);
            }
        }
        /* half h (128 weights): ql[64h+l] = q[l] | q[l+64] << 4,
         * ql[64h+32+l] = q[l+32] | q[l+96] << 4, qh[32h+l] packs the top two
         * bits of q[l], q[l+32], q[l+64], q[l+96]. */
        for (int h = 0; h < 2; h++) {
            const int8_t *q = lv + 128 * h;
            for (int l = 0; l < 32; l++) {
                y->ql[64 * h + l] = (uint8_t)((q[l] & 0xF) | ((q[l + 64] & 0xF) << 4));
                y->ql[64 * h + 32 + l] =
                    (uint8_t)((q[l + 32] & 0xF) | ((q[l + 96] & 0xF) << 4));
                y->qh[32 * h + l] = (uint8_t)(((q[l] >> 4) & 3) |
                                              (((q[l + 32] >> 4) & 3) << 2) |
                                              (((q[l + 64] >> 4) & 3) << 4) |
                                              (((q[l + 96] >> 4) & 3) << 6));
            }
        }
    }
}

void or_quantize_q8k(const float *x, int64_t n, void *out, int round_mode) {
    or_block_q8k *blk = (or_block_q8k *)out;
    int64_t nb = n / OR_QK_K;
    for (int64_t b = 0; b < nb; b++) {
        const float *xb = x + b * OR_QK_K;
        or_block_q8k *y = blk + b;
        float mx = 0.f, amax = 0.f;
        for (int i = 0; i < OR_QK_K; i++) {
            float a = fabsf(xb[i]);
            if (amax < a) {
                amax = a;
                mx = xb[i];
            }
        }
        if (amax == 0.f) {
            memset(y, 0, sizeof *y);
            continue;
        }
        float iscale = -128.f / mx;
        for (int i = 0; i < OR_QK_K; i++) {
            int v = nearest_int(iscale * xb[i], round_mode);
            y->qs[i] = (int8_t)(v > 127 ? 127 : v);
        }
        for (int g = 0; g < 16; g++) {
            int s = 0;
            for (int i = 0; i < 16; i++) s += y->qs[16 * g + i];
            y->bsums[g] = (int16_t)s;
        }
        y->d = 1.0f / iscale;
    }
}

/* ------------------------------------------------------- dequantize ---- */
static void dequant_q4k_block(const or_block_q4k *b, float *y) {
    float d = or_f16_to_f32(b->d), dm = or_f16_to_f32(b->dmin);
    for (int g = 0; g < 4; g++) {
        int sc0, m0, sc1, m1;
        q4k_scale_min(2 * g, b->scales, &sc0, &m0);
        q4k_scale_min(2 * g + 1, b->scales, &sc1, &m1);
        float d0 = d * (float)sc0, o0 = dm * (float)m0;
        float d1 = d * (float)sc1, o1 = dm * (float)m1;
        const uint8_t *q = b->qs + 32 * g;
        for (int l = 0; l < 32; l++) y[64 * g + l] = d0 * (float)(q[l] & 0xF) - o0;
        for (int l = 0; l < 32; l++) y[64 * g + 32 + l] = d1 * (float)(q[l] >> 4) - o1;
    }
}

static inline int q6k_quant(const or_block_q6k *b, int i) {
    /* weight i (0..255) of a Q6_K block, centred: -32..31 */
    int h = i >> 7, r = i & 127, l = r & 31, part = r >> 5;
    uint8_t lo = b->ql[64 * h + l + ((part & 1) ? 32 : 0)];
    int low = (part < 2) ? (lo & 0xF) : (lo >> 4);
    int high = (b->qh[32 * h + l] >> (2 * part)) & 3;
    return (low | (high << 4)) - 32;
}

static void dequant_q6k_block(const or_block_q6k *b, float *y) {
    float d = or_f16_to_f32(b->d);
    for (int i = 0; i < OR_QK_K; i++)
        y[i] = d * (float)b->scales[i >> 4] * (float)q6k_quant(b, i);
}

/* The factors of each weight's dequantization, w = scale * q - offset, with
 * scale = d * sc (Q4_K, Q6_K) and offset = dmin * m (Q4_K; 0 for Q6_K): both
 * products are exact in f32 (an fp16 times a 6- or 8-bit integer), q is the
 * integer code (0..15, or -32..31 for Q6_K).  Lets a test restate other
 * rounding orders of the same dequantization exactly. */
void or_dequant_parts(int dtype, const void *blocks, int64_t n, float *scale, float *offset, int8_t *q) {
    int64_t nb = n / OR_QK_K;
    if (dtype == OR_Q4_K) {
        const or_block_q4k *b = (const or_block_q4k *)blocks;
        for (int64_t i = 0; i < nb; i++) {
            float d = or_f16_to_f32(b[i].d), dm = or_f16_to_f32(b[i].dmin);
            for (int j = 0; j < OR_QK_K; j++) {
                int g = j / 64, hi = (j % 64) >= 32, l = j % 32, sc, m;
                q4k_scale_min(2 * g + hi, b[i].scales, &sc, &m);
                int64_t o = i * OR_QK_K + j;
                scale[o] = d * (float)sc;
                offset[o] = dm * (float)m;
                q[o] = (int8_t)(hi ? (b[i].qs[32 * g + l] >> 4) : (b[i].qs[32 * g + l] & 0xF));
            }
        }
    } else if (dtype == OR_Q6_K) {
        const or_block_q6k *b = (const or_block_q6k *)blocks;
        for (int64_t i = 0; i < nb; i++) {
            float d = or_f16_to_f32(b[i].d);
            for (int j = 0; j < OR_QK_K; j++) {
                int64_t o = i * OR_QK_K + j;
                scale[o] = d * (float)b[i].scales[j >> 4];
                offset[o] = 0.0f;
                q[o] = (int8_t)q6k_quant(b + i, j);
            }
        }
    }
}

void or_dequantize(int dtype, const void *blocks, int64_t n, float *y) {
    int64_t nb = n / OR_QK_K;
    if (dtype == OR_Q4_K) {
        const or_block_q4k *b = (const or_block_q4k *)blocks;
        for (int64_t i = 0; i < nb; i++) dequant_q4k_block(b + i, y + i * OR_QK_K);
    } else if (dtype == OR_Q6_K) {
        const or_block_q6k *b = (const or_block_q6k *)blocks;
        for (int64_t i = 0; i < nb; i++) dequant_q6k_block(b + i, y + i * OR_QK_K);
    } else if (dtype == OR_Q8_K) {
        const or_block_q8k *b = (const or_block_q8k *)blocks;
        for (int64_t i = 0; i < nb; i++)
            for (int j = 0; j < OR_QK_K; j++) y[i * OR_QK_K + j] = (float)b[i].qs[j] * b[i].d;
    } else if (dtype == OR_F32) {
        memcpy(y, blocks, (size_t)n * 4);
    }
}

static int resolve_threads(int nthreads);

/* ---------------------------------------------------------- vec_dot ---- */
/* Per-block integer partials.  lanes[l] accumulates sc_j * q * a over the
 * weights whose index is l mod 8 (the scalar k_quants vec_dot shape). */
static void q4k_block_int(const or_block_q4k *x, const or_block_q8k *y,
                          int32_t lanes[8], int32_t *sum_min) {
    int8_t q[OR_QK_K];
    for (int g = 0; g < 4; g++)
        for (int l = 0; l < 32; l++) {
            q[64 * g + l] = (int8_t)(x->qs[32 * g + l] & 0xF);
            q[64 * g + 32 + l] = (int8_t)(x->qs[32 * g + l] >> 4);
        }
    int32_t sm = 0;
    for (int j = 0; j < 8; j++) {
        int sc, mn;
        q4k_scale_min(j, x->scales, &sc, &mn);
        sm += mn * ((int32_t)y->bsums[2 * j] + (int32_t)y->bsums[2 * j + 1]);
        for (int i = 0; i < 32; i++)
            lanes[i & 7] += sc * ((int32_t)q[32 * j + i] * (int32_t)y->qs[32 * j + i]);
    }
    *sum_min = sm;
}

static void q6k_block_int(const or_block_q6k *x, const or_block_q8k *y,
                          int32_t lanes[8]) {
    for (int j = 0; j < 16; j++) {
        int sc = x->scales[j];
        for (int i = 0; i < 16; i++) {
            int w = 16 * j + i;
            lanes[w & 7] += sc * (q6k_quant(x, w) * (int32_t)y->qs[w]);
        }
    }
}

/* Per super-block the integer partials are exact; they are combined with the
 * fp16 super-block scales in binary64 (one rounding to f32 at the end) so the
 * result does not depend on the order in which blocks are summed.  candle
 * combines in f32 (8 lane sums); the two differ in the last bits only. */
double or_vec_dot64(int dtype, int64_t n, const void *w, const void *a) {
    int64_t nb = n / OR_QK_K;
    const or_block_q8k *y = (const or_block_q8k *)a;
    double acc = 0.0;
    for (int64_t b = 0; b < nb; b++) {
        int32_t lanes[8] = {0};
        int32_t isum = 0;
        if (dtype == OR_Q4_K) {
            const or_block_q4k *x = (const or_block_q4k *)w + b;
            int32_t smin;
            q4k_block_int(x, y + b, lanes, &smin);
            for (int l = 0; l < 8; l++) isum += lanes[l];
            double dy = (double)y[b].d;
            acc += (double)or_f16_to_f32(x->d) * dy * (double)isum;
            acc -= (double)or_f16_to_f32(x->dmin) * dy * (double)smin;
        } else {
            const or_block_q6k *x = (const or_block_q6k *)w + b;
            q6k_block_int(x, y + b, lanes);
            for (int l = 0; l < 8; l++) isum += lanes[l];
            acc += (double)or_f16_to_f32(x->d) * (double)y[b].d * (double)isum;
        }
    }
    return acc;
}

float or_vec_dot(int dtype, int64_t n, const void *w, const void *a) {
    return (float)or_vec_dot64(dtype, n, w, a);
}

/* The same integer partials combined in f32 the way candle-core 0.8.4's
 * scalar k_quants vec_dot does (the published ggml reference form): per
 * super-block d = d_w * d_y in f32, eight lane sums sums[l] += d * lane[l],
 * for Q4_K sumf -= (dmin_w * d_y) * sum_min, and at the end the lane sums
 * are added to sumf in lane order.  Used by the oracle's candle-f32 forward
 * (or_model_forward numerics 3) to measure how far the binary64 combine
 * sits from candle's own float order. */
float or_vec_dot_candle_f32(int dtype, int64_t n, const void *w, const void *a) {
    int64_t nb = n / OR_QK_K;
    const or_block_q8k *y = (const or_block_q8k *)a;
    float sums[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float sumf = 0.f;
    for (int64_t b = 0; b < nb; b++) {
        int32_t lanes[8] = {0};
        if (dtype == OR_Q4_K) {
            const or_block_q4k *x = (const or_block_q4k *)w + b;
            int32_t smin;
            q4k_block_int(x, y + b, lanes, &smin);
            const float d = or_f16_to_f32(x->d) * y[b].d;
            for (int l = 0; l < 8; l++) sums[l] += d * (float)lanes[l];
            const float dmin = or_f16_to_f32(x->dmin) * y[b].d;
            sumf -= dmin * (float)smin;
        } else {
            const or_block_q6k *x = (const or_block_q6k *)w + b;
            q6k_block_int(x, y + b, lanes);
            const float d = or_f16_to_f32(x->d) * y[b].d;
            for (int l = 0; l < 8; l++) sums[l] += d * (float)lanes[l];
        }
    }
    for (int l = 0; l < 8; l++) sumf += sums[l];
    return sumf;
}

void or_qmatmul_candle_f32(int dtype, const void *w, int64_t n, int64_t k, const float *x, int64_t m, float *y,
                           int nthreads) {
    int64_t nb = k / OR_QK_K;
    size_t bb = or_block_bytes(dtype);
    or_block_q8k *xq = (or_block_q8k *)malloc((size_t)(m * nb) * sizeof(or_block_q8k));
    for (int64_t r = 0; r < m; r++) or_quantize_q8k(x + r * k, k, xq + r * nb, 0);
    int nt = resolve_threads(nthreads);
    for (int64_t r = 0; r < m; r++) {
        const or_block_q8k *xr = xq + r * nb;
        float *yr = y + r * n;
#pragma omp parallel for num_threads(nt) schedule(dynamic, 256)
        for (int64_t c = 0; c < n; c++)
            yr[c] = or_vec_dot_candle_f32(dtype, k, (const uint8_t *)w + (size_t)c * nb * bb, xr);
    }
    free(xq);
}

void or_block_dots(int dtype, int64_t nrows, int64_t k, const void *w,
                   const void *a, int32_t *out_sc, int32_t *out_min) {
    int64_t nb = k / OR_QK_K;
    const or_block_q8k *y = (const or_block_q8k *)a;
    for (int64_t r = 0; r < nrows; r++)
        for (int64_t b = 0; b < nb; b++) {
            int32_t lanes[8] = {0}, smin = 0;
            if (dtype == OR_Q4_K)
                q4k_block_int((const or_block_q4k *)w + r * nb + b, y + b, lanes, &smin);
            else
                q6k_block_int((const or_block_q6k *)w + r * nb + b, y + b, lanes);
            int32_t s = 0;
            for (int l = 0; l < 8; l++) s += lanes[l];
            out_sc[r * nb + b] = s;
            out_min[r * nb + b] = smin;
        }
}

/* ----------------------------------------------------------- matmul ---- */
static int resolve_threads(int nthreads) {
#ifdef _OPENMP
    return nthreads > 0 ? nthreads : omp_get_max_threads();
#else
    (void)nthreads;
    return 1;
#endif
}

void or_qmatmul(int dtype, const void *w, int64_t n, int64_t k,
                const float *x, int64_t m, float *y, int nthreads) {
    int64_t nb = k / OR_QK_K;
    size_t bb = or_block_bytes(dtype);
    or_block_q8k *xq = (or_block_q8k *)malloc((size_t)(m * nb) * sizeof(or_block_q8k));
    for (int64_t r = 0; r < m; r++) or_quantize_q8k(x + r * k, k, xq + r * nb, 0);
    int nt = resolve_threads(nthreads);
    for (int64_t r = 0; r < m; r++) {
        const or_block_q8k *xr = xq + r * nb;
        float *yr = y + r * n;
#pragma omp parallel for num_threads(nt) schedule(dynamic, 256)
        for (int64_t c = 0; c < n; c++)
            yr[c] = or_vec_dot(dtype, k, (const uint8_t *)w + (size_t)c * nb * bb, xr);
    }
    free(xq);
}

/* Same sums as or_qmatmul without the final rounding: the binary64 partial
 * a tensor-parallel rank holding input columns [c0, c0 + k) contributes. */
void or_qmatmul64(int dtype, const void *w, int64_t n, int64_t k,
                  const float *x, int64_t m, double *y, int nthreads) {
    int64_t nb = k / OR_QK_K;
    size_t bb = or_block_bytes(dtype);
    or_block_q8k *xq = (or_block_q8k *)malloc((size_t)(m * nb) * sizeof(or_block_q8k));
    for (int64_t r = 0; r < m; r++) or_quantize_q8k(x + r * k, k, xq + r * nb, 0);
    int nt = resolve_threads(nthreads);
    for (int64_t r = 0; r < m; r++) {
        const or_block_q8k *xr = xq + r * nb;
        double *yr = y + r * n;
#pragma omp parallel for num_threads(nt) schedule(dynamic, 256)
        for (int64_t c = 0; c < n; c++)
            yr[c] = or_vec_dot64(dtype, k, (const uint8_t *)w + (size_t)c * nb * bb, xr);
    }
    free(xq);
}

void or_qmatmul_f32(int dtype, const void *w, int64_t n, int64_t k,
                    const float *x, int64_t m, float *y, int nthreads) {
    int64_t nb = k / OR_QK_K;
    size_t bb = or_block_bytes(dtype);
    int nt = resolve_threads(nthreads);
#pragma omp parallel num_threads(nt)
    {
        float *row = (float *)malloc((size_t)k * sizeof(float));
#pragma omp for schedule(dynamic, 64)
        for (int64_t c = 0; c < n; c++) {
            or_dequantize(dtype, (const uint8_t *)w + (size_t)c * nb * bb, k, row);
            for (int64_t r = 0; r < m; r++) {
                const float *xr = x + r * k;
                double acc = 0.0;
                for (int64_t i = 0; i < k; i++) acc += (double)row[i] * (double)xr[i];
                y[r * n + c] = (float)acc;
            }
        }
        free(row);
    }
}
