/*
 * CPU oracle, part 2: elementwise ops, the synthetic-weight generator, and the
 * quantized Llama / Qwen3 forward with a KV cache.  Test infrastructure only.
 *
 * Forward structure restates candle-transformers 0.8.4
 * models/quantized_llama.rs (crates.io, Cargo.lock:707-723, not vendored) as
 * called from crates/ferrite-wasm-host/src/adapter.rs:41-70:
 *   x = embed(tokens); per layer: x += wo(attn(rope(wq·n1(x)), rope(wk·n1(x)),
 *   wv·n1(x))); x += w_down(silu(w_gate·n2(x)) * w_up·n2(x)); logits =
 *   output(norm(x)) at the last position.
 * Ops follow candle-nn 0.8.4: rms_norm = x / sqrt(mean(x^2) + eps) * g
 * (CUDA form at ferrite-os/crates/internal/ptx-kernels/kernels/candle/
 * reduce.cu:189-230), softmax_last_dim (reduce.cu:233-273), rope_i
 * interleaved pairs (reduce.cu:275-292) and rope rotate-half
 * (reduce.cu:294-318), silu = v / (1 + exp(-v)) (unary.cu:59).
 * Qwen3 additions (not in the reference's candle path, which loads qwen3
 * GGUFs through the llama loader, crates/ferrite-core/src/registry/
 * spec.rs:73,84-94): per-head RMSNorm of q and k before RoPE, rotate-half
 * RoPE.  rope_mode 0 / qk_norm 0 reproduces what the reference runs.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ----------------------------------------------------------- ops ------ */
/* Reductions accumulate in binary64 (each f32 square / product is exact
 * there), so the result does not depend on summation order; candle sums in
 * f32 left to right, which differs from this in the last bits only. */
void or_rmsnorm(const float *x, const float *g, float *y, int64_t rows,
                int64_t dim, float eps) {
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * dim;
        float *yr = y + r * dim;
        double ss = 0.0;
        for (int64_t i = 0; i < dim; i++) ss += (double)xr[i] * (double)xr[i];
        float mean = (float)(ss / (double)dim);
        float m = sqrtf(mean + eps);
        for (int64_t i = 0; i < dim; i++) yr[i] = xr[i] / m * g[i];
    }
}

/* Attention score q.k in f32 with a fixed evaluation order: eight slices of
 * hd/8 consecutive dims, each a fused multiply-add chain from zero in
 * increasing dim order, then the slice sums added left to right. */
float or_attn_dot(const float *q, const float *k, int hd) {
    const int sl = hd / 8;
    float dot = 0.f;
    for (int w = 0; w < 8; w++) {
        float pw = 0.f;
        for (int e = w * sl; e < (w + 1) * sl; e++) pw = fmaf(q[e], k[e], pw);
        dot = w == 0 ? pw : dot + pw;
    }
    return dot;
}

double or_exp64(double x) {
    static const double C[14] = {1.0, 1.0, 0.5, 0.16666666666666666, 0.041666666666666664,
                                 0.008333333333333333, 0.001388888888888889, 0.0001984126984126984,
                                 2.48015873015873e-05, 2.7557319223985893e-06, 2.755731922398589e-07,
                                 2.505210838544172e-08, 2.08767569878681e-09, 1.6059043836821613e-10};
    const double LOG2E = 1.4426950408889634, LN2_HI = 0.6931471803691238, LN2_LO = 1.9082149292705877e-10;
    if (x != x) return x;
    if (x > 709.5) return INFINITY;
    if (x < -745.5) return 0.0;
    double k = nearbyint(x * LOG2E);
    double r = (x - k * LN2_HI) - k * LN2_LO;
    double p = C[13];
    for (int i = 12; i >= 0; i--) p = fma(p, r, C[i]);
    return ldexp(p, (int)k);
}

static float rope_inv_freq(int i, int head_dim, float theta) {
    /* candle precompute_freqs_cis: 1 / theta^(2i / head_dim) in f32 */
    return 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
}

void or_rope(float *x, int64_t n_heads, int64_t head_dim, int64_t pos,
             float theta, int mode) {
    int64_t half = head_dim / 2;
    for (int64_t i = 0; i < half; i++) {
        float ang = (float)pos * rope_inv_freq((int)i, (int)head_dim, theta);
        float c = cosf(ang), s = sinf(ang);
        for (int64_t h = 0; h < n_heads; h++) {
            float *xh = x + h * head_dim;
            int64_t a = mode ? i : 2 * i, b = mode ? i + half : 2 * i + 1;
            float x0 = xh[a], x1 = xh[b];
            xh[a] = x0 * c - x1 * s;
            xh[b] = x0 * s + x1 * c;
        }
    }
}

/* candle-nn's CPU rms_norm in its own order: the f32 sum of squares left to
 * right, m = sqrt(sum / dim + eps), y = x / m * g. */
static void rmsnorm_f32(const float *x, const float *g, float *y, int64_t rows, int64_t dim, float eps) {
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * dim;
        float *yr = y + r * dim;
        float ss = 0.f;
        for (int64_t i = 0; i < dim; i++) ss += xr[i] * xr[i];
        const float m = sqrtf(ss / (float)dim + eps);
        for (int64_t i = 0; i < dim; i++) yr[i] = xr[i] / m * g[i];
    }
}

void or_softmax(float *x, int64_t n) {
    float mx = -INFINITY;
    for (int64_t i = 0; i < n; i++) mx = x[i] > mx ? x[i] : mx;
    float s = 0.f;
    for (int64_t i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        s += x[i];
    }
    for (int64_t i = 0; i < n; i++) x[i] /= s;
}

float or_silu(float v) { return (float)((double)v / (or_exp64(-(double)v) + 1.0)); }

int or_argmax(const float *x, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 1; i < n; i++)
        if (x[i] > x[best]) best = i;
    return (int)best;
}

/* -------------------------------------------- synthetic generator ----- */
static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static inline uint64_t synth_hash(uint64_t seed, uint64_t idx) {
    return mix64(mix64(seed) ^ idx);
}
static inline float synth_unit(uint64_t h) { /* [0, 1) with 24 bits */
    return (float)(h >> 40) * (1.0f / 16777216.0f);
}

void or_synth_q4k(uint64_t seed, int64_t nblocks, float sigma, void *out) {
    or_block_q4k *blk = (or_block_q4k *)out;
    uint16_t base = or_f32_to_f16(sigma / 219.0f);
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nblocks; b++) {
        or_block_q4k *y = blk + b;
        uint64_t i0 = (uint64_t)b * 32u;
        for (int w = 0; w < 16; w++) {
            uint64_t h = synth_hash(seed, i0 + (uint64_t)w);
            memcpy(y->qs + 8 * w, &h, 8);
        }
        uint64_t hs = synth_hash(seed, i0 + 16u);
        uint8_t sc[8], mn[8];
        for (int j = 0; j < 8; j++) {
            sc[j] = (uint8_t)(32u + ((hs >> (5 * j)) & 31u));
            mn[j] = (uint8_t)((sc[j] * 15u + 8u) >> 4);
        }
        memset(y->scales, 0, 12);
        for (int j = 0; j < 8; j++) {
            if (j < 4) {
                y->scales[j] = sc[j];
                y->scales[j + 4] = mn[j];
            } else {
                y->scales[j + 4] = (uint8_t)((sc[j] & 0x0F) | ((mn[j] & 0x0F) << 4));
                y->scales[j - 4] |= (uint8_t)((sc[j] >> 4) << 6);
                y->scales[j] |= (uint8_t)((mn[j] >> 4) << 6);
            }
        }
        uint64_t hd = synth_hash(seed, i0 + 17u);
        y->d = (uint16_t)(base + (hd & 15u));
        y->dmin = or_f32_to_f16(8.0f * or_f16_to_f32(y->d));
    }
}

void or_synth_q6k(uint64_t seed, int64_t nblocks, float sigma, void *out) {
    or_block_q6k *blk = (or_block_q6k *)out;
    uint16_t base = or_f32_to_f16(sigma / 1468.0f);
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nblocks; b++) {
        or_block_q6k *y = blk + b;
        uint64_t i0 = (uint64_t)b * 32u;
        for (int w = 0; w < 16; w++) {
            uint64_t h = synth_hash(seed, i0 + (uint64_t)w);
            memcpy(y->ql + 8 * w, &h, 8);
        }
        for (int w = 0; w < 8; w++) {
            uint64_t h = synth_hash(seed, i0 + 16u + (uint64_t)w);
            memcpy(y->qh + 8 * w, &h, 8);
        }
        for (int half = 0; half < 2; half++) {
            uint64_t h = synth_hash(seed, i0 + 24u + (uint64_t)half);
            for (int j = 0; j < 8; j++)
                y->scales[8 * half + j] = (int8_t)(48u + ((h >> (6 * j)) & 63u));
        }
        uint64_t hd = synth_hash(seed, i0 + 26u);
        y->d = (uint16_t)(base + (hd & 15u));
    }
}

void or_synth_f32(uint64_t seed, int64_t n, float mean, float stddev,
                  float *out) {
    float s3 = stddev * 1.7320508f;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        float u = synth_unit(synth_hash(seed, (uint64_t)i));
        out[i] = mean + s3 * (2.0f * u - 1.0f);
    }
}

void or_synth_tokens(uint64_t seed, int64_t n, int32_t vocab, int32_t *out) {
    for (int64_t i = 0; i < n; i++)
        out[i] = (int32_t)(synth_hash(seed, (uint64_t)i) % (uint64_t)vocab);
}

/* --------------------------------------------------------- model ------ */
struct or_model {
    or_config c;
    or_tensor tok_embd, out_norm, output;
    or_layer *layers;
    float *kc, *vc; /* [L][max_ctx][n_kv * head_dim] */
    int len;
    int nthreads;
};

static float round_f16(float v) { return or_f16_to_f32(or_f32_to_f16(v)); }

or_model *or_model_create(const or_config *cfg, const or_tensor *tok_embd,
                          const or_layer *layers, const or_tensor *out_norm,
                          const or_tensor *output, int nthreads) {
    or_model *m = (or_model *)calloc(1, sizeof *m);
    if (!m) return NULL;
    m->c = *cfg;
    m->tok_embd = *tok_embd;
    m->out_norm = *out_norm;
    m->output = *output;
    m->layers = (or_layer *)malloc(sizeof(or_layer) * (size_t)cfg->n_layers);
    memcpy(m->layers, layers, sizeof(or_layer) * (size_t)cfg->n_layers);
    size_t kvn = (size_t)cfg->n_layers * (size_t)cfg->max_ctx *
                 (size_t)cfg->n_kv_heads * (size_t)cfg->head_dim;
    m->kc = (float *)calloc(kvn, sizeof(float));
    m->vc = (float *)calloc(kvn, sizeof(float));
    m->nthreads = nthreads;
    if (!m->kc || !m->vc) {
        or_model_free(m);
        return NULL;
    }
    return m;
}

void or_model_free(or_model *m) {
    if (!m) return;
    free(m->layers);
    free(m->kc);
    free(m->vc);
    free(m);
}

void or_model_clear(or_model *m) { m->len = 0; }
int or_model_length(const or_model *m) { return m->len; }

static int nthreads_of(const or_model *m) {
#ifdef _OPENMP
    return m->nthreads > 0 ? m->nthreads : omp_get_max_threads();
#else
    (void)m;
    return 1;
#endif
}

static void linear(const or_model *m, const or_tensor *w, const float *x,
                   int64_t rows, float *y, int mode) {
    /* mode 2: candle 0.8.4's CUDA QMatMul dispatch -- more than 8 activation
     * rows dequantize the weights and run a float matmul, up to 8 rows take
     * the quantized-activation integer path. */
    if (mode == 2) mode = rows > 8 ? 1 : 0;
    if (mode == 3 && w->dtype != OR_F32) {
        or_qmatmul_candle_f32(w->dtype, w->data, w->rows, w->cols, x, rows, y, m->nthreads);
        return;
    }
    if (w->dtype == OR_F32) {
        const float *wf = (const float *)w->data;
        int nt = nthreads_of(m);
#pragma omp parallel for num_threads(nt) schedule(static)
        for (int64_t c = 0; c < w->rows; c++)
            for (int64_t r = 0; r < rows; r++) {
                float acc = 0.f;
                for (int64_t i = 0; i < w->cols; i++) acc += x[r * w->cols + i] * wf[c * w->cols + i];
                y[r * w->rows + c] = acc;
            }
    } else if (mode == 0) {
        or_qmatmul(w->dtype, w->data, w->rows, w->cols, x, rows, y, m->nthreads);
    } else {
        or_qmatmul_f32(w->dtype, w->data, w->rows, w->cols, x, rows, y, m->nthreads);
    }
}

static void embed_row(const or_tensor *t, int32_t tok, float *out) {
    size_t bb = or_block_bytes(t->dtype);
    int64_t cols = t->cols;
    if (t->dtype == OR_F32) {
        memcpy(out, (const float *)t->data + (size_t)tok * cols, (size_t)cols * 4);
    } else {
        const uint8_t *row = (const uint8_t *)t->data + (size_t)tok * (cols / OR_QK_K) * bb;
        or_dequantize(t->dtype, row, cols, out);
    }
}

int or_model_forward(or_model *m, const int32_t *tokens, int n, int pos,
                     float *logits, int all_logits, int matmul_mode) {
    const or_config *c = &m->c;
    if (n <= 0 || pos < 0 || pos > m->len || pos + n > c->max_ctx) return 1;
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= c->vocab) return 2;
    m->len = pos;
    const int H = c->hidden, hd = c->head_dim, nq = c->n_heads, nkv = c->n_kv_heads;
    const int qd = nq * hd, kd = nkv * hd, F = c->ffn;
    const int grp = nq / nkv;
    float *x = (float *)malloc(sizeof(float) * (size_t)n * H);
    float *h = (float *)malloc(sizeof(float) * (size_t)n * H);
    float *q = (float *)malloc(sizeof(float) * (size_t)n * qd);
    float *k = (float *)malloc(sizeof(float) * (size_t)n * kd);
    float *v = (float *)malloc(sizeof(float) * (size_t)n * kd);
    float *o = (float *)malloc(sizeof(float) * (size_t)n * qd);
    float *t = (float *)malloc(sizeof(float) * (size_t)n * (H > F ? H : F));
    float *g = (float *)malloc(sizeof(float) * (size_t)n * F);
    float *u = (float *)malloc(sizeof(float) * (size_t)n * F);
    for (int i = 0; i < n; i++) embed_row(&m->tok_embd, tokens[i], x + (size_t)i * H);
    const float scale = (float)(1.0 / sqrt((double)hd));
    const int nt = nthreads_of(m);
    const int f32 = matmul_mode == 3;
    void (*norm)(const float *, const float *, float *, int64_t, int64_t, float) = f32 ? rmsnorm_f32 : or_rmsnorm;
    for (int l = 0; l < c->n_layers; l++) {
        const or_layer *L = &m->layers[l];
        norm(x, (const float *)L->attn_norm.data, h, n, H, c->eps);
        linear(m, &L->wq, h, n, q, matmul_mode);
        linear(m, &L->wk, h, n, k, matmul_mode);
        linear(m, &L->wv, h, n, v, matmul_mode);
        for (int i = 0; i < n; i++) {
            float *qi = q + (size_t)i * qd, *ki = k + (size_t)i * kd;
            if (c->qk_norm) {
                norm(qi, (const float *)L->q_norm.data, qi, nq, hd, c->eps);
                norm(ki, (const float *)L->k_norm.data, ki, nkv, hd, c->eps);
            }
            or_rope(qi, nq, hd, pos + i, c->rope_theta, c->rope_mode);
            or_rope(ki, nkv, hd, pos + i, c->rope_theta, c->rope_mode);
            size_t off = ((size_t)l * c->max_ctx + (size_t)(pos + i)) * kd;
            for (int e = 0; e < kd; e++) {
                float kv = ki[e], vv = v[(size_t)i * kd + e];
                m->kc[off + e] = c->kv_f16 ? round_f16(kv) : kv;
                m->vc[off + e] = c->kv_f16 ? round_f16(vv) : vv;
            }
        }
        const float *kl = m->kc + (size_t)l * c->max_ctx * kd;
        const float *vl = m->vc + (size_t)l * c->max_ctx * kd;
#pragma omp parallel for num_threads(nt) collapse(2) schedule(dynamic, 1)
        for (int i = 0; i < n; i++)
            for (int hq = 0; hq < nq; hq++) {
                /* softmax(q.k^T * scale) . v; the score dots in f32 in the
                 * fixed order of or_attn_dot, 16-position unit partials in
                 * f32, their combination in binary64 with one rounding to f32
                 * at the end */
                int T = pos + i + 1, hk = hq / grp;
                const float *qh = q + (size_t)i * qd + (size_t)hq * hd;
                float *sc = (float *)malloc(sizeof(float) * (size_t)T);
                double *pr = (double *)malloc(sizeof(double) * (size_t)(T > hd ? T : hd));
                double *acc = (double *)calloc((size_t)hd, sizeof(double));
                float mx = -INFINITY;
                for (int s = 0; s < T; s++) {
                    const float *ks = kl + (size_t)s * kd + (size_t)hk * hd;
                    if (f32) {
                        float d = 0.f;
                        for (int e = 0; e < hd; e++) d += qh[e] * ks[e];
                        sc[s] = d * scale;
                    } else {
                        sc[s] = or_attn_dot(qh, ks, hd) * scale;
                    }
                    mx = sc[s] > mx ? sc[s] : mx;
                }
                if (f32) {  /* softmax_last_dim then att.v, f32 left to right */
                    float l32 = 0.f;
                    for (int s = 0; s < T; s++) {
                        sc[s] = expf(sc[s] - mx);
                        l32 += sc[s];
                    }
                    float *oh = o + (size_t)i * qd + (size_t)hq * hd;
                    for (int e = 0; e < hd; e++) {
                        float a32 = 0.f;
                        for (int s = 0; s < T; s++) a32 += (sc[s] / l32) * vl[(size_t)s * kd + (size_t)hk * hd + e];
                        oh[e] = a32;
                    }
                    free(sc);
                    free(pr);
                    free(acc);
                    continue;
                }
                /* Positions in units of 16 (16u .. 16u + 15), as the device
                 * kernel splits them: per unit, in f32 and a fixed order, its
                 * max m_u, p_t = f32(exp64(s_t - m_u)), l_u = the pairwise
                 * sum of the 16 slots (absent positions 0) and o_u = the FMA
                 * chain of p_t v_t in position order; the units then combine
                 * in binary64 with weights exp64(m_u - max). */
                double l = 0.0;
                float *ou = (float *)pr; /* hd floats */
                for (int u0 = 0; u0 < T; u0 += 16) {
                    const int nu = T - u0 < 16 ? T - u0 : 16;
                    float mu = -INFINITY, pu[16], tr[16];
                    for (int t = 0; t < nu; t++) mu = sc[u0 + t] > mu ? sc[u0 + t] : mu;
                    for (int t = 0; t < 16; t++)
                        pu[t] = tr[t] = t < nu ? (float)or_exp64((double)sc[u0 + t] - (double)mu) : 0.f;
                    for (int w = 1; w < 16; w *= 2)
                        for (int t = 0; t < 16; t += 2 * w) tr[t] = tr[t] + tr[t + w];
                    for (int e = 0; e < hd; e++) ou[e] = 0.f;
                    for (int t = 0; t < nu; t++) {
                        const float *vs = vl + (size_t)(u0 + t) * kd + (size_t)hk * hd;
                        for (int e = 0; e < hd; e++) ou[e] = fmaf(pu[t], vs[e], ou[e]);
                    }
                    const double w = or_exp64((double)mu - (double)mx);
                    l += w * (double)tr[0];
                    for (int e = 0; e < hd; e++) acc[e] += w * (double)ou[e];
                }
                float *oh = o + (size_t)i * qd + (size_t)hq * hd;
                for (int e = 0; e < hd; e++) oh[e] = (float)(acc[e] / l);
                free(sc);
                free(pr);
                free(acc);
            }
        linear(m, &L->wo, o, n, t, matmul_mode);
        for (size_t e = 0; e < (size_t)n * H; e++) x[e] = t[e] + x[e];
        norm(x, (const float *)L->ffn_norm.data, h, n, H, c->eps);
        linear(m, &L->w_gate, h, n, g, matmul_mode);
        linear(m, &L->w_up, h, n, u, matmul_mode);
        for (size_t e = 0; e < (size_t)n * F; e++)
            g[e] = (f32 ? g[e] / (1.0f + expf(-g[e])) : or_silu(g[e])) * u[e];
        linear(m, &L->w_down, g, n, t, matmul_mode);
        for (size_t e = 0; e < (size_t)n * H; e++) x[e] = t[e] + x[e];
    }
    m->len = pos + n;
    int first = all_logits ? 0 : n - 1;
    int rows = n - first;
    norm(x + (size_t)first * H, (const float *)m->out_norm.data, h, rows, H, c->eps);
    linear(m, &m->output, h, rows, logits, matmul_mode);
    free(x); free(h); free(q); free(k); free(v); free(o); free(t); free(g); free(u);
    return 0;
}

int or_model_synth_kv(or_model *m, uint64_t seed, int ctx, float scale) {
    const or_config *c = &m->c;
    if (ctx < 0 || ctx > c->max_ctx) return 1;
    const int kd = c->n_kv_heads * c->head_dim;
    const float s3 = scale * 1.7320508f;
    int nt = nthreads_of(m);
#pragma omp parallel for num_threads(nt) collapse(2) schedule(static)
    for (int l = 0; l < c->n_layers; l++)
        for (int p = 0; p < ctx; p++)
            for (int which = 0; which < 2; which++) {
                float *dst = (which ? m->vc : m->kc) + ((size_t)l * c->max_ctx + (size_t)p) * kd;
                for (int e = 0; e < kd; e++) {
                    uint64_t idx = (((uint64_t)l * 2u + (uint64_t)which) << 40) |
                                   ((uint64_t)p << 20) | (uint64_t)e;
                    float u = synth_unit(synth_hash(seed, idx));
                    dst[e] = round_f16(s3 * (2.0f * u - 1.0f));
                }
            }
    m->len = ctx;
    return 0;
}

int or_model_read_kv(const or_model *m, int layer, int which, int pos,
                     float *out) {
    const or_config *c = &m->c;
    if (layer < 0 || layer >= c->n_layers || pos < 0 || pos >= c->max_ctx) return 1;
    const int kd = c->n_kv_heads * c->head_dim;
    const float *src = (which ? m->vc : m->kc) + ((size_t)layer * c->max_ctx + (size_t)pos) * kd;
    memcpy(out, src, sizeof(float) * (size_t)kd);
    return 0;
}
