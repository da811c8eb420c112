/*
 * CPU oracle for the quantized decode/prefill path — TEST INFRASTRUCTURE ONLY.
 *
 * This library restates, in plain C, the arithmetic that ferrite-llm's candle
 * backend runs for a quantized Llama/Qwen forward:
 *   - GGUF k-quant block formats Q4_K / Q6_K / Q8_K
 *     (layouts as declared in ferrite-os/crates/internal/ptx-kernels/kernels/
 *      candle/quantized.cu:388-393 (block_q4_K), :419-424 (block_q6_K),
 *      :428-432 (block_q8_K));
 *   - dequantization (quantized.cu:925-1022 get_scale_min_k4 + q4_K,
 *     :1024-1129 q6_K);
 *   - candle-core 0.8.4 CPU QMatMul: activations quantized to Q8_K, integer
 *     vec_dot per output feature (candle-core 0.8.4 src/quantized/k_quants.rs,
 *     a crates.io dependency pinned at Cargo.lock:598-601, not vendored in the
 *     reference tree — restated from the published ggml k-quant algorithm);
 *   - candle-nn 0.8.4 rms_norm / softmax_last_dim / rope_i and the
 *     candle-transformers 0.8.4 quantized_llama forward
 *     (call site crates/ferrite-wasm-host/src/adapter.rs:41-70), plus the Qwen3
 *     additions (per-head QK RMSNorm, rotate-half RoPE).
 *
 * Only tests/, the smoke check and the CPU-baseline leg of the bench may load
 * this library, and only as the checker: it is never the product path.
 *
 * Parity pinning: the reference's own tests hold no vectors for this path.
 * Dequantization is pinned against the reference's vendored CUDA k-quant
 * kernels (quantized.cu, compiled from the reference sources into oracle/_ref
 * and run on a B200; fixtures under tests/golden/). Q8_K activation
 * quantization and the integer vec_dot decomposition are restated from the
 * published algorithm and cross-checked by identities (integer dot ==
 * float dot of the dequantized operands); they are not pinned by reference
 * vectors because candle's CPU k_quants.rs is not present.
 */
#ifndef FERRITE_ORACLE_H
#define FERRITE_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OR_QK_K 256

/* dtype tags (same numbering as the GGML type ids for the k-quants). */
enum { OR_F32 = 0, OR_F16 = 1, OR_Q4_K = 12, OR_Q6_K = 14, OR_Q8_K = 15 };

typedef struct {            /* 144 bytes */
    uint16_t d;             /* fp16 super-block scale for the 6-bit scales */
    uint16_t dmin;          /* fp16 super-block scale for the 6-bit mins */
    uint8_t scales[12];     /* 8 scales + 8 mins, 6 bits each, packed */
    uint8_t qs[128];        /* 256 4-bit quants */
} or_block_q4k;

typedef struct {            /* 210 bytes */
    uint8_t ql[128];        /* low 4 bits */
    uint8_t qh[64];         /* high 2 bits */
    int8_t scales[16];      /* one int8 scale per 16 weights */
    uint16_t d;             /* fp16 super-block scale */
} or_block_q6k;

typedef struct {            /* 292 bytes */
    float d;
    int8_t qs[256];
    int16_t bsums[16];      /* sums of qs in groups of 16 */
} or_block_q8k;

size_t or_block_bytes(int dtype);

/* fp16 <-> f32 (IEEE binary16, round to nearest even). */
float or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_f16(float f);

/* f32 -> k-quant (n must be a multiple of 256). */
void or_quantize_q4k(const float *x, int64_t n, void *out);
void or_quantize_q6k(const float *x, int64_t n, void *out);
/* round_mode 0 = half away from zero (Rust f32::round), 1 = half to even. */
void or_quantize_q8k(const float *x, int64_t n, void *out, int round_mode);

/* k-quant -> f32. */
void or_dequantize(int dtype, const void *blocks, int64_t n, float *y);

/* Scalar vec_dot of one weight row (n values) with one Q8_K row. */
float or_vec_dot(int dtype, int64_t n, const void *w, const void *a);

/* Integer partials of every (row, super-block) pair of W[nrows, k] against
 * one Q8_K activation row.  Q4_K: out_sc = sum_j sc_j * dot_j,
 * out_min = sum_j m_j * (bsum_{2j} + bsum_{2j+1}).  Q6_K: out_sc =
 * sum_j sc_j * dot_j over 16 groups (quants centred at -32), out_min = 0. */
void or_block_dots(int dtype, int64_t nrows, int64_t k, const void *w,
                   const void *a, int32_t *out_sc, int32_t *out_min);

/* candle CPU QMatMul: y[m, n] = x[m, k] . W[n, k]^T with x quantized to Q8_K
 * row by row, then vec_dot per output feature.  nthreads <= 0 = all cores. */
void or_qmatmul(int dtype, const void *w, int64_t n, int64_t k,
                const float *x, int64_t m, float *y, int nthreads);

/* Dequantize-then-f32 matmul (the large-batch form: no activation
 * quantization).  Used as the oracle for the prefill GEMM. */
/* Unrounded binary64 row sums of or_qmatmul (tensor-parallel partials). */
double or_vec_dot64(int dtype, int64_t n, const void *w, const void *a);
/* candle's own f32 combine of the same integer partials (8 lane sums). */
float or_vec_dot_candle_f32(int dtype, int64_t n, const void *w, const void *a);
void or_qmatmul_candle_f32(int dtype, const void *w, int64_t n, int64_t k, const float *x, int64_t m, float *y,
                           int nthreads);
void or_qmatmul64(int dtype, const void *w, int64_t n, int64_t k,
                  const float *x, int64_t m, double *y, int nthreads);
void or_qmatmul_f32(int dtype, const void *w, int64_t n, int64_t k,
                    const float *x, int64_t m, float *y, int nthreads);

/* ---------------------------------------------------------------- ops ---- */
void or_rmsnorm(const float *x, const float *g, float *y, int64_t rows,
                int64_t dim, float eps);
/* mode 0 = interleaved pairs (candle rope_i), 1 = rotate-half (NEOX). */
void or_rope(float *x, int64_t n_heads, int64_t head_dim, int64_t pos,
             float theta, int mode);
void or_softmax(float *x, int64_t n);
float or_silu(float x);
/* exp in binary64: Cody-Waite reduction x = k ln2 + r, Taylor polynomial of
 * degree 13 in r (|r| <= ln2/2, truncation < 5e-18), scaling by 2^k.  The
 * device path evaluates the same operations, so both sides agree bit for
 * bit. */
double or_exp64(double x);
/* per-weight dequantization factors (w = scale * q - offset, exact f32 products) */
void or_dequant_parts(int dtype, const void *blocks, int64_t n, float *scale, float *offset, int8_t *q);
/* attention score dot in f32: 8 slices of hd/8 dims (fmaf chains), summed in order */
float or_attn_dot(const float *q, const float *k, int hd);

/* -------------------------------------------------------------- model ---- */
typedef struct {
    int n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab;
    int max_ctx;
    float rope_theta, eps;
    int qk_norm;        /* 1: Qwen3 per-head RMSNorm on q and k */
    int rope_mode;      /* 0 interleaved (llama-compat), 1 rotate-half (qwen3) */
    int kv_f16;         /* 1: KV cache stored as fp16 (rounded), 0: f32 */
} or_config;

typedef struct {
    int dtype;          /* OR_F32, OR_Q4_K, OR_Q6_K */
    int64_t rows, cols; /* [rows, cols]: rows = output features */
    const void *data;   /* caller-owned; must outlive the model */
} or_tensor;

typedef struct {
    or_tensor attn_norm, wq, wk, wv, wo, q_norm, k_norm;
    or_tensor ffn_norm, w_gate, w_up, w_down;
} or_layer;

typedef struct or_model or_model;

or_model *or_model_create(const or_config *cfg, const or_tensor *tok_embd,
                          const or_layer *layers, const or_tensor *out_norm,
                          const or_tensor *output, int nthreads);
void or_model_free(or_model *m);
void or_model_clear(or_model *m);
/* Runs tokens[0..n) at positions pos..pos+n-1 (causal), appending to the KV
 * cache.  logits: [n, vocab] when all_logits, else [vocab] for the last token.
 * matmul_mode 0 = Q8_K integer path (decode), 1 = dequantize + f32 matmul
 * (prefill form), 2 = per call by row count as candle's CUDA QMatMul
 * dispatches (> 8 rows float, else integer), 3 = candle's f32 CPU order
 * throughout: the Q8_K integer path with candle's f32 lane combine, RMSNorm
 * sums of squares, attention dots, softmax sums and P.V in f32 left to
 * right, f32 exp in softmax and SiLU -- no binary64 step (measures the
 * binary64 oracle's distance from candle's float arithmetic).  Returns 0 on
 * success. */
int or_model_forward(or_model *m, const int32_t *tokens, int n, int pos,
                     float *logits, int all_logits, int matmul_mode);
/* Fill the first ctx KV positions of every layer with synthetic values
 * (same generator as the product's fb_synth_kv) and set the length. */
int or_model_synth_kv(or_model *m, uint64_t seed, int ctx, float scale);
/* Read back a KV row: which 0 = K, 1 = V; out [n_kv_heads * head_dim]. */
int or_model_read_kv(const or_model *m, int layer, int which, int pos,
                     float *out);
int or_model_length(const or_model *m);
int or_argmax(const float *x, int64_t n);

/* -------------------------------------------- synthetic weight generator -- */
/* Restatement of the product's counter-based generator (splitmix64 hashing
 * of (seed, index)); used to build identical random-init tensors on the CPU
 * for the CPU baseline and for parity checks of the device generator. */
void or_synth_q4k(uint64_t seed, int64_t nblocks, float sigma, void *out);
void or_synth_q6k(uint64_t seed, int64_t nblocks, float sigma, void *out);
void or_synth_f32(uint64_t seed, int64_t n, float mean, float stddev,
                  float *out);
void or_synth_tokens(uint64_t seed, int64_t n, int32_t vocab, int32_t *out);

#ifdef __cplusplus
}
#endif
#endif
