/*
 * ferrite_b200 — C ABI of the B200 (sm_100a) quantized decode/prefill path.
 *
 * The entry points replace the arithmetic behind ferrite-llm's candle-backend
 * quantized Llama/Qwen forward.  Reference interfaces they stand in for:
 *   - QTensor / QMatMul (candle-core 0.8.4, quantized/mod.rs; constructed by
 *     quantized_llama::ModelWeights::from_gguf at
 *     crates/ferrite-wasm-host/src/adapter.rs:47-55, called per layer from
 *     the forward at adapter.rs:61-70)            -> fb_qtensor_*, fb_qmatmul
 *   - GGUF k-quant blocks block_q4_K / block_q6_K / block_q8_K
 *     (ferrite-os/crates/internal/ptx-kernels/kernels/candle/
 *      quantized.cu:388-393, :419-424, :428-432)  -> FB_Q4_K / FB_Q6_K / FB_Q8_K
 *   - QTensor::dequantize / dequantize_block_q4_K|q6_K_{f32,f16}
 *     (quantized.cu:936-1151)                      -> fb_dequantize
 *   - candle-nn rms_norm / rope_i / rope / softmax / silu
 *     (ptx-kernels/kernels/candle/reduce.cu:189-345, unary.cu:59)
 *                                                  -> fb_rmsnorm, fb_rope,
 *                                                     fb_attn_decode, fb_swiglu
 *   - ferrite_core::InferenceModel { forward, prefill, clear_cache }
 *     (crates/ferrite-core/src/generation.rs:187-195; implemented for candle
 *      at adapter.rs:60-93)                        -> fb_model_forward,
 *                                                     fb_model_prefill,
 *                                                     fb_model_clear_cache
 *   - Sampler::argmax greedy path (crates/ferrite-core/src/sampling.rs:108-112)
 *                                                  -> fb_model_decode_greedy
 *
 * Conventions: every function returns 0 (FB_OK) or a negative FB_ERR_* code
 * and records a message readable with fb_last_error() (thread-local).  No
 * call aborts or exits.  Pointers named *_dev are device pointers; *_host are
 * host pointers.  All device work is ordered on the context's stream; only
 * fb_sync and the *_host model calls synchronise.  One context per host
 * thread / stream; handles are not thread-safe.
 */
#ifndef FERRITE_B200_H
#define FERRITE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FB_ABI_VERSION 1

enum fb_status {
    FB_OK = 0,
    FB_ERR_INVALID = -1,   /* bad argument (shape, dtype, null pointer) */
    FB_ERR_CUDA = -2,      /* a CUDA runtime call failed */
    FB_ERR_OOM = -3,       /* device allocation failed */
    FB_ERR_DEVICE = -4,    /* a kernel reported an error through the error word */
    FB_ERR_NCCL = -5,      /* a collective failed or timed out */
    FB_ERR_STATE = -6      /* call not valid in the current state */
};

/* dtype ids follow the GGML type numbering for the k-quants. */
enum fb_dtype {
    FB_F32 = 0,
    FB_F16 = 1,
    FB_Q4_K = 12,
    FB_Q6_K = 14,
    FB_Q8_K = 15,
    FB_BF16 = 30
};

typedef struct fb_ctx fb_ctx;
typedef struct fb_qtensor fb_qtensor;
typedef struct fb_model fb_model;

/* ------------------------------------------------------------ context --- */
const char *fb_last_error(void);
int fb_abi_version(void);
/* stream: the cudaStream_t all work of this context is ordered on, used as
 * given (NULL = the CUDA default stream).  Model steps replay their CUDA
 * graph on a private stream joined to this one by events. */
int fb_ctx_create(int device, void *stream, fb_ctx **out);
int fb_ctx_destroy(fb_ctx *ctx);
int fb_ctx_set_stream(fb_ctx *ctx, void *stream);
void *fb_ctx_stream(fb_ctx *ctx);
int fb_sync(fb_ctx *ctx);
/* Reads and clears the device error word (bit flags set by kernels whose
 * bounded waits ran out or whose inputs failed a device-side check). */
int fb_ctx_error_word(fb_ctx *ctx, uint32_t *flags);
/* Programmatic dependent launch between consecutive kernels (default on). */
int fb_ctx_set_pdl(fb_ctx *ctx, int enable);
/* Prompt passes of 512 rows or more dequantize each Q4_K / Q6_K projection
 * to fp16 before its tensor-core GEMM.  With the cache on (the default) the
 * first such pass keeps each tensor's fp16 copy (2 bytes per weight, freed
 * with the tensor) while at least max(16 GiB, a quarter of the device) stays
 * free, and later passes skip the dequantization; enable = 0 dequantizes on
 * every pass and keeps nothing.  No reference counterpart (candle's CUDA
 * path dequantizes on every call). */
int fb_ctx_set_prefill_weight_cache(fb_ctx *ctx, int enable);

/* ------------------------------------------------------------ QTensor --- */
/* A weight matrix W[n, k] (n output features, k inputs, k % 256 == 0 for
 * k-quants) held in device memory.  host_blocks holds GGUF blocks in row
 * order (n * k/256 blocks).  The device copy is re-laid out for the GEMV;
 * fb_qtensor_download returns the original GGUF bytes. */
int fb_qtensor_upload(fb_ctx *ctx, int dtype, int64_t n, int64_t k,
                      const void *host_blocks, fb_qtensor **out);
int fb_qtensor_upload_dev(fb_ctx *ctx, int dtype, int64_t n, int64_t k,
                          const void *dev_blocks, fb_qtensor **out);
/* Random-init weights generated on the device (counter-based hash of
 * (seed, block index); sigma = target standard deviation). */
int fb_qtensor_synth(fb_ctx *ctx, int dtype, int64_t n, int64_t k,
                     uint64_t seed, float sigma, fb_qtensor **out);
/* Stacks the rows of several tensors of one dtype and k (fused QKV, gate/up). */
int fb_qtensor_concat_rows(fb_ctx *ctx, const fb_qtensor *const *parts,
                           int nparts, fb_qtensor **out);
/* Uploads the sub-matrix W[row0 : row0+rows, col0 : col0+cols] of a GGUF
 * tensor W[n, k] given in full (blocks in row order; on the host when
 * src_on_device == 0, else in device memory).  col0 and cols are multiples
 * of 256 (whole super-blocks), so the slice's blocks are the source's bytes.
 * Tensor-parallel shards: a row slice is a column-parallel shard (split
 * output features), a column slice a row-parallel shard (split inputs). */
int fb_qtensor_upload_slice(fb_ctx *ctx, int dtype, int64_t n, int64_t k,
                            const void *src_blocks, int src_on_device,
                            int64_t row0, int64_t rows, int64_t col0,
                            int64_t cols, fb_qtensor **out);
int fb_qtensor_info(const fb_qtensor *t, int *dtype, int64_t *n, int64_t *k,
                    int64_t *device_bytes);
int fb_qtensor_download(fb_ctx *ctx, const fb_qtensor *t, void *host_blocks);
int fb_qtensor_destroy(fb_qtensor *t);
/* W -> dense [n, k] in out_dtype (FB_F32, FB_F16 or FB_BF16). */
int fb_dequantize(fb_ctx *ctx, const fb_qtensor *t, void *out_dev,
                  int out_dtype);

/* ------------------------------------------------------------ QMatMul --- */
/* y[m, n] = x[m, k] . W[n, k]^T, f32 in and out.  m <= 16: activations are
 * quantized to Q8_K and dotted in integer arithmetic (candle's CPU QMatMul);
 * m > 16: the prefill path (W dequantized to 16-bit tiles on chip, tensor-core
 * MMA with f32 accumulation). */
int fb_qmatmul(fb_ctx *ctx, const fb_qtensor *w, const float *x_dev,
               float *y_dev, int64_t m);
/* Forces the Q8_K integer path for any m (chunks of 16 rows). */
int fb_qmatmul_q8k(fb_ctx *ctx, const fb_qtensor *w, const float *x_dev,
                   float *y_dev, int64_t m);
/* f32 [m, k] -> GGUF block_q8_K array (m * k/256 blocks of 292 bytes). */
int fb_quantize_q8k(fb_ctx *ctx, const float *x_dev, int64_t m, int64_t k,
                    void *q8k_dev);
/* Integer partials of W[n, k] against one activation row x[k] (quantized to
 * Q8_K on the device): per (row, super-block) sum_j sc_j*dot_j and, for
 * Q4_K, sum_j m_j*bsum_j.  out_* are int32 [n, k/256]. */
int fb_block_dots(fb_ctx *ctx, const fb_qtensor *w, const float *x_dev,
                  int32_t *out_sc_dev, int32_t *out_min_dev);

/* ---------------------------------------------------------------- ops --- */
/* y = x / sqrt(mean(x^2) + eps) * g, rows of length dim. */
int fb_rmsnorm(fb_ctx *ctx, const float *x_dev, const float *g_dev,
               float *y_dev, int64_t rows, int64_t dim, float eps);
/* In-place RoPE of x[n_tok, n_heads, head_dim] at positions pos0 + t.
 * mode 0 = interleaved pairs (candle rope_i), 1 = rotate-half (NEOX). */
int fb_rope(fb_ctx *ctx, float *x_dev, int64_t n_tok, int64_t n_heads,
            int64_t head_dim, int64_t pos0, float theta, int mode);
/* out[m, f] = silu(gate[m, f]) * up[m, f]. */
int fb_swiglu(fb_ctx *ctx, const float *gate_dev, const float *up_dev,
              float *out_dev, int64_t m, int64_t f);
/* GQA decode attention of one query token per sequence over a paged fp16 KV
 * cache.  q[b, n_heads, head_dim] f32; K pages fp16 dim-major
 * [num_pages, n_kv_heads, head_dim, page_size]; V pages fp16
 * [num_pages, n_kv_heads, page_size, head_dim]; block_table[b, max_pages]
 * int32 physical page ids, each checked against num_pages (the pages the
 * K and V pools hold): an id outside [0, num_pages) is not read, its tokens
 * are skipped and the context's error word gets its bad-page bit
 * (fb_ctx_error_word); seq_lens[b] int32 (tokens to attend, including the
 * current one); out[b, n_heads, head_dim] f32.  scale = 1/sqrt(hd).
 * head_dim 128, page_size 32 or 64, n_heads / n_kv_heads in {1, 2, 4, 8}.
 * Allocates nothing when the GPU can hold a 16-CTA thread-block cluster
 * (the split merge runs in distributed shared memory); otherwise grows a
 * workspace once (cudaMalloc plus a stream synchronisation). */
int fb_attn_decode(fb_ctx *ctx, const float *q_dev, const void *k_pages_dev,
                   const void *v_pages_dev, const int32_t *block_table_dev,
                   const int32_t *seq_lens_dev, float *out_dev, int batch,
                   int n_heads, int n_kv_heads, int head_dim, int page_size,
                   int max_pages, int num_pages, int max_seq_len,
                   float scale);

/* Causal attention of a prompt chunk: n_tokens queries q_dev [n_tokens]
 * [n_heads][128] at positions pos0 .. pos0 + n_tokens - 1 of one sequence
 * (block_table_dev: its max_pages page ids) over the cache pages, which must
 * already hold positions 0 .. pos0 + n_tokens - 1 (K dim-major, V
 * token-major, page_size 64); out_dev [n_tokens][n_heads][128] f32.
 * Tensor cores (fp16 operands with q and the probabilities split into two
 * fp16 parts, f32 accumulation).  Replaces the prompt pass of candle's
 * quantized_llama attention (adapter.rs:61-70 with all prompt tokens). */
int fb_attn_prefill(fb_ctx *ctx, const float *q_dev, const void *k_pages_dev,
                    const void *v_pages_dev, const int32_t *block_table_dev,
                    int max_pages, int num_pages, int pos0, int n_tokens,
                    int n_heads, int n_kv_heads, int head_dim, int page_size,
                    float scale, float *out_dev);

/* Same computation and arguments as fb_attn_decode, for callers that cannot
 * allocate device memory: no reference counterpart (the reference's candle
 * path allocates freely).  fb_attn_decode may grow a workspace with
 * cudaMalloc (plus a stream synchronisation) on first use; code that runs
 * under a pooled or hooked device allocator that forbids direct
 * cudaMalloc/cudaFree, or in a loop that must not take the synchronisation
 * those calls can imply, uses this entry point instead.  It allocates
 * nothing: its split scratch (16 splits per kv head and sequence) is a fixed
 * 4 MiB array in the library's device image, so it accepts
 * batch * n_heads * 16 * (head_dim + 2) * 8 bytes plus the merge counters,
 * round_up(batch * n_kv_heads * 4, 256) bytes, <= 4 MiB (e.g. batch 7 with
 * 32 heads and 8 kv heads, any context length) and returns FB_ERR_INVALID
 * beyond that.  Its first call on a device looks up the array's
 * device address (make that first call before any stream capture).  All calls
 * on a device share the array, so calls that overlap on the GPU race. */
int fb_attn_decode_noalloc(fb_ctx *ctx, const float *q_dev,
                           const void *k_pages_dev, const void *v_pages_dev,
                           const int32_t *block_table_dev,
                           const int32_t *seq_lens_dev, float *out_dev,
                           int batch, int n_heads, int n_kv_heads,
                           int head_dim, int page_size, int max_pages,
                           int num_pages, int max_seq_len, float scale);

/* -------------------------------------------------------------- model --- */
typedef struct {
    int n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab;
    int max_ctx;      /* KV capacity per sequence (tokens) */
    int max_batch;    /* decode batch capacity (1..32) */
    float rope_theta, eps;
    int qk_norm;      /* 1: Qwen3 per-head RMSNorm on q and k */
    int rope_mode;    /* 0 interleaved (llama), 1 rotate-half (qwen3) */
} fb_model_config;

int fb_model_create(fb_ctx *ctx, const fb_model_config *cfg, fb_model **out);
int fb_model_destroy(fb_model *m);
/* GGUF tensor names: "token_embd", "output_norm", "output", and per layer
 * "attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "attn_q_norm",
 * "attn_k_norm", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down" (layer >= 0).
 * data_host: GGUF blocks for k-quants, f32 values for FB_F32. */
int fb_model_set_tensor(fb_model *m, const char *name, int layer, int dtype,
                        int64_t rows, int64_t cols, const void *data_host);
/* Random-init every tensor on the device: linear layers Q4_K except
 * ffn_down / output (Q6_K), i.e. a Q4_K_M-like mix; norms 1 + U(+-0.02*sqrt3). */
int fb_model_synth(fb_model *m, uint64_t seed);
/* Must be called after all tensors are set (fuses QKV and gate/up). */
int fb_model_finalize(fb_model *m);
/* InferenceModel::forward for one sequence: tokens_host[n] at positions
 * pos..pos+n-1; logits of the last token -> logits_host[vocab] (may be NULL).
 * n >= 17 (single GPU) runs as a batched prefill: the projections as
 * tensor-core GEMMs over chunks of up to 2048 rows, causal prefill attention,
 * then the last row through the decode step's final norm, lm_head and argmax;
 * shorter inputs (and tensor-parallel models) go token by token. */
int fb_model_forward(fb_model *m, const int32_t *tokens_host, int n, int pos,
                     float *logits_host);
/* Greedy decode step for a batch: tokens_host[b] at positions pos_host[b]
 * (sequence i uses KV slot i); writes argmax ids to next_host[b]. */
int fb_model_decode_greedy(fb_model *m, const int32_t *tokens_host,
                           const int32_t *pos_host, int batch,
                           int32_t *next_host);
/* Device-resident form of the same step (inputs and outputs on the device,
 * no synchronisation; replays a captured CUDA graph when available). */
int fb_model_decode_dev(fb_model *m, const int32_t *tokens_dev,
                        const int32_t *pos_dev, int batch, int32_t *next_dev,
                        float *logits_dev);
int fb_model_prefill(fb_model *m, const int32_t *tokens_host, int n,
                     float *logits_host);
/* Multi-token forward (speculative verification, re-prefill after a context
 * slide; the reference runs these token by token: crates/ferrite-core/src/
 * generation.rs:340-535, chat_session.rs:576-629): like fb_model_forward but
 * logits_host receives the logits of every token, [n][vocab] (the rank's
 * vocab slice under tensor parallelism).  n >= 17 on one GPU: batched, the
 * lm_head as a tensor-core GEMM over the final-normed rows (fp16 operands,
 * f32 accumulation); otherwise token by token through the decode step. */
int fb_model_forward_all(fb_model *m, const int32_t *tokens_host, int n,
                         int pos, float *logits_host);
int fb_model_clear_cache(fb_model *m);
/* Fill the first ctx positions of every sequence slot's KV cache with
 * synthetic fp16 values (bench / parity setup). */
int fb_model_synth_kv(fb_model *m, uint64_t seed, int ctx, float scale);
/* Reads one KV row (which 0 = K, 1 = V) of slot 0 as f32 [n_kv*head_dim]. */
int fb_model_read_kv(fb_model *m, int layer, int which, int pos,
                     float *out_host);
int fb_model_weight_bytes(const fb_model *m, int64_t *bytes);
/* Kernel classes of one decode step, for fb_model_profile (QK-norm, RoPE
 * and the KV write run inside the attention kernel: FB_PROF_ROPE_KV stays 0). */
enum fb_prof_kind {
    FB_PROF_EMBED_NORM = 0, FB_PROF_QKV = 1, FB_PROF_ROPE_KV = 2, FB_PROF_ATTN = 3,
    FB_PROF_O = 4, FB_PROF_NORM = 5, FB_PROF_GATE_UP = 6, FB_PROF_SWIGLU = 7,
    FB_PROF_DOWN = 8, FB_PROF_LM_HEAD = 9, FB_PROF_ARGMAX = 10, FB_PROF_KINDS = 11
};
/* Runs `steps` eager decode steps (batch rows, device-resident inputs as in
 * fb_model_decode_dev) with a CUDA event after every kernel class and writes
 * the summed milliseconds per class into ms_out[FB_PROF_KINDS] and the
 * launches per class into launches_out[FB_PROF_KINDS] (per step).  Kernels
 * run serialised, without PDL overlap. */
int fb_model_profile(fb_model *m, const int32_t *tokens_dev,
                     const int32_t *pos_dev, int batch, int steps,
                     float *ms_out, int *launches_out);
/* Kernels the last decode step launched (graph nodes of the captured step;
 * before any step, the kernel-chain count). */
int fb_model_launches_per_step(const fb_model *m, int *launches);
/* Selects how a single-GPU batch-1 decode step runs: enable = 1 as one
 * persistent cooperative kernel that streams every layer's weights and KV
 * pages through shared memory across grid barriers (plus the argmax kernel),
 * enable = 0 (default, faster on B200) as the chain of per-op kernels.  Both
 * compute the same values.  *supported (may be NULL) tells whether the model's shape allows
 * the persistent kernel (GQA group 2, 4 or 8; Q4_K / Q6_K tensors; not
 * tensor parallel); batches above 1 always run the chain.  No reference
 * counterpart: candle runs one kernel per op. */
int fb_model_set_persistent(fb_model *m, int enable, int *supported);
/* Runs one batch-1 persistent decode step eagerly (device-resident token and
 * position as in fb_model_decode_dev) and returns its phase timeline:
 * stamps_host[(cta * (n_layers + 1) + layer) * 16 + k] = %globaltimer (ns)
 * when CTA cta's consumers finished phase k of layer `layer` (k: 0 norm,
 * 1 QKV, 2 barrier, 3 attention, 4 barrier, 5 O, 6 barrier, 7 norm, 8
 * gate/up, 9 barrier, 10 SwiGLU, 11 barrier, 12 down, 13 barrier; slot 15 of
 * layer 0 = kernel start; layer n_layers: 0 final norm, 1 lm_head), 0 where
 * not reached.  capacity >= num_sms * (n_layers + 1) * 16. */
int fb_model_step_timeline(fb_model *m, const int32_t *tokens_dev,
                           const int32_t *pos_dev, uint64_t *stamps_host,
                           int64_t capacity, int *ctas_out, int *slots_out);
/* Diagnostic read of the last decode step's f32 activations of batch row
 * `row` (values of the last layer for per-layer buffers): "x" (residual
 * stream, hidden), "qkv", "q" (after QK-norm + RoPE), "attn" (attention
 * output, n_heads*head_dim), "o" (output projection), "gate_up" (2*ffn),
 * "down", "logits".  count must equal the buffer's row length. */
int fb_model_read_activation(fb_model *m, const char *name, int row,
                             float *out_host, int64_t count);

/* --------------------------------------------------------- sampling ---
 * Sampler::sample of the reference (crates/ferrite-core/src/sampling.rs:
 * 61-239; config fields as its SamplerConfig): repetition penalty over the
 * distinct previous tokens, temperature == 0 -> argmax, else softmax of
 * logits / temperature, min-p, top-p, top-k (each renormalizing), and a draw
 * with the reference's xorshift64 uniform (rng_state is advanced in place,
 * seeded with SamplerConfig::seed).  logits_dev: one row of vocab f32 on the
 * device (e.g. fb_model_decode_dev's logits); the token is returned on the
 * host.  Runs on the device (one CTA); sorting is replaced by threshold
 * searches with the same keep rules (ties in index order). */
typedef struct {
    double temperature, top_p;
    int top_k;
    float min_p, repetition_penalty;
} fb_sampler_config;
int fb_sample(fb_ctx *ctx, const float *logits_dev, int vocab,
              const fb_sampler_config *cfg, const int32_t *prev_tokens_host,
              int n_prev, uint64_t *rng_state, int32_t *token_out);
/* Top-k logits candidates of each row for the logits-hook path: the k
 * largest logits of logits_dev [rows][vocab] in the order of the reference's
 * stable descending sort (larger logit first, equal logits in index order),
 * ids_dev [rows][k] int32 and vals_dev [rows][k] f32 on the device (stream
 * ordered, no synchronisation).  Replaces top_logits_candidates
 * (crates/ferrite-core/src/hooks.rs:19-38), which copies the row to the host
 * and sorts all of it, as used with GpuLogitsExecutor::WIDTH = 16
 * (crates/ferrite-wasm-host/src/adapter.rs:508-515).  k in 1..16 (the
 * reference takes limit.max(1)); rows with fewer than k selectable entries
 * are padded with id -1, value -inf; NaN logits are never selected.
 * ceil(vocab / 2048) * k <= 2048 (vocab 262144 at k = 16). */
int fb_top_logits(fb_ctx *ctx, const float *logits_dev, int rows,
                  int64_t vocab, int k, int32_t *ids_dev, float *vals_dev);

/* ------------------------------------------------------ GGUF ingest ---
 * Replaces candle's gguf_file::Content + ModelWeights::from_gguf
 * (crates/ferrite-wasm-host/src/adapter.rs:48-54) and the reference's
 * metadata reader (crates/ferrite-core/src/registry/loader.rs:247-339).
 * fb_gguf_config reads a GGUF v2/v3 file's metadata into a model config
 * (architecture "llama" -> arch 0, "qwen3" -> arch 1 with qk_norm and
 * rotate-half RoPE; max_ctx = the file's context_length, max_batch = 1: set
 * both before fb_model_create).  fb_model_load_gguf reads every tensor of the
 * file into a created model (full tensors; a tensor-parallel model keeps its
 * shard), uses token_embd as the lm_head when the file has no output tensor,
 * and finalizes the model.  Tensor types: F32, Q4_K, Q6_K. */
int fb_gguf_config(const char *path, fb_model_config *cfg_out, int *arch_out);
int fb_model_load_gguf(fb_model *m, const char *path);

/* ------------------------------------------------- tensor parallelism ---
 * One process (one fb_ctx) per GPU of a node; the reference has no tensor
 * parallelism (candle runs on one device) and its multi-GPU primitives are
 * peer copies with gather-to-root reductions (ferrite-os/native/core/runtime/
 * modules/hot_multi_gpu_primitives.inl:99-123, hot_multi_gpu_reduction.inl).
 *
 * fb_comm is a device region per rank (exchange inboxes and flags) that
 * every rank maps through CUDA IPC.  Setup: fb_comm_create on each rank,
 * fb_comm_handle -> exchange the FB_COMM_HANDLE_BYTES blobs between the
 * processes (any host channel), fb_comm_open with all world handles in rank
 * order.  The ranks must be started in step (a host barrier) before the
 * first decode step; the device waits on peers are bounded (about 10 s),
 * after which a kernel sets the error word and the step's output is
 * undefined.
 *
 * A model created with fb_model_create_tp takes the FULL model config and
 * full tensors in fb_model_set_tensor / fb_model_synth and keeps its shard:
 * attn_q / attn_k / attn_v rows of its n_heads/world query and
 * n_kv_heads/world kv heads, ffn_gate / ffn_up rows and ffn_down columns of
 * its ffn/world slice, attn_output columns of its heads, output (lm_head)
 * rows of its vocab/world slice; token_embd and the norms whole.  The
 * outputs of attn_output and ffn_down are partial sums over the rank's
 * inputs; each rank pushes its binary64 partials into every rank's inbox
 * from the projection kernel and the residual + RMSNorm kernel adds the
 * world partials in rank order (one f32 rounding, as on one GPU).  Greedy
 * argmax exchanges each rank's (max, index) pair.  Every rank calls the
 * same decode functions with the same tokens; all ranks get the same next
 * tokens.  fb_model_forward's logits_host receives the rank's vocab slice
 * (fb_model_tp_info gives its offset and length); fb_model_read_kv returns
 * the rank's kv heads.  world is 2, 4 or 8 with n_kv_heads, ffn/256 and
 * n_heads*head_dim/256 divisible by world. */
typedef struct fb_comm fb_comm;
#define FB_TP_MAX 8
#define FB_COMM_HANDLE_BYTES 64
int fb_comm_create(fb_ctx *ctx, int rank, int world, int max_batch,
                   int hidden, fb_comm **out);
int fb_comm_handle(const fb_comm *comm, void *handle_out);
int fb_comm_open(fb_comm *comm, const void *handles);
/* Bound of the device waits on peers (default 10 s); read when a model's
 * decode step is first run or captured for a batch size. */
int fb_comm_set_timeout_ms(fb_comm *comm, int ms);
int fb_comm_destroy(fb_comm *comm);
int fb_model_create_tp(fb_ctx *ctx, const fb_model_config *cfg,
                       fb_comm *comm, fb_model **out);
int fb_model_tp_info(const fb_model *m, int *rank, int *world,
                     int *vocab_offset, int *vocab_count);

#ifdef __cplusplus
}
#endif
#endif
