// Host-side internals shared by the C ABI, the kernels' launchers and the
// model runtime.  Not part of the public interface.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/ferrite_b200.h"

namespace fb {

// Exception carrying a status code; caught at the C boundary.
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void fail(int code, const std::string &msg);
void set_last_error(const std::string &msg);

// Runs f, converting exceptions into a status code + thread-local message.
template <class F> int guarded(F &&f) {
    try {
        f();
        return FB_OK;
    } catch (const Error &e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc &) {
        set_last_error("host allocation failed");
        return FB_ERR_OOM;
    } catch (const std::exception &e) {
        set_last_error(e.what());
        return FB_ERR_INVALID;
    }
}
void check_cuda(cudaError_t e, const char *what, const char *file, int line);
#define FB_CUDA(call) ::fb::check_cuda((call), #call, __FILE__, __LINE__)
#define FB_REQUIRE(cond, msg)                                              \
    do {                                                                   \
        if (!(cond)) ::fb::fail(FB_ERR_INVALID, std::string(msg));         \
    } while (0)

// Device error-word bits (set by kernels, read by fb_ctx_error_word).
enum : uint32_t {
    ERRBIT_WAIT_TIMEOUT = 1u << 0,  // a bounded spin-wait gave up
    ERRBIT_BAD_TOKEN = 1u << 1,     // token id outside [0, vocab)
    ERRBIT_BAD_POS = 1u << 2,       // position outside the KV capacity
    ERRBIT_BAD_PAGE = 1u << 3,      // block-table entry outside the pool
    ERRBIT_PEER_TIMEOUT = 1u << 4,  // a tensor-parallel peer did not arrive in time
};

// A device buffer owned by the library.
struct DevBuf {
    void *ptr = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    ~DevBuf();
    void alloc(size_t n);
    void release();
    template <class T> T *as() const { return reinterpret_cast<T *>(ptr); }
};

}  // namespace fb

struct fb_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    bool pdl = true;
    bool prefill_cache = true;  // fb_ctx_set_prefill_weight_cache
    int num_sms = 148;
    uint32_t *err_word = nullptr;          // device, zero-initialised
    fb::DevBuf scratch;                    // grow-only workspace
    void *ensure_scratch(size_t bytes);
};

// Device layouts of k-quant weights W[n, k] (nb = k/256 super-blocks per
// row): tile-major, 16 rows per tile (n padded to a multiple of 16 with zero
// rows).  The 16 rows' super-block b of tile T form one contiguous record,
// records ordered (T, b), so the GEMV streams (tile, block) records with one
// bulk copy each.
//  Q4_K record = 16 x 144 B: row slot r at +144r holds the GGUF header (d,
//        dmin, scales[12]) in bytes 0..15 and the 128 quant bytes permuted so
//        MMA quad lane t reads bytes [16+32t, 48+32t): for g = 0..3, GGUF
//        qs[32g + 8t .. 32g + 8t + 7].
//  Q6_K record = 16 x 208 B + 16 x 2 B: row slot r at +208r: bytes [48t,
//        48t+48) for quad lane t hold 8 ql words (h, j, x) = GGUF
//        ql[64h + 32j + 8t + 4x .. +3] and 4 qh words (h, x) = GGUF
//        qh[32h + 8t + 4x .. +3]; bytes 192..207 the 16 int8 scales.  The
//        fp16 super-block scale d of row slot r is at +3328 + 2r.
struct fb_qtensor {
    int dtype = 0;
    int64_t n = 0, k = 0;
    fb::DevBuf buf;
    fb::DevBuf f16;           // prefill weight cache: W dequantized to fp16 [n][k] (empty: none)
    bool f16_tried = false;   // the cache was considered (allocated or refused) once
    int64_t nb() const { return k / 256; }
    int64_t n_pad() const { return (n + 15) / 16 * 16; }
    int64_t n_tiles() const { return (n + 15) / 16; }
    const uint8_t *main() const { return buf.as<uint8_t>(); }
    static size_t device_bytes(int dtype, int64_t n, int64_t k);
};

namespace fb {
constexpr int Q4K_REC = 16 * 144;  // 2304
constexpr int Q6K_REC = 16 * 210;  // 3360
// Byte offset of row `row`, super-block `b` (nb per row) in the tile-major
// layout: the row's 144-byte Q4_K block / the row's 208-byte Q6_K part.
__host__ __device__ inline size_t q4k_offset(int64_t row, int64_t b, int64_t nb) {
    return (size_t)(((row >> 4) * nb + b) * Q4K_REC) + (size_t)(row & 15) * 144;
}
__host__ __device__ inline size_t q6k_offset(int64_t row, int64_t b, int64_t nb) {
    return (size_t)(((row >> 4) * nb + b) * Q6K_REC) + (size_t)(row & 15) * 208;
}
__host__ __device__ inline size_t q6k_d_offset(int64_t row, int64_t b, int64_t nb) {
    return (size_t)(((row >> 4) * nb + b) * Q6K_REC) + 3328 + (size_t)(row & 15) * 2;
}
}  // namespace fb

namespace fb {

// Q8_K activations in the device's SoA form for m rows of k values:
//  qs  [m][k] int8, each 256-block permuted so quad lane t reads bytes
//      [64t, 64t+64): for s = 0..7, the values 32s + 8t .. 32s + 8t + 7;
//  d   [m][k/256] f32;  bs16 [m][k/16] int16;  bs32 [m][k/32] int16.
struct Q8Act {
    int8_t *qs;
    float *d;
    int16_t *bs16;
    int16_t *bs32;
    int64_t k;
};
size_t q8act_bytes(int64_t m, int64_t k);
Q8Act q8act_view(void *base, int64_t m, int64_t k);

// ---- kernel launchers (stream-ordered, no sync) ----
void launch_quantize_q8k(fb_ctx *ctx, const float *x, int64_t m, int64_t k, const Q8Act &a);
void launch_quantize_q8k_gguf(fb_ctx *ctx, const float *x, int64_t m, int64_t k, void *out);
void launch_repack(fb_ctx *ctx, int dtype, int64_t n, int64_t k, const void *gguf, void *dev);
void launch_unpack(fb_ctx *ctx, int dtype, int64_t n, int64_t k, const void *dev, void *gguf);
void launch_synth(fb_ctx *ctx, int dtype, int64_t nblocks, uint64_t seed, float sigma, void *gguf_out);
void launch_synth_f32(fb_ctx *ctx, float *out, int64_t n, uint64_t seed, float mean, float stddev);
void launch_dequantize(fb_ctx *ctx, const fb_qtensor *t, void *out, int out_dtype);
// y[m, n] (+)= x.W^T for m <= 16 from pre-quantized activations.
void launch_gemv(fb_ctx *ctx, const fb_qtensor *w, const Q8Act &a, int m, float *y, int64_t ldy);
// y[n] = W . x for one f32 row with the f32 dequantized weights (float form).
void launch_gemv_float(fb_ctx *ctx, const fb_qtensor *w, const float *x, float *y);
// m > 16 QMatMul (prefill form).
void qmatmul_prefill(fb_ctx *ctx, const fb_qtensor *w, const float *x, float *y, int64_t m);
// Tensor-core prefill QMatMul (fp16 operands, f32 accumulation): m >= 17 rows,
// n a multiple of 128.
bool prefill_gemm_supported(const fb_qtensor *w, int64_t m);
void prefill_gemm(fb_ctx *ctx, const fb_qtensor *w, const float *x, float *y, int64_t m);
// The same from fp16 rows xh [m][k] already scaled by powers of two
// (rowscale[m], the rule of launch_x_to_f16 / the fused producers).
void prefill_gemm_x16(fb_ctx *ctx, const fb_qtensor *w, const __half *xh, const float *rowscale, float *y,
                      int64_t m);
// x [m][k] f32 -> fp16 with a per-row power-of-two scale s (the smallest
// 2^e, e >= 0, with max |x| / s <= 32768).
void launch_x_to_f16(fb_ctx *ctx, const float *x, __half *xh, float *rowscale, int64_t m, int64_t k);
void launch_block_dots(fb_ctx *ctx, const fb_qtensor *w, const Q8Act &a, int32_t *out_sc, int32_t *out_min);
void launch_rmsnorm(fb_ctx *ctx, const float *x, const float *g, float *y, int64_t rows, int64_t dim, float eps);
void launch_rope(fb_ctx *ctx, float *x, int64_t n_tok, int64_t n_heads, int64_t hd, int64_t pos0,
                 const float *cos_tab, const float *sin_tab, int mode);
void launch_swiglu(fb_ctx *ctx, const float *g, const float *u, float *out, int64_t m, int64_t f);

// Fused decode-step kernels (ops.cu).
// Reads the residual x (+ add), writes it to x_out (must not alias x).
void launch_residual_rmsnorm_q8k(fb_ctx *ctx, const float *x, const float *add, float *x_out, const float *g, int rows,
                                 int dim, float eps, const Q8Act &a, const fb_qtensor *emb, const int32_t *tokens,
                                 int vocab);
void launch_swiglu_q8k(fb_ctx *ctx, const float *y, int f, int rows, const Q8Act &a);
// ws: argmax_ws_bytes(rows) bytes, zeroed once before first use.
size_t argmax_ws_bytes(int rows);
void launch_argmax(fb_ctx *ctx, const float *logits, int rows, int64_t vocab, int32_t *out, void *ws);
// kv_head0: global index of the pool's first kv head (tensor-parallel shards)
void launch_synth_kv(fb_ctx *ctx, void *pool, int layer, int which, int nctx, int nkv, int hd, int page_size,
                     const int32_t *block_table, int max_pages, int slots, uint64_t seed, float scale,
                     int kv_head0 = 0);

// Batched prefill (ops.cu, prefill_attn.cu): T token rows, f32 activations.
void launch_embed_rows(fb_ctx *ctx, const fb_qtensor *emb, const int32_t *tokens, int T, int vocab, int dim,
                       float *x);
// x += y (y may be null), xn = RMSNorm(x) * g, row by row
// (xh, rs != null: also the normalized rows as the prefill GEMM's fp16
// operand, see launch_x_to_f16; xn may then be null)
void launch_add_rmsnorm_rows(fb_ctx *ctx, float *x, const float *y, const float *g, float *xn, int T, int dim,
                             float eps, __half *xh = nullptr, float *rs = nullptr);
void launch_swiglu_rows(fb_ctx *ctx, const float *y, int f, int T, float *act);
// SwiGLU rows straight into the fp16 operand of the next prefill GEMM.
void launch_swiglu_rows_x16(fb_ctx *ctx, const float *y, int f, int T, __half *xh, float *rs);
void launch_prefill_qkv_rope(fb_ctx *ctx, const float *y, int64_t ld, int T, int pos0, int n_heads, int n_kv,
                             const float *q_norm, const float *k_norm, float eps, const float *rope_cos,
                             const float *rope_sin, int rope_mode, float *q_out, void *kpool, void *vpool,
                             const int32_t *bt, int page_size, int num_pages);
// Causal attention of T queries (positions pos0 .. pos0 + T - 1, q f32
// [T][n_heads][128]) over one sequence's paged fp16 KV cache (64-token
// pages, dim-major K); out f32 [T][n_heads][128].
void launch_attn_prefill(fb_ctx *ctx, const float *q, const void *kpool, const void *vpool, const int32_t *bt,
                         int max_pages, int num_pages, int pos0, int T, int n_heads, int n_kv, float scale,
                         float *out);

// Paged flash-decode attention (attention.cu).
constexpr int ATT_SPLITS = 16;      // attention splits (cluster CTAs) per (kv head, sequence)
constexpr int ATT_SPLITS_MAX = 64;  // cluster-free merge: splits when the grid is small
constexpr int ATT_MERGE1_MAX = 32;  // up to this many splits merge in one level
constexpr int ATT_GROUP = 8;        // more than ATT_MERGE1_MAX splits merge in groups of 8, then the groups
constexpr int ATT_CNT_PER = 1 + ATT_SPLITS_MAX / ATT_GROUP;  // merge counters per (kv head, sequence) then
constexpr int ATT_SLOTS_MAX = ATT_SPLITS_MAX + ATT_SPLITS_MAX / ATT_GROUP;  // partial slots per head
struct AttnArgs {
    const float *q;              // [b, n_heads, hd]
    const void *kpool;           // fp16 [num_pages, n_kv, hd, page] (dim-major pages)
    const void *vpool;           // fp16 [num_pages, n_kv, page, hd]
    const int32_t *block_table;  // [b, max_pages]
    const int32_t *seq_lens;     // [b] or null (then pos[b] + 1)
    const int32_t *pos;          // [b]
    double *part_o;              // cluster-free merge: [b, n_heads, slots, hd] unnormalised sum p*v
    double *part_ml;             // cluster-free merge: [b, n_heads, slots, 2] (running max, sum p)
                                 // (slots = splits, + splits / ATT_GROUP above ATT_MERGE1_MAX splits)
    int n_heads, n_kv, page_size, max_pages, num_pages, nsplit_max;
    float scale;
    uint32_t *err;
    // fused prologue (model path): when qkv != null the kernel takes q, k, v
    // of the new token from the projection output [b][qkv_ld] = (q | k | v),
    // applies the optional QK RMSNorm (q_norm / k_norm gains) and RoPE at
    // position seq_len - 1, writes k / v into the pools and (q_out != null) a
    // copy of the transformed q [b][n_heads][hd]
    const float *qkv;
    int64_t qkv_ld;
    const float *q_norm, *k_norm;
    float eps;
    const float *rope_cos, *rope_sin;  // [rope_rows][hd / 2]
    int rope_rows, rope_mode;
    float *q_out;
};
void launch_attn_decode(fb_ctx *ctx, const AttnArgs &A, int batch, int max_seq_len, float *out_f32,
                        const Q8Act *aq, int *counters, bool pdl, bool want_cluster);
bool attn_uses_cluster(fb_ctx *ctx, const AttnArgs &A, int batch);

// ---- tensor parallelism (tp.cu) ----
// Exchange region of one rank (cudaMalloc, mapped by every rank via IPC):
//   flags    [FB_TP_MAX] u32      (unused by the row-parallel exchange)
//   am_flags [FB_TP_MAX][B] u32   argmax exchange: step epoch per (src, row)
//   inbox_o / inbox_d [W][B][H][2] u64  partial sums of attn_output /
//                                 ffn_down: each binary64 as two words
//                                 (seq << 32) | 32-bit half (lo, hi)
//   am_inbox [W][B] u64           (f32 bits of the max << 32) | global index
struct CommLayout {
    size_t flags, am_flags, inbox_o, inbox_d, am_inbox, total;
};
CommLayout comm_layout(int world, int max_batch, int hidden);

// Row-parallel GEMV output: the binary64 row sums (not rounded) are stored
// to every rank p < world as the word pair dst[p][2 (col * ld + row) + {0, 1}]
// = (seq << 32) | lo / hi 32 bits, each an 8-byte single-copy-atomic store:
// a reader that sees seq in both words has the value, with no fence or flag
// (seq = (*epoch - 1) * nx + xi + 1 numbers the step's exchange points).
struct PeerOut {
    uint64_t *dst[FB_TP_MAX];
    int64_t ld;
    int world;
    const uint32_t *epoch;  // device step counter (>= 1 inside a step)
    int nx, xi;
};
// Residual + RMSNorm after a row-parallel projection (one exchange point).
struct TpNorm {
    const uint64_t *inbox;           // this rank's inbox [W][B][H][2] (PeerOut word pairs)
    const uint32_t *epoch;           // device step counter (>= 1 inside a step)
    double *ss_part;                 // [B][H/256] per-block sums of squares
    uint32_t *ss_tag;                // [B][H/256] exchange sequence of ss_part
    uint64_t limit_ns;               // bound of every wait
    int world, batch_cap, nx;        // nx = exchange points per step
};
struct TpArgmax {
    uint64_t *peer_slot[FB_TP_MAX];  // &am_inbox[rank][0] in rank p's region
    uint32_t *peer_flag[FB_TP_MAX];  // &am_flags[rank][0] in rank p's region
    const uint64_t *my_inbox;        // [W][B]
    const uint32_t *my_flags;        // [FB_TP_MAX][B]
    const uint32_t *epoch;
    uint64_t limit_ns;
    int world, batch_cap, vocab_off;
};
void launch_tp_residual_rmsnorm_q8k(fb_ctx *ctx, const float *x, float *x_out, const float *g, int rows, int dim,
                                    float eps, const Q8Act &a, const TpNorm &t, int xi);
// y[m, n] from pre-quantized activations, with the row sums pushed to peers.
void launch_gemv_peer(fb_ctx *ctx, const fb_qtensor *w, const Q8Act &a, int m, const PeerOut &po);
void launch_argmax_tp(fb_ctx *ctx, const float *logits, int rows, int64_t vocab, int32_t *out, void *ws,
                      const TpArgmax &t);
// First kernel of a step: embedding + RMSNorm, bumping the step counter.
void launch_embed_rmsnorm_q8k(fb_ctx *ctx, float *x_out, const float *g, int rows, int dim, float eps,
                              const Q8Act &a, const fb_qtensor *emb, const int32_t *tokens, int vocab,
                              uint32_t *epoch_inc);

}  // namespace fb

struct fb_comm {
    fb_ctx *ctx = nullptr;
    int rank = 0, world = 1, max_batch = 0, hidden = 0;
    fb::CommLayout L{};
    fb::DevBuf region;                       // this rank's exchange region
    uint8_t *peer[FB_TP_MAX] = {nullptr};    // every rank's region in this process
    uint64_t timeout_ns = 10ull * 1000 * 1000 * 1000;  // bound of the device waits on peers
    bool opened = false;
    ~fb_comm();
    template <class T> T *at(int p, size_t off) const { return reinterpret_cast<T *>(peer[p] + off); }
};

namespace fb {

// RoPE tables [max_pos][hd/2] computed on the host exactly as the oracle does
// (candle precompute_freqs_cis: angle = pos * theta^(-2i/hd) in f32).
void rope_tables(int max_pos, int head_dim, float theta, std::vector<float> &cos_t,
                 std::vector<float> &sin_t);

}  // namespace fb
