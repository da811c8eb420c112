// On-device token sampling: the reference Sampler (crates/ferrite-core/src/
// sampling.rs:61-239) -- repetition penalty, temperature, softmax, min-p,
// top-p, top-k (each filter renormalizes), then a draw from the filtered
// distribution with the caller's uniform r -- as one CTA per logits row.
//
// Arithmetic follows the reference's steps in f32 (penalty as candle's affine
// x * (1/p) or x * p, then x + (pen - x); scaling x * (1/T); softmax
// exp(s - max) / sum; min-p threshold min_p * max_p; the filters keep what
// the sorted-order rules keep), with the sums (softmax, renormalizations,
// the top-p running mass, the draw's cumulative sum) in binary64 and one
// rounding per value, where the reference accumulates left to right in f32.
// Sorting is replaced by threshold searches:
// top-p keeps the K most probable tokens where K is the first rank whose
// cumulative probability reaches top_p (the value v_K = max{v : mass of p >= v
// >= top_p} is found by bisection over the bit patterns of non-negative
// floats, ties at v_K kept in index order as a stable sort does); top-k keeps
// the k most probable (ties in index order).  The result equals the
// reference's whenever its f32 running sums stay clear of a boundary (a few
// tokens holding the mass); over thousands of kept tokens its f32 sums drift
// by ~1e-4 and move its boundaries.
#include <math.h>

#include <vector>

#include "fb_internal.h"
#include "kq_common.cuh"

namespace fb {

constexpr int SAMP_THREADS = 1024;

template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, T *sh, Op op) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, off));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    T r = sh[0];
    for (int w = 1; w < SAMP_THREADS / 32; w++) r = op(r, sh[w]);
    return r;
}
struct OpAdd {
    template <typename T> __device__ T operator()(T a, T b) const { return a + b; }
};
struct OpMax {
    __device__ float operator()(float a, float b) const { return fmaxf(a, b); }
};

// Keeps the tokens selected by a count/mass threshold search: p > v stay,
// the first `nties` tokens with p == v (index order) stay, the rest become 0.
__device__ void keep_above(float *p, int vocab, float v, int nties, int *shi) {
    // exclusive scan of tie counts over contiguous per-thread ranges
    const int per = (vocab + SAMP_THREADS - 1) / SAMP_THREADS;
    const int i0 = threadIdx.x * per, i1 = min(vocab, i0 + per);
    int c = 0;
    for (int i = i0; i < i1; i++) c += p[i] == v;
    // block exclusive scan (simple two-level through shared memory)
    __syncthreads();
    shi[threadIdx.x] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int t = 0; t < SAMP_THREADS; t++) {
            const int x = shi[t];
            shi[t] = run;
            run += x;
        }
    }
    __syncthreads();
    int before = shi[threadIdx.x];
    for (int i = i0; i < i1; i++) {
        const float x = p[i];
        if (x > v) continue;
        if (x == v && before < nties) {
            before++;
            continue;
        }
        if (x == v) before++;
        p[i] = 0.f;
    }
    __syncthreads();
}

// p /= sum(p): binary64 sum, one rounding per value
__device__ void renormalize(float *p, int vocab, double *shd) {
    double s = 0.0;
    for (int i = threadIdx.x; i < vocab; i += SAMP_THREADS) s += p[i];
    s = block_reduce(s, shd, OpAdd());
    if (s > 0.0)
        for (int i = threadIdx.x; i < vocab; i += SAMP_THREADS) p[i] = __double2float_rn(__ddiv_rn((double)p[i], s));
    __syncthreads();
}

// p (scratch, the penalized logits on entry) -> sampled index in *out.
__global__ void __launch_bounds__(SAMP_THREADS) k_sample(float *__restrict__ p, int vocab, float inv_t, float min_p,
                                                          float top_p, int top_k, float r, int32_t *__restrict__ out) {
    __shared__ float shf[SAMP_THREADS / 32];
    __shared__ double shd[SAMP_THREADS / 32];
    __shared__ int shi[SAMP_THREADS];
    __shared__ int s_cnt[SAMP_THREADS / 32];
    // temperature and softmax
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < vocab; i += SAMP_THREADS) {
        const float s = __fadd_rn(__fmul_rn(p[i], inv_t), 0.f);
        p[i] = s;
        mx = fmaxf(mx, s);
    }
    mx = block_reduce(mx, shf, OpMax());
    double sum = 0.0;
    for (int i = threadIdx.x; i < vocab; i += SAMP_THREADS) {
        const float e = expf(__fsub_rn(p[i], mx));
        p[i] = e;
        sum += e;
    }
    sum = block_reduce(sum, shd, OpAdd());
    float pmax = 0.f;
    for (int i = threadIdx.x; i < vocab; i += SAMP_THREADS) {
        const float q = __double2float_rn(__ddiv_rn((double)p[i], sum));
        p[i] = q;
        pmax = fmaxf(pmax, q);
    }
    pmax = block_reduce(pmax, shf, OpMax());
    // min-p: keep p >= min_p * max_p
    if (min_p > 0.f) {
        const float thr = __fmul_rn(min_p, pmax);
        for (int i = threadIdx.x; i < vocab; i += SAMP_THREADS)
            if (!(p[i] >= thr)) p[i] = 0.f;
        __syncthreads();
        renormalize(p, vocab, shd);
    }
    // top-p: v_K = max{v : sum_{p >= v} p >= top_p} by bisection on float bits
    if (top_p < 1.f) {
        uint32_t lo = 0, hi = 0x3F800001u;  // g(lo) >= top_p assumed; g(hi) = 0
        double mass_lo = 0.0;
        {
            double m = 0.0;
            for (int i = threadIdx.x; i < vocab; i += SAMP_THREADS) m += p[i];
            mass_lo = block_reduce(m, shd, OpAdd());
        }
        if (mass_lo >= (double)top_p) {
            while (hi - lo > 1) {
                const uint32_t mid = lo + (hi - lo) / 2;
                const float v = __uint_as_float(mid);
                double m = 0.0;
                for (int i = threadIdx.x; i < vocab; i += SAMP_THREADS)
                    if (p[i] >= v) m += p[i];
                m = block_reduce(m, shd, OpAdd());
                if (m >= (double)top_p) lo = mid;
                else hi = mid;
            }
            const float vk = __uint_as_float(lo);
            // mass strictly above v_K, then how many ties at v_K the
            // cumulative rule keeps (preceding mass < top_p)
            double above = 0.0;
            for (int i = threadIdx.x; i < vocab; i += SAMP_THREADS)
                if (p[i] > vk) above += p[i];
            above = block_reduce(above, shd, OpAdd());
            int nt = 1;
            if (vk > 0.f) {
                const double need = ((double)top_p - above) / (double)vk;
                nt = need <= 1.0 ? 1 : (int)ceil(need);
            }
            keep_above(p, vocab, vk, nt, shi);
            renormalize(p, vocab, shd);
        }
    }
    // top-k: v_k = max{v : count(p >= v) >= k}
    if (top_k > 0 && top_k < vocab) {
        uint32_t lo = 0, hi = 0x3F800001u;
        while (hi - lo > 1) {
            const uint32_t mid = lo + (hi - lo) / 2;
            const float v = __uint_as_float(mid);
            int c = 0;
            for (int i = threadIdx.x; i < vocab; i += SAMP_THREADS) c += p[i] >= v;
            c = block_reduce(c, s_cnt, OpAdd());
            if (c >= top_k) lo = mid;
            else hi = mid;
        }
        const float vk = __uint_as_float(lo);
        int above = 0;
        for (int i = threadIdx.x; i < vocab; i += SAMP_THREADS) above += p[i] > vk;
        above = block_reduce(above, s_cnt, OpAdd());
        keep_above(p, vocab, vk, top_k - above, shi);
        renormalize(p, vocab, shd);
    }
    // draw: first index whose cumulative probability exceeds r (index order)
    const int per = (vocab + SAMP_THREADS - 1) / SAMP_THREADS;
    const int i0 = threadIdx.x * per, i1 = min(vocab, i0 + per);
    double part = 0.0;
    for (int i = i0; i < i1; i++) part += p[i];
    __shared__ double shs[SAMP_THREADS];
    __shared__ int s_pick;
    shs[threadIdx.x] = part;
    if (threadIdx.x == 0) s_pick = -1;
    __syncthreads();
    if (threadIdx.x == 0) {  // exclusive scan of the per-thread masses
        double run = 0.0;
        for (int t = 0; t < SAMP_THREADS; t++) {
            const double x = shs[t];
            shs[t] = run;
            run += x;
        }
    }
    __syncthreads();
    double cum = shs[threadIdx.x];
    if ((double)r < cum + part) {
        for (int i = i0; i < i1; i++) {
            cum += p[i];
            if ((double)r < cum) {
                atomicMin(reinterpret_cast<unsigned *>(&s_pick), (unsigned)i);  // -1 = 0xFFFFFFFF
                break;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int pick = s_pick;
        if (pick < 0) {  // r beyond the total: last token with a nonzero probability
            for (int i = vocab - 1; i >= 0; i--)
                if (p[i] > 0.f) {
                    pick = i;
                    break;
                }
            if (pick < 0) pick = 0;
        }
        *out = pick;
    }
}

// x[t] -> x[t] + (pen - x[t]) for each listed token (deduplicated on the host)
__global__ void k_rep_penalty(float *__restrict__ x, const int32_t *__restrict__ toks, int n, float inv_p, float p) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = x[toks[i]];
    const float pen = v > 0.f ? __fadd_rn(__fmul_rn(v, inv_p), 0.f) : __fadd_rn(__fmul_rn(v, p), 0.f);
    x[toks[i]] = __fadd_rn(v, __fsub_rn(pen, v));
}

}  // namespace fb

using namespace fb;

extern "C" {

int fb_sample(fb_ctx *ctx, const float *logits_dev, int vocab, const fb_sampler_config *cfg,
              const int32_t *prev_tokens_host, int n_prev, uint64_t *rng_state, int32_t *token_out) {
    return guarded([&] {
        FB_REQUIRE(ctx && logits_dev && cfg && rng_state && token_out, "null argument");
        FB_REQUIRE(vocab >= 1 && n_prev >= 0 && (n_prev == 0 || prev_tokens_host), "bad arguments");
        const fb_sampler_config &c = *cfg;
        FB_REQUIRE(c.temperature >= 0.0 && c.top_k >= 0, "temperature and top_k must be non-negative");
        // scratch: the row (f32), the deduplicated token list, argmax workspace, result
        const size_t row_b = ((size_t)vocab * 4 + 255) & ~(size_t)255;
        std::vector<int32_t> uniq;
        if (c.repetition_penalty != 1.0f && n_prev > 0) {
            std::vector<char> seen((size_t)vocab, 0);
            for (int i = 0; i < n_prev; i++) {
                const int32_t t = prev_tokens_host[i];
                if (t >= 0 && t < vocab && !seen[(size_t)t]) {
                    seen[(size_t)t] = 1;
                    uniq.push_back(t);
                }
            }
        }
        const size_t tok_b = ((uniq.size() + 1) * 4 + 255) & ~(size_t)255;
        const size_t ws_b = (argmax_ws_bytes(1) + 255) & ~(size_t)255;
        uint8_t *scr = static_cast<uint8_t *>(ctx->ensure_scratch(row_b + tok_b + ws_b + 256));
        float *row = reinterpret_cast<float *>(scr);
        int32_t *toks = reinterpret_cast<int32_t *>(scr + row_b);
        void *ws = scr + row_b + tok_b;
        int32_t *res = reinterpret_cast<int32_t *>(scr + row_b + tok_b + ws_b);
        cudaStream_t s = ctx->stream;
        FB_CUDA(cudaMemcpyAsync(row, logits_dev, (size_t)vocab * 4, cudaMemcpyDeviceToDevice, s));
        if (!uniq.empty()) {
            FB_CUDA(cudaMemcpyAsync(toks, uniq.data(), uniq.size() * 4, cudaMemcpyHostToDevice, s));
            const int n = (int)uniq.size();
            k_rep_penalty<<<(n + 255) / 256, 256, 0, s>>>(row, toks, n, (float)(1.0 / (double)c.repetition_penalty),
                                                          c.repetition_penalty);
            FB_CUDA(cudaGetLastError());
        }
        if (c.temperature == 0.0) {
            FB_CUDA(cudaMemsetAsync(ws, 0, argmax_ws_bytes(1), s));
            launch_argmax(ctx, row, 1, vocab, res, ws);
        } else {
            // the reference's xorshift64 and its f32 uniform
            uint64_t x = *rng_state;
            x ^= x << 13;
            x ^= x >> 7;
            x ^= x << 17;
            *rng_state = x;
            const float r = (float)x / (float)UINT64_MAX;
            k_sample<<<1, SAMP_THREADS, 0, s>>>(row, vocab, (float)(1.0 / c.temperature), c.min_p, (float)c.top_p,
                                                c.top_k, r, res);
            FB_CUDA(cudaGetLastError());
        }
        int32_t out = 0;
        FB_CUDA(cudaMemcpyAsync(&out, res, 4, cudaMemcpyDeviceToHost, s));
        FB_CUDA(cudaStreamSynchronize(s));
        *token_out = out;
    });
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Top-k logits candidates for the logits-hook path (k <= 16).
//
// The reference collects them on the host: the whole vocab row is copied out,
// sorted by descending logit with a stable sort (ties keep index order) and
// the first `limit` taken (crates/ferrite-core/src/hooks.rs:19-38); the GPU
// logits executor rewrites 16 of them (crates/ferrite-wasm-host/src/
// adapter.rs:508-515).  Here the selection stays on the device in two
// launches: grid (chunks, rows) picks each chunk's k best (value, index)
// pairs by k rounds of a block-wide selection, each round taking the best
// pair ordered strictly after the previous pick; a second kernel (one CTA per
// row) selects the row's k best from the chunks' candidates the same way.
// Order: a before b when a.v > b.v, or a.v == b.v and a.i < b.i -- the
// stable descending sort's order for non-NaN logits (NaN logits are never
// selected here; the reference's comparator treats NaN as equal to
// everything, which has no stable-sort equivalent).
namespace fb {

constexpr int TOPK_MAX = 16;
constexpr int TOPK_THREADS = 256;
constexpr int TOPK_PER_THREAD = 8;  // values a thread holds per chunk
constexpr int TOPK_CHUNK = TOPK_THREADS * TOPK_PER_THREAD;

struct VI {
    float v;
    int i;
};
__device__ __forceinline__ bool vi_before(float av, int ai, float bv, int bi) {
    return av > bv || (av == bv && ai < bi);
}
// Best pair of the block among (vals[j], idx[j]) entries strictly after
// (pv, pi) in the order; returns (-inf, INT_MAX) when none is left.
template <int PER>
__device__ __forceinline__ VI topk_round(const float (&vals)[PER], const int (&idx)[PER], float pv, int pi, VI *sh) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const float v = vals[j];
        const int i = idx[j];
        if (i != 0x7fffffff && vi_before(pv, pi, v, i) && vi_before(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (vi_before(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();  // the previous round's readers of sh are done
    if (lane == 0) sh[warp] = VI{bv, bi};
    __syncthreads();
    VI r = sh[0];
#pragma unroll
    for (int w = 1; w < TOPK_THREADS / 32; w++)
        if (vi_before(sh[w].v, sh[w].i, r.v, r.i)) r = sh[w];
    return r;
}

// Candidates of chunk blockIdx.x of row blockIdx.y -> cand[row][chunk][k].
__global__ void __launch_bounds__(TOPK_THREADS) k_topk_chunks(const float *__restrict__ logits, int64_t vocab, int k,
                                                              VI *__restrict__ cand) {
    __shared__ VI sh[TOPK_THREADS / 32];
    const int64_t row = blockIdx.y;
    const int64_t base = (int64_t)blockIdx.x * TOPK_CHUNK;
    float vals[TOPK_PER_THREAD];
    int idx[TOPK_PER_THREAD];
#pragma unroll
    for (int j = 0; j < TOPK_PER_THREAD; j++) {
        const int64_t i = base + threadIdx.x + (int64_t)j * TOPK_THREADS;
        const float v = i < vocab ? logits[row * vocab + i] : -INFINITY;
        const bool ok = i < vocab && !isnan(v);
        vals[j] = ok ? v : -INFINITY;
        idx[j] = ok ? (int)i : 0x7fffffff;
    }
    float pv = INFINITY;  // before every finite or infinite value: (+inf, -1)
    int pi = -1;
    VI *out = cand + (row * gridDim.x + blockIdx.x) * k;
    for (int r = 0; r < k; r++) {
        const VI b = topk_round<TOPK_PER_THREAD>(vals, idx, pv, pi, sh);
        if (threadIdx.x == 0) out[r] = b;
        pv = b.v;
        pi = b.i;
    }
}

// Final selection of one row from its chunks' candidates.
__global__ void __launch_bounds__(TOPK_THREADS) k_topk_final(const VI *__restrict__ cand, int ncand, int k,
                                                             int32_t *__restrict__ ids, float *__restrict__ vals_out) {
    __shared__ VI sh[TOPK_THREADS / 32];
    constexpr int PER = 8;  // ncand <= TOPK_THREADS * PER (checked on the host)
    const int64_t row = blockIdx.x;
    float vals[PER];
    int idx[PER];
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int c = threadIdx.x + j * TOPK_THREADS;
        const VI x = c < ncand ? cand[row * ncand + c] : VI{-INFINITY, 0x7fffffff};
        vals[j] = x.v;
        idx[j] = x.i;
    }
    float pv = INFINITY;
    int pi = -1;
    for (int r = 0; r < k; r++) {
        const VI b = topk_round<PER>(vals, idx, pv, pi, sh);
        if (threadIdx.x == 0) {
            ids[row * k + r] = b.i == 0x7fffffff ? -1 : b.i;
            vals_out[row * k + r] = b.i == 0x7fffffff ? -INFINITY : b.v;
        }
        pv = b.v;
        pi = b.i;
    }
}

}  // namespace fb

extern "C" int fb_top_logits(fb_ctx *ctx, const float *logits_dev, int rows, int64_t vocab, int k, int32_t *ids_dev,
                             float *vals_dev) {
    using namespace fb;
    return guarded([&] {
        FB_REQUIRE(ctx && logits_dev && ids_dev && vals_dev, "null argument");
        FB_REQUIRE(rows >= 1 && vocab >= 1 && vocab < 0x7fffffff, "bad shape");
        FB_REQUIRE(k >= 1 && k <= TOPK_MAX, "k must be in 1..16");
        const int64_t nchunk = (vocab + TOPK_CHUNK - 1) / TOPK_CHUNK;
        const int64_t ncand = nchunk * k;
        FB_REQUIRE(ncand <= (int64_t)TOPK_THREADS * 8, "top_logits: ceil(vocab / 2048) * k must be <= 2048");
        FB_REQUIRE(rows <= 65535, "top_logits: at most 65535 rows");
        VI *cand = static_cast<VI *>(ctx->ensure_scratch((size_t)rows * ncand * sizeof(VI)));
        k_topk_chunks<<<dim3((unsigned)nchunk, (unsigned)rows), TOPK_THREADS, 0, ctx->stream>>>(logits_dev, vocab, k,
                                                                                               cand);
        FB_CUDA(cudaGetLastError());
        k_topk_final<<<rows, TOPK_THREADS, 0, ctx->stream>>>(cand, (int)ncand, k, ids_dev, vals_dev);
        FB_CUDA(cudaGetLastError());
    });
}
