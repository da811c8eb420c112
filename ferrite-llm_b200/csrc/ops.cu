// Norm / RoPE / SwiGLU / embedding / argmax kernels of the decode step, in
// standalone form (C-ABI ops) and fused with the Q8_K quantization of the
// next QMatMul's input.
//
// Semantics (candle-nn 0.8.4 CPU ops as used by quantized_llama; CUDA forms
// in the reference's vendored ptx-kernels/kernels/candle/reduce.cu):
//   rms_norm  y = x / sqrt(mean(x^2) + eps) * g          (reduce.cu:189-230)
//   rope_i    interleaved pairs (x[2i], x[2i+1])         (reduce.cu:275-292)
//   rope      rotate-half pairs (x[i], x[i + d/2])       (reduce.cu:294-318)
//   silu      v / (1 + exp(-v))                          (unary.cu:59)
// Elementwise float steps use round-to-nearest intrinsics (no contraction);
// reductions and the SiLU exponential run in binary64 with one rounding to
// f32, so values match the CPU oracle bit for bit regardless of summation
// order.
#include <math.h>

#include <algorithm>

#include "fb_internal.h"
#include "kq_common.cuh"
#include "q8k_store.cuh"

namespace fb {

// 1 / rms from a binary64 sum of squares, as the oracle computes it:
// m = sqrtf((float)(ss / dim) + eps).

// ------------------------------------------------------------------------
// Residual add + RMSNorm + Q8_K.  One CTA per (256-value block, row): every
// CTA sums the squares of the whole row itself (binary64; the row is a few
// KB in L2) and then normalizes and quantizes only its own block, so the row
// is processed by dim/256 CTAs in parallel.  x[row] (+= add[row] when add !=
// null) is written to x_out block by block (a different buffer: other CTAs
// are still reading x); the EMB instantiation takes the dequantized
// embedding row of token[row] (emb_tab) instead of x.
constexpr int NORM_THREADS = 256;

__device__ __forceinline__ float q4k_value(const uint8_t *blk, int i) {
    const uint32_t *hw = reinterpret_cast<const uint32_t *>(blk);
    const Q4Scales s = q4k_unpack_scales(hw[1], hw[2], hw[3]);
    const float d = h2f((uint16_t)(hw[0] & 0xFFFF)), dmin = h2f((uint16_t)(hw[0] >> 16));
    const int g = i >> 6, r = i & 63, hi = r >> 5, l = r & 31;
    const int j = 2 * g + hi;
    const int sc = byte_of(j < 4 ? s.sc_lo : s.sc_hi, j & 3);
    const int mn = byte_of(j < 4 ? s.mn_lo : s.mn_hi, j & 3);
    const int t = l >> 3, e = l & 7;
    const int nib = (blk[16 + 32 * t + 8 * g + e] >> (4 * hi)) & 0xF;
    return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)nib), __fmul_rn(dmin, (float)mn));
}

// EMB: the first norm of the step, which dequantizes the token's embedding
// row instead of reading a residual (a separate instantiation keeps the
// per-layer kernel's code small).
template <bool EMB>
__global__ void __launch_bounds__(NORM_THREADS)
    k_residual_rmsnorm_q8k(const float *__restrict__ x, const float *__restrict__ add, float *__restrict__ x_out,
                           const float *__restrict__ g, int dim, float eps, Q8Act a,
                           const uint8_t *__restrict__ emb_tab, const int32_t *__restrict__ tokens, int vocab,
                           uint32_t *err, uint32_t *epoch_inc) {
    __shared__ double sh[NORM_THREADS / 32];
    __shared__ __align__(16) float xb[QK];
    __shared__ float qb[2 * QK / 32];
    __shared__ int s_qi[QK / 32];
    const int blk = blockIdx.x;
    const int64_t row = blockIdx.y;
    // Loads that do not depend on the preceding kernel come first: the gain
    // of this thread's value of the block (weights; usually evicted from L2
    // by the weight stream) and the residual row x, written two or more
    // launches earlier.  Only `add` (the preceding projection's output) is
    // read after the wait.
    const float gt = g[blk * QK + threadIdx.x];
    constexpr int MAXP = 8;  // passes held in registers: dim <= 8192
    const float *xr = x ? x + row * dim : nullptr;
    const int nv = dim / 4;
    float4 v[MAXP];
    if constexpr (!EMB) {
        const float4 *x4 = reinterpret_cast<const float4 *>(xr);
#pragma unroll
        for (int p = 0; p < MAXP; p++) {
            const int i = threadIdx.x + p * NORM_THREADS;
            v[p] = i < nv ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    pdl_launch();  // the next projection may launch and stream its weights now
    pdl_wait();
    // first kernel of a tensor-parallel step: advance the step counter that
    // numbers the step's exchanges (read by later kernels after their wait)
    if (epoch_inc && blk == 0 && row == 0 && threadIdx.x == 0) *epoch_inc += 1u;
    const int nbe = dim / QK;
    int tok = 0;
    if constexpr (EMB) {
        tok = tokens[row];
        if (tok < 0 || tok >= vocab) {
            if (threadIdx.x == 0 && blk == 0) atomicOr(err, ERRBIT_BAD_TOKEN);
            tok = 0;
        }
    }
    double ss = 0.0;
    if constexpr (EMB) {
        for (int i = threadIdx.x; i < dim; i += NORM_THREADS) {
            const float e = q4k_value(emb_tab + q4k_offset(tok, i / QK, nbe), i % QK);
            ss = __fma_rn((double)e, (double)e, ss);
            if (i / QK == blk) xb[i % QK] = e;
        }
    } else {
        const float4 *a4 = add ? reinterpret_cast<const float4 *>(add + row * dim) : nullptr;
        if (a4) {
            float4 d[MAXP];
#pragma unroll
            for (int p = 0; p < MAXP; p++) {
                const int i = threadIdx.x + p * NORM_THREADS;
                d[p] = i < nv ? a4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int p = 0; p < MAXP; p++)
                v[p] = make_float4(__fadd_rn(d[p].x, v[p].x), __fadd_rn(d[p].y, v[p].y), __fadd_rn(d[p].z, v[p].z),
                                   __fadd_rn(d[p].w, v[p].w));
        }
#pragma unroll
        for (int p = 0; p < MAXP; p++) {
            const int i = threadIdx.x + p * NORM_THREADS;
            if (i < nv) {
                ss = __fma_rn((double)v[p].x, (double)v[p].x, ss);
                ss = __fma_rn((double)v[p].y, (double)v[p].y, ss);
                ss = __fma_rn((double)v[p].z, (double)v[p].z, ss);
                ss = __fma_rn((double)v[p].w, (double)v[p].w, ss);
                if ((4 * i) / QK == blk) *reinterpret_cast<float4 *>(&xb[(4 * i) % QK]) = v[p];
            }
        }
        const float4 *x4 = reinterpret_cast<const float4 *>(xr);
        for (int i = threadIdx.x + MAXP * NORM_THREADS; i < nv; i += NORM_THREADS) {  // dim > 8192
            float4 w = x4[i];
            if (a4) {
                const float4 dd = a4[i];
                w = make_float4(__fadd_rn(dd.x, w.x), __fadd_rn(dd.y, w.y), __fadd_rn(dd.z, w.z), __fadd_rn(dd.w, w.w));
            }
            ss = __fma_rn((double)w.x, (double)w.x, ss);
            ss = __fma_rn((double)w.y, (double)w.y, ss);
            ss = __fma_rn((double)w.z, (double)w.z, ss);
            ss = __fma_rn((double)w.w, (double)w.w, ss);
            if ((4 * i) / QK == blk) *reinterpret_cast<float4 *>(&xb[(4 * i) % QK]) = w;
        }
    }
    ss = block_sum64<NORM_THREADS / 32>(ss, sh);  // (has a __syncthreads before the shared reads)
    const float m = rms_of(ss, dim, eps);
    const float xv = xb[threadIdx.x];
    if (x_out) x_out[row * dim + blk * QK + threadIdx.x] = xv;
    q8k_store_block(__fmul_rn(__fdiv_rn(xv, m), gt), a, row, blk, qb, s_qi);
}

// ------------------------------------------------------------------------
// Tensor-parallel residual add + RMSNorm + Q8_K, after a row-parallel
// projection (attn_output or ffn_down sharded along its inputs).  Every
// rank's GEMV has pushed its binary64 partial row sums into this rank's
// inbox [src][row][col]; they are added in rank order and rounded to f32
// once -- the rounding the single-GPU GEMV applies to the full sum -- and
// the residual add, RMSNorm and Q8_K follow k_residual_rmsnorm_q8k.
// Exchange protocol (sequence number seq of this exchange point in the
// step): every rank's GEMV stores each partial into this rank's inbox as two
// 8-byte words (seq << 32) | 32-bit half, and each thread here polls
// (bounded) the W word pairs of its value until both carry seq -- no fence
// on the writer's side and no flag round trip.  Inboxes alternate between
// attn_output and ffn_down, so a rank can only overwrite an inbox slot after
// every rank has passed the exchange in between, i.e. after the slot was
// read.
// One CTA per (256-value block, row) reduces only its own block; the blocks'
// sums of squares meet through global slots tagged with seq.
__global__ void __launch_bounds__(NORM_THREADS)
    k_tp_residual_rmsnorm_q8k(const float *__restrict__ x, float *__restrict__ x_out, const float *__restrict__ g,
                              int dim, float eps, Q8Act a, TpNorm t, int xi, uint32_t *err) {
    __shared__ double sh[NORM_THREADS / 32];
    __shared__ __align__(16) float xb[QK];
    __shared__ double s_ss;
    const int blk = blockIdx.x, nblk = gridDim.x;
    const int64_t row = blockIdx.y;
    const int tid = threadIdx.x;
    const int64_t j = row * dim + (int64_t)blk * QK + tid;
    // weights and the residual row first (they do not depend on the GEMV)
    const float xv = x[j];
    const float gt = g[blk * QK + tid];
    pdl_wait();
    pdl_launch();
    const uint32_t seq = (*t.epoch - 1u) * (uint32_t)t.nx + (uint32_t)xi + 1u;
    const int64_t plane = (int64_t)t.batch_cap * dim;
    double s = 0.0;
    bool ok = true;
    for (int r = 0; r < t.world; r++) {
        const uint64_t *wp = t.inbox + 2 * (r * plane + j);
        uint64_t w0 = ld_relaxed_sys_u64(wp), w1 = ld_relaxed_sys_u64(wp + 1);
        if ((uint32_t)(w0 >> 32) != seq || (uint32_t)(w1 >> 32) != seq) {
            const uint64_t t0 = globaltimer_ns();
            while (ok && ((uint32_t)(w0 >> 32) != seq || (uint32_t)(w1 >> 32) != seq)) {
                __nanosleep(64);
                w0 = ld_relaxed_sys_u64(wp);
                w1 = ld_relaxed_sys_u64(wp + 1);
                ok = globaltimer_ns() - t0 <= t.limit_ns;
            }
        }
        const double v = __longlong_as_double((long long)((w1 << 32) | (w0 & 0xffffffffull)));
        s = __dadd_rn(s, v);
    }
    if (!ok) atomicOr(err, ERRBIT_PEER_TIMEOUT);
    const float xn = __fadd_rn(__double2float_rn(s), xv);
    x_out[j] = xn;
    xb[tid] = xn;
    const double ssb = block_sum64<NORM_THREADS / 32>(__dmul_rn((double)xn, (double)xn), sh);
    const int64_t slot0 = row * nblk;
    if (tid == 0) {
        t.ss_part[slot0 + blk] = ssb;
        __threadfence();
        st_release_gpu(&t.ss_tag[slot0 + blk], seq);
    }
    if (tid < nblk && !wait_seq<false>(&t.ss_tag[slot0 + tid], seq, t.limit_ns))
        atomicOr(err, ERRBIT_WAIT_TIMEOUT);
    __syncthreads();
    if (tid == 0) {
        double ss = 0.0;
        for (int b = 0; b < nblk; b++) ss = __dadd_rn(ss, __ldcg(&t.ss_part[slot0 + b]));
        s_ss = ss;
    }
    __syncthreads();
    const float m = rms_of(s_ss, dim, eps);
    q8k_store_block(__fmul_rn(__fdiv_rn(xn, m), gt), a, row, blk, xb, reinterpret_cast<int *>(xb + 16));
}

// ------------------------------------------------------------------------
// SwiGLU + Q8_K: y[row] = [gate (f) | up (f)] -> act = Q8K(silu(gate) * up).
// One CTA of 256 threads per (row, 256-value block): every thread evaluates
// one binary64 SiLU (the exponential and division chains run side by side
// instead of eight per lane), warp 0 quantizes the block.
__global__ void __launch_bounds__(QK) k_swiglu_q8k(const float *__restrict__ y, int f, int64_t rows, Q8Act a) {
    __shared__ float shv[2 * QK / 32];
    __shared__ int shi[QK / 32];
    pdl_launch();  // the next projection may launch and stream its weights now
    pdl_wait();
    const int64_t nbk = f / QK;
    const int64_t row = blockIdx.x / nbk, blk = blockIdx.x % nbk;
    if (row >= rows) return;
    const int t = threadIdx.x;
    const float g = y[row * 2 * f + blk * QK + t], u = y[row * 2 * f + f + blk * QK + t];
    q8k_store_block(__fmul_rn(silu64(g), u), a, row, blk, shv, shi);
}

// ------------------------------------------------------------------------
// Greedy argmax over each logits row (first index of the maximum, like the
// CPU oracle).  grid (chunks, rows): every CTA reduces one chunk of the row
// to (max, first index); the last CTA of a row (counter) reduces the chunk
// results.  ws: rows * ARGMAX_CHUNKS (value, index) pairs + rows counters
// (zero between launches).
constexpr int ARGMAX_CHUNKS = 128;
__device__ __forceinline__ void argmax_merge(float &best, int &bi, float ov, int oi) {
    if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
    }
}
__device__ __forceinline__ void argmax_block(float &best, int &bi, float *sv, int *si) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
        argmax_merge(best, bi, __shfl_xor_sync(0xffffffffu, best, off), __shfl_xor_sync(0xffffffffu, bi, off));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = bi;
    }
    __syncthreads();
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
        argmax_merge(best, bi, __shfl_xor_sync(0xffffffffu, best, off), __shfl_xor_sync(0xffffffffu, bi, off));
}
// Tensor parallel (t.world > 0): each rank holds a vocab slice; the last CTA
// of a row pushes the slice's (max, global index) to every rank, waits
// (bounded) for all ranks' pairs of this step and merges them.
__global__ void __launch_bounds__(256) k_argmax(const float *__restrict__ logits, int64_t vocab,
                                                int32_t *__restrict__ out, float *__restrict__ ws_v,
                                                int *__restrict__ ws_i, int *__restrict__ counters, TpArgmax t,
                                                uint32_t *err) {
    __shared__ float sv[8];
    __shared__ int si[8];
    __shared__ int s_last;
    __shared__ unsigned long long s_pack;
    pdl_wait();
    const int64_t row = blockIdx.y, chunk = (vocab + gridDim.x - 1) / gridDim.x;
    const int64_t i0 = blockIdx.x * chunk, i1 = min(vocab, i0 + chunk);
    const float *r = logits + row * vocab;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) argmax_merge(best, bi, r[i], (int)i);
    argmax_block(best, bi, sv, si);
    if (threadIdx.x == 0) {
        ws_v[row * gridDim.x + blockIdx.x] = best;
        ws_i[row * gridDim.x + blockIdx.x] = bi;
        __threadfence();
        const int prev = atomicAdd(&counters[row], 1);
        s_last = prev == (int)gridDim.x - 1;
        if (s_last) counters[row] = 0;  // ready for the next launch
    }
    __syncthreads();
    if (s_last) {
        __threadfence();
        best = -INFINITY;
        bi = 0x7fffffff;
        for (int c = threadIdx.x; c < (int)gridDim.x; c += blockDim.x)
            argmax_merge(best, bi, __ldcg(&ws_v[row * gridDim.x + c]), __ldcg(&ws_i[row * gridDim.x + c]));
        __syncthreads();  // sv / si are reused
        argmax_block(best, bi, sv, si);
        if (t.world == 0) {
            if (threadIdx.x == 0) out[row] = bi == 0x7fffffff ? 0 : bi;
        } else {
            if (threadIdx.x == 0) {
                const uint32_t gi = bi == 0x7fffffff ? 0x7fffffffu : (uint32_t)(bi + t.vocab_off);
                s_pack = ((unsigned long long)__float_as_uint(best) << 32) | gi;
            }
            __syncthreads();
            const uint32_t ep = *t.epoch;
            if (threadIdx.x < t.world) {
                t.peer_slot[threadIdx.x][row] = s_pack;
                __threadfence_system();
                st_release_sys(t.peer_flag[threadIdx.x] + row, ep);
                if (!wait_seq<true>(t.my_flags + (int64_t)threadIdx.x * t.batch_cap + row, ep, t.limit_ns))
                    atomicOr(err, ERRBIT_PEER_TIMEOUT);
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                float gb = -INFINITY;
                int gx = 0x7fffffff;
                for (int r = 0; r < t.world; r++) {
                    const unsigned long long v =
                        __ldcg(reinterpret_cast<const unsigned long long *>(t.my_inbox) + (int64_t)r * t.batch_cap + row);
                    argmax_merge(gb, gx, __uint_as_float((uint32_t)(v >> 32)), (int)(uint32_t)v);
                }
                out[row] = gx == 0x7fffffff ? 0 : gx;
            }
        }
    }
    pdl_launch();
}

// ------------------------------------------------------------------------
// Batched prefill (T token rows at once, f32 in and out; the projections run
// on the tensor cores in between).
//
// x[t] = dequantized embedding row of tokens[t]; one CTA per row.
__global__ void __launch_bounds__(256) k_embed_rows(const uint8_t *__restrict__ emb, const int32_t *__restrict__ tokens,
                                                    int vocab, int dim, float *__restrict__ x, uint32_t *err) {
    const int64_t row = blockIdx.x;
    int tok = tokens[row];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) atomicOr(err, ERRBIT_BAD_TOKEN);
        tok = 0;
    }
    const int nbe = dim / QK;
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        x[row * dim + i] = q4k_value(emb + q4k_offset(tok, i / QK, nbe), i % QK);
}

// The fp16 operand of the prefill GEMM from one row's values (one 256-thread
// CTA per row; value(i) recomputes them): the power-of-two scale s = 2^e, the
// smallest e >= 0 with max |v| / s <= 32768, into *rs and fp16(v / s) into
// xh -- the rule of launch_x_to_f16, so the operands are the same bits.
// The exponent e of that scale from each thread's partial max |v|.
__device__ __forceinline__ int x16_row_exponent(float amax, float *shm) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if ((threadIdx.x & 31) == 0) shm[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = shm[0];
#pragma unroll
    for (int w = 1; w < 8; w++) amax = fmaxf(amax, shm[w]);
    int e = 0;
    while (e < 120 && amax > ldexpf(32768.f, e)) e++;
    return e;
}
template <class F>
__device__ __forceinline__ void x16_row_store(float amax, float *shm, F value, int dim, __half *xh, float *rs) {
    const int e = x16_row_exponent(amax, shm);
    const float inv = ldexpf(1.f, -e);
    if (threadIdx.x == 0) *rs = ldexpf(1.f, e);
    for (int i = threadIdx.x; i < dim; i += 256) xh[i] = __float2half_rn(__fmul_rn(value(i), inv));
}

// x[t] (+= y[t] when y != null), xn[t] = RMSNorm(x[t]) * g: the decode
// step's residual + RMSNorm arithmetic (binary64 sum of squares), without
// the Q8_K quantization.  One CTA per row.
__global__ void __launch_bounds__(256) k_add_rmsnorm_rows(float *__restrict__ x, const float *__restrict__ y,
                                                          const float *__restrict__ g, float *__restrict__ xn, int dim,
                                                          float eps, __half *__restrict__ xh, float *__restrict__ rs) {
    __shared__ double sh[8];
    __shared__ float shm[8];
    const int64_t row = blockIdx.x;
    float *xr = x + row * dim;
    double ss = 0.0;
    for (int i = threadIdx.x; i < dim; i += 256) {
        float v = xr[i];
        if (y) {
            v = __fadd_rn(y[row * dim + i], v);
            xr[i] = v;
        }
        ss = __fma_rn((double)v, (double)v, ss);
    }
    ss = block_sum64<8>(ss, sh);
    const float m = rms_of(ss, dim, eps);
    float amax = 0.f;
    for (int i = threadIdx.x; i < dim; i += 256) {
        const float v = __fmul_rn(__fdiv_rn(xr[i], m), g[i]);
        if (xn) xn[row * dim + i] = v;
        amax = fmaxf(amax, fabsf(v));
    }
    if (xh) x16_row_store(amax, shm, [&](int i) { return __fmul_rn(__fdiv_rn(xr[i], m), g[i]); }, dim,
                          xh + row * dim, rs + row);
}

// The same rows with the row held in registers (dim <= 1024 P, dim % 4 ==
// 0): float4 loads, x and y read once, one division per value.  The sum of
// squares runs in the order of the decode step's k_residual_rmsnorm_q8k
// (thread t: float4s t, t + 256, ...; x, y, z, w in order; then the block
// tree), so a prompt row normalizes to the same bits as a decoded one.
template <int P>
__global__ void __launch_bounds__(256) k_add_rmsnorm_rows4(float *__restrict__ x, const float *__restrict__ y,
                                                           const float *__restrict__ g, float *__restrict__ xn,
                                                           int dim, float eps, __half *__restrict__ xh,
                                                           float *__restrict__ rs) {
    __shared__ double sh[8];
    __shared__ float shm[8];
    const int64_t row = blockIdx.x;
    float4 *x4 = reinterpret_cast<float4 *>(x + row * dim);
    const int nv = dim / 4;
    float4 v[P];
#pragma unroll
    for (int p = 0; p < P; p++) {
        const int i = threadIdx.x + p * 256;
        v[p] = i < nv ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (y) {
        const float4 *y4 = reinterpret_cast<const float4 *>(y + row * dim);
#pragma unroll
        for (int p = 0; p < P; p++) {
            const int i = threadIdx.x + p * 256;
            if (i < nv) {
                const float4 d = y4[i];
                v[p] = make_float4(__fadd_rn(d.x, v[p].x), __fadd_rn(d.y, v[p].y), __fadd_rn(d.z, v[p].z),
                                   __fadd_rn(d.w, v[p].w));
                x4[i] = v[p];
            }
        }
    }
    double ss = 0.0;
#pragma unroll
    for (int p = 0; p < P; p++) {
        if (threadIdx.x + p * 256 < nv) {
            ss = __fma_rn((double)v[p].x, (double)v[p].x, ss);
            ss = __fma_rn((double)v[p].y, (double)v[p].y, ss);
            ss = __fma_rn((double)v[p].z, (double)v[p].z, ss);
            ss = __fma_rn((double)v[p].w, (double)v[p].w, ss);
        }
    }
    ss = block_sum64<8>(ss, sh);
    const float m = rms_of(ss, dim, eps);
    const float4 *g4 = reinterpret_cast<const float4 *>(g);
    float amax = 0.f;
#pragma unroll
    for (int p = 0; p < P; p++) {
        const int i = threadIdx.x + p * 256;
        if (i < nv) {
            const float4 gg = g4[i];
            v[p] = make_float4(__fmul_rn(__fdiv_rn(v[p].x, m), gg.x), __fmul_rn(__fdiv_rn(v[p].y, m), gg.y),
                               __fmul_rn(__fdiv_rn(v[p].z, m), gg.z), __fmul_rn(__fdiv_rn(v[p].w, m), gg.w));
            if (xn) reinterpret_cast<float4 *>(xn + row * dim)[i] = v[p];
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[p].x), fabsf(v[p].y)), fmaxf(fabsf(v[p].z), fabsf(v[p].w))));
        }
    }
    if (xh) {
        const int e = x16_row_exponent(amax, shm);
        const float inv = ldexpf(1.f, -e);
        if (threadIdx.x == 0) rs[row] = ldexpf(1.f, e);
        uint2 *xh4 = reinterpret_cast<uint2 *>(xh + row * dim);
#pragma unroll
        for (int p = 0; p < P; p++) {
            const int i = threadIdx.x + p * 256;
            if (i < nv) {
                const __half2 a = __halves2half2(__float2half_rn(__fmul_rn(v[p].x, inv)),
                                                 __float2half_rn(__fmul_rn(v[p].y, inv)));
                const __half2 b = __halves2half2(__float2half_rn(__fmul_rn(v[p].z, inv)),
                                                 __float2half_rn(__fmul_rn(v[p].w, inv)));
                xh4[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
            }
        }
    }
}

// act[t][i] = silu(gate) * up for the rows y[t] = [gate (f) | up (f)]
// (batched prefill, the float path: silu in f32, gate / (1 + e^-gate),
// within an ulp of the decode path's binary64 form).  grid (f / 1024, T):
// thread = four consecutive values of one row, vectorised.
__global__ void __launch_bounds__(256) k_swiglu_rows(const float *__restrict__ y, int f, int64_t rows,
                                                     float *__restrict__ act) {
    const int64_t r = blockIdx.y;
    const int c = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (r >= rows || c >= f) return;
    const float4 g = *reinterpret_cast<const float4 *>(y + r * 2 * f + c);
    const float4 u = *reinterpret_cast<const float4 *>(y + r * 2 * f + f + c);
    auto sw = [](float gv, float uv) { return __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.f, expf(-gv))), uv); };
    *reinterpret_cast<float4 *>(act + r * f + c) = make_float4(sw(g.x, u.x), sw(g.y, u.y), sw(g.z, u.z), sw(g.w, u.w));
}

// The same SwiGLU as the fp16 operand of the down projection, no f32
// output: one CTA per row, the row's values computed once (float4 loads)
// into shared memory, then scaled and stored by x16_row_store.
__global__ void __launch_bounds__(256) k_swiglu_rows_x16(const float *__restrict__ y, int f,
                                                         __half *__restrict__ xh, float *__restrict__ rs) {
    extern __shared__ float act[];  // [f]
    __shared__ float shm[8];
    const int64_t r = blockIdx.x;
    const float4 *g4 = reinterpret_cast<const float4 *>(y + r * 2 * f), *u4 = g4 + f / 4;
    auto sw = [](float gv, float uv) { return __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.f, expf(-gv))), uv); };
    float amax = 0.f;
    // four float4 pairs in flight per thread (the kernel streams the row once)
#pragma unroll 4
    for (int i = threadIdx.x; i < f / 4; i += 256) {
        const float4 g = g4[i], u = u4[i];
        const float4 a = make_float4(sw(g.x, u.x), sw(g.y, u.y), sw(g.z, u.z), sw(g.w, u.w));
        reinterpret_cast<float4 *>(act)[i] = a;
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
    }
    // x16_row_store's rule, four values per thread and 8-byte stores
    // (x16_row_exponent's __syncthreads orders the act writes before the reads)
    const int e = x16_row_exponent(amax, shm);
    const float inv = ldexpf(1.f, -e);
    if (threadIdx.x == 0) rs[r] = ldexpf(1.f, e);
    uint2 *xh4 = reinterpret_cast<uint2 *>(xh + r * f);
#pragma unroll 4
    for (int i = threadIdx.x; i < f / 4; i += 256) {
        const float4 a = reinterpret_cast<const float4 *>(act)[i];
        const __half2 lo = __halves2half2(__float2half_rn(__fmul_rn(a.x, inv)), __float2half_rn(__fmul_rn(a.y, inv)));
        const __half2 hi = __halves2half2(__float2half_rn(__fmul_rn(a.z, inv)), __float2half_rn(__fmul_rn(a.w, inv)));
        xh4[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&lo), *reinterpret_cast<const uint32_t *>(&hi));
    }
}

// Prefill prologue of attention for T new tokens at positions pos0 + t, per
// (token, head) of the projection output y[t] = (q | k | v): QK RMSNorm
// (optional) and RoPE of q (-> q_out f32 [T][n_heads][hd]) and k, and the
// fp16 KV-cache write of k (dim-major pages) and v (token-major) -- the decode
// attention prologue's arithmetic, token by token.  One CTA per (32
// consecutive tokens, head); warp w takes tokens w, w + 8, w + 16, w + 24 of
// the group and issues their loads before the arithmetic.  A k head's values
// pass through shared memory so that each dim row of a page is written as
// consecutive tokens (64 contiguous bytes per warp, not 2-byte scatter).
constexpr int QR_TT = 32;  // tokens per CTA
__global__ void __launch_bounds__(256) k_prefill_qkv_rope(const float *__restrict__ y, int64_t ld, int T, int pos0,
                                                          int n_heads, int n_kv, const float *__restrict__ q_norm,
                                                          const float *__restrict__ k_norm, float eps,
                                                          const float *__restrict__ rope_cos,
                                                          const float *__restrict__ rope_sin, int rope_mode,
                                                          float *__restrict__ q_out, __half *__restrict__ kpool,
                                                          __half *__restrict__ vpool, const int32_t *__restrict__ bt,
                                                          int page_size, int num_pages, uint32_t *err) {
    constexpr int TPW = QR_TT / 8;          // tokens per warp
    __shared__ __half kst[128][QR_TT + 1];  // k head: [dim][token of the group]
    __shared__ int s_page[QR_TT], s_slot[QR_TT];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hh = blockIdx.y, t0 = blockIdx.x * QR_TT;
    const bool is_q = hh < n_heads, is_k = !is_q && hh < n_heads + n_kv;
    const int kvh = is_k ? hh - n_heads : hh - n_heads - n_kv;
    if (!is_q && threadIdx.x < QR_TT) {
        // cache page and slot of each token of the group (-1: not written)
        const int t = t0 + (int)threadIdx.x;
        int page = -1, slot = 0;
        if (t < T) {
            const int p = pos0 + t;
            page = bt[p / page_size];
            slot = p % page_size;
            if (page < 0 || page >= num_pages) {
                atomicOr(err, ERRBIT_BAD_PAGE);
                page = -1;
            }
        }
        s_page[threadIdx.x] = page;
        s_slot[threadIdx.x] = slot;
    }
    float v[TPW][4];
#pragma unroll
    for (int i = 0; i < TPW; i++) {
        const int t = t0 + warp + 8 * i;
        const float4 x4 = t < T ? *reinterpret_cast<const float4 *>(y + (int64_t)t * ld + (int64_t)hh * 128 + 4 * lane)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        v[i][0] = x4.x;
        v[i][1] = x4.y;
        v[i][2] = x4.z;
        v[i][3] = x4.w;
    }
    if (is_q || is_k) {
#pragma unroll
        for (int i = 0; i < TPW; i++) {
            const int t = t0 + warp + 8 * i;
            if (t < T) {  // warp-uniform
                const int p = pos0 + t;
                const QkHead qh = qk_head_load(lane, q_norm ? (is_q ? q_norm : k_norm) : nullptr,
                                               rope_cos + (int64_t)p * 64, rope_sin + (int64_t)p * 64, rope_mode);
                qk_head_apply(v[i], lane, qh, eps, rope_mode);
            }
        }
    }
    if (is_q) {
#pragma unroll
        for (int i = 0; i < TPW; i++) {
            const int t = t0 + warp + 8 * i;
            if (t < T)
                *reinterpret_cast<float4 *>(q_out + ((int64_t)t * n_heads + hh) * 128 + 4 * lane) =
                    make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
        }
        return;  // uniform over the CTA: no barrier follows for q heads
    }
    if (is_k) {
#pragma unroll
        for (int i = 0; i < TPW; i++)
#pragma unroll
            for (int e = 0; e < 4; e++) kst[4 * lane + e][warp + 8 * i] = __float2half_rn(v[i][e]);
    }
    __syncthreads();  // s_page / s_slot, and the k tile
    if (!is_k) {
        // v: token-major pages, 8 bytes per lane and token
#pragma unroll
        for (int i = 0; i < TPW; i++) {
            const int tl = warp + 8 * i, page = s_page[tl];
            if (t0 + tl < T && page >= 0) {
                const __half2 a = __halves2half2(__float2half_rn(v[i][0]), __float2half_rn(v[i][1]));
                const __half2 b = __halves2half2(__float2half_rn(v[i][2]), __float2half_rn(v[i][3]));
                *reinterpret_cast<uint2 *>(vpool + (((size_t)page * n_kv + kvh) * page_size + s_slot[tl]) * 128 +
                                           4 * lane) =
                    make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
            }
        }
        return;
    }
    // k: dim-major pages; consecutive threads take consecutive tokens of one dim
    for (int idx = threadIdx.x; idx < 128 * QR_TT; idx += 256) {
        const int tl = idx % QR_TT, d = idx / QR_TT, page = s_page[tl];
        if (t0 + tl < T && page >= 0)
            kpool[(((size_t)page * n_kv + kvh) * 128 + d) * page_size + s_slot[tl]] = kst[d][tl];
    }
}

void launch_embed_rows(fb_ctx *ctx, const fb_qtensor *emb, const int32_t *tokens, int T, int vocab, int dim,
                       float *x) {
    FB_REQUIRE(emb->dtype == FB_Q4_K && emb->k == dim, "embedding table must be Q4_K [vocab, hidden]");
    k_embed_rows<<<T, 256, 0, ctx->stream>>>(emb->main(), tokens, vocab, dim, x, ctx->err_word);
    FB_CUDA(cudaGetLastError());
}

void launch_add_rmsnorm_rows(fb_ctx *ctx, float *x, const float *y, const float *g, float *xn, int T, int dim,
                             float eps, __half *xh, float *rs) {
    FB_REQUIRE(xn || (xh && rs), "add_rmsnorm_rows: no output");
    cudaStream_t s = ctx->stream;
    if (dim % 4 != 0 || dim > 8192) k_add_rmsnorm_rows<<<T, 256, 0, s>>>(x, y, g, xn, dim, eps, xh, rs);
    else if (dim <= 1024) k_add_rmsnorm_rows4<1><<<T, 256, 0, s>>>(x, y, g, xn, dim, eps, xh, rs);
    else if (dim <= 2048) k_add_rmsnorm_rows4<2><<<T, 256, 0, s>>>(x, y, g, xn, dim, eps, xh, rs);
    else if (dim <= 4096) k_add_rmsnorm_rows4<4><<<T, 256, 0, s>>>(x, y, g, xn, dim, eps, xh, rs);
    else k_add_rmsnorm_rows4<8><<<T, 256, 0, s>>>(x, y, g, xn, dim, eps, xh, rs);
    FB_CUDA(cudaGetLastError());
}

void launch_swiglu_rows_x16(fb_ctx *ctx, const float *y, int f, int T, __half *xh, float *rs) {
    FB_REQUIRE(f % 4 == 0 && (size_t)f * 4 <= 200 * 1024, "swiglu_rows_x16: f must be a multiple of 4, <= 51200");
    const size_t smem = (size_t)f * 4;
    FB_CUDA(cudaFuncSetAttribute(k_swiglu_rows_x16, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_swiglu_rows_x16<<<(unsigned)T, 256, smem, ctx->stream>>>(y, f, xh, rs);
    FB_CUDA(cudaGetLastError());
}

void launch_swiglu_rows(fb_ctx *ctx, const float *y, int f, int T, float *act) {
    FB_REQUIRE(f % 4 == 0 && T >= 1 && T <= 65535, "swiglu_rows: f must be a multiple of 4, 1 <= T <= 65535");
    k_swiglu_rows<<<dim3((unsigned)((f / 4 + 255) / 256), (unsigned)T), 256, 0, ctx->stream>>>(y, f, T, act);
    FB_CUDA(cudaGetLastError());
}

void launch_prefill_qkv_rope(fb_ctx *ctx, const float *y, int64_t ld, int T, int pos0, int n_heads, int n_kv,
                             const float *q_norm, const float *k_norm, float eps, const float *rope_cos,
                             const float *rope_sin, int rope_mode, float *q_out, void *kpool, void *vpool,
                             const int32_t *bt, int page_size, int num_pages) {
    FB_REQUIRE(T >= 1 && n_heads + 2 * n_kv <= 65535 && ld % 4 == 0, "prefill_qkv_rope: bad shape");
    const dim3 grid((unsigned)((T + QR_TT - 1) / QR_TT), (unsigned)(n_heads + 2 * n_kv));
    k_prefill_qkv_rope<<<grid, 256, 0, ctx->stream>>>(
        y, ld, T, pos0, n_heads, n_kv, q_norm, k_norm, eps, rope_cos, rope_sin, rope_mode, q_out, (__half *)kpool,
        (__half *)vpool, bt, page_size, num_pages, ctx->err_word);
    FB_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------------
// Standalone ops for the C ABI.
__global__ void k_rmsnorm(const float *__restrict__ x, const float *__restrict__ g, float *__restrict__ y, int64_t dim,
                          float eps) {
    __shared__ double sh[8];
    const float *xr = x + (int64_t)blockIdx.x * dim;
    float *yr = y + (int64_t)blockIdx.x * dim;
    double ss = 0.0;
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) ss = __fma_rn((double)xr[i], (double)xr[i], ss);
    ss = block_sum64<8>(ss, sh);
    const float m = rms_of(ss, (int)dim, eps);
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) yr[i] = __fmul_rn(__fdiv_rn(xr[i], m), g[i]);
}

__global__ void k_rope(float *__restrict__ x, int64_t n_tok, int64_t n_heads, int64_t hd, int64_t pos0,
                       const float *__restrict__ cos_t, const float *__restrict__ sin_t, int mode) {
    const int64_t half = hd / 2;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // over tok*heads*half
    if (idx >= n_tok * n_heads * half) return;
    const int64_t i = idx % half, th = idx / half, t = th / n_heads;
    float *xh = x + th * hd;
    const int64_t a = mode ? i : 2 * i, b = mode ? i + half : 2 * i + 1;
    const float c = cos_t[(pos0 + t) * half + i], s = sin_t[(pos0 + t) * half + i];
    const float x0 = xh[a], x1 = xh[b];
    xh[a] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    xh[b] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

__global__ void k_swiglu(const float *__restrict__ g, const float *__restrict__ u, float *__restrict__ o, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    o[i] = __fmul_rn(silu64(g[i]), u[i]);
}

void launch_rmsnorm(fb_ctx *ctx, const float *x, const float *g, float *y, int64_t rows, int64_t dim, float eps) {
    k_rmsnorm<<<(unsigned)rows, 256, 0, ctx->stream>>>(x, g, y, dim, eps);
    FB_CUDA(cudaGetLastError());
}

void launch_rope(fb_ctx *ctx, float *x, int64_t n_tok, int64_t n_heads, int64_t hd, int64_t pos0,
                 const float *cos_tab, const float *sin_tab, int mode) {
    const int64_t n = n_tok * n_heads * (hd / 2);
    k_rope<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(x, n_tok, n_heads, hd, pos0, cos_tab, sin_tab, mode);
    FB_CUDA(cudaGetLastError());
}

void launch_swiglu(fb_ctx *ctx, const float *g, const float *u, float *out, int64_t m, int64_t f) {
    const int64_t n = m * f;
    k_swiglu<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(g, u, out, n);
    FB_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------------
// PDL launch helper for the fused step kernels.
template <typename K, typename... Args>
static void launch_k(fb_ctx *ctx, K kernel, dim3 grid, dim3 block, size_t smem, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = ctx->pdl ? 1 : 0;
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    FB_CUDA(cudaLaunchKernelEx(&cfg, kernel, args...));
}

void launch_residual_rmsnorm_q8k(fb_ctx *ctx, const float *x, const float *add, float *x_out, const float *g, int rows,
                                 int dim, float eps, const Q8Act &a, const fb_qtensor *emb, const int32_t *tokens,
                                 int vocab) {
    FB_REQUIRE(dim % QK == 0, "rmsnorm_q8k: dim must be a multiple of 256");
    const uint8_t *tab = nullptr;
    if (emb) {
        FB_REQUIRE(emb->dtype == FB_Q4_K && emb->k == dim, "embedding table must be Q4_K [vocab, hidden]");
        tab = emb->main();
    }
    FB_REQUIRE(x_out != x, "rmsnorm_q8k: x_out must not alias x");
    if (tab)
        launch_k(ctx, k_residual_rmsnorm_q8k<true>, dim3(dim / QK, rows), dim3(NORM_THREADS), 0, x, add, x_out, g, dim,
                 eps, a, tab, tokens, vocab, ctx->err_word, (uint32_t *)nullptr);
    else
        launch_k(ctx, k_residual_rmsnorm_q8k<false>, dim3(dim / QK, rows), dim3(NORM_THREADS), 0, x, add, x_out, g,
                 dim, eps, a, tab, tokens, vocab, ctx->err_word, (uint32_t *)nullptr);
}

void launch_embed_rmsnorm_q8k(fb_ctx *ctx, float *x_out, const float *g, int rows, int dim, float eps,
                              const Q8Act &a, const fb_qtensor *emb, const int32_t *tokens, int vocab,
                              uint32_t *epoch_inc) {
    FB_REQUIRE(dim % QK == 0, "rmsnorm_q8k: dim must be a multiple of 256");
    FB_REQUIRE(emb && emb->dtype == FB_Q4_K && emb->k == dim, "embedding table must be Q4_K [vocab, hidden]");
    launch_k(ctx, k_residual_rmsnorm_q8k<true>, dim3(dim / QK, rows), dim3(NORM_THREADS), 0, (const float *)nullptr,
             (const float *)nullptr, x_out, g, dim, eps, a, emb->main(), tokens, vocab, ctx->err_word, epoch_inc);
}

void launch_tp_residual_rmsnorm_q8k(fb_ctx *ctx, const float *x, float *x_out, const float *g, int rows, int dim,
                                    float eps, const Q8Act &a, const TpNorm &t, int xi) {
    FB_REQUIRE(dim % QK == 0 && dim / QK <= NORM_THREADS, "tp rmsnorm: dim must be a multiple of 256, <= 65536");
    FB_REQUIRE(rows <= t.batch_cap && t.world >= 1 && t.world <= FB_TP_MAX, "tp rmsnorm: bad rows / world");
    FB_REQUIRE(x_out != x, "rmsnorm_q8k: x_out must not alias x");
    launch_k(ctx, k_tp_residual_rmsnorm_q8k, dim3(dim / QK, rows), dim3(NORM_THREADS), 0, x, x_out, g, dim, eps, a, t,
             xi, ctx->err_word);
}

void launch_swiglu_q8k(fb_ctx *ctx, const float *y, int f, int rows, const Q8Act &a) {
    const int64_t blocks = (int64_t)rows * (f / QK);
    launch_k(ctx, k_swiglu_q8k, dim3((unsigned)blocks), dim3(QK), 0, y, f, (int64_t)rows, a);
}

size_t argmax_ws_bytes(int rows) { return (size_t)rows * ARGMAX_CHUNKS * 8 + (size_t)rows * 4; }

void launch_argmax(fb_ctx *ctx, const float *logits, int rows, int64_t vocab, int32_t *out, void *ws) {
    // ws: values, indices, counters (zero on first use, zero again after each launch)
    float *wv = static_cast<float *>(ws);
    int *wi = reinterpret_cast<int *>(wv + (size_t)rows * ARGMAX_CHUNKS);
    int *cnt = wi + (size_t)rows * ARGMAX_CHUNKS;
    const int chunks = (int)std::min<int64_t>(ARGMAX_CHUNKS, (vocab + 1023) / 1024);
    launch_k(ctx, k_argmax, dim3(chunks, rows), dim3(256), 0, logits, vocab, out, wv, wi, cnt, TpArgmax{},
             ctx->err_word);
}

void launch_argmax_tp(fb_ctx *ctx, const float *logits, int rows, int64_t vocab, int32_t *out, void *ws,
                      const TpArgmax &t) {
    FB_REQUIRE(t.world >= 1 && t.world <= FB_TP_MAX && rows <= t.batch_cap, "argmax: bad tensor-parallel args");
    float *wv = static_cast<float *>(ws);
    int *wi = reinterpret_cast<int *>(wv + (size_t)rows * ARGMAX_CHUNKS);
    int *cnt = wi + (size_t)rows * ARGMAX_CHUNKS;
    const int chunks = (int)std::min<int64_t>(ARGMAX_CHUNKS, (vocab + 1023) / 1024);
    launch_k(ctx, k_argmax, dim3(chunks, rows), dim3(256), 0, logits, vocab, out, wv, wi, cnt, t, ctx->err_word);
}

void rope_tables(int max_pos, int head_dim, float theta, std::vector<float> &cos_t, std::vector<float> &sin_t) {
    const int half = head_dim / 2;
    cos_t.resize((size_t)max_pos * half);
    sin_t.resize((size_t)max_pos * half);
    for (int i = 0; i < half; i++) {
        // same expression as the oracle's rope_inv_freq / or_rope
        const float inv = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
        for (int p = 0; p < max_pos; p++) {
            const float ang = (float)p * inv;
            cos_t[(size_t)p * half + i] = cosf(ang);
            sin_t[(size_t)p * half + i] = sinf(ang);
        }
    }
}

}  // namespace fb

namespace fb {

static uint64_t kv_mix64_host(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Synthetic KV fill (bench / parity setup): value of (layer, K|V, position p,
// element e = kv_head*hd + d) = fp16(scale*sqrt(3)*(2u - 1)), u the 24-bit
// uniform of splitmix64(mix(seed) ^ ((layer*2 + which) << 40 | p << 20 | e)).
// The CPU oracle's or_model_synth_kv uses the same function.
__device__ __forceinline__ uint64_t kv_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void k_synth_kv(__half *__restrict__ pool, int layer, int which, int ctx, int nkv, int hd, int page_size,
                           const int32_t *__restrict__ block_table, int max_pages, int slots, uint64_t sm,
                           float s3, int e0) {
    const int64_t kd = (int64_t)nkv * hd;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // over ctx * kd
    if (i >= (int64_t)ctx * kd) return;
    const int p = (int)(i / kd);
    const int e = (int)(i % kd);
    const uint64_t idx = (((uint64_t)layer * 2u + (uint64_t)which) << 40) | ((uint64_t)p << 20) | (uint64_t)(e0 + e);
    const uint64_t h = kv_mix64(sm ^ idx);
    const float u = (float)(h >> 40) * (1.0f / 16777216.0f);
    const __half v = __float2half_rn(__fmul_rn(s3, __fsub_rn(__fmul_rn(2.0f, u), 1.0f)));
    const int kvh = e / hd, d = e % hd;
    for (int s = 0; s < slots; s++) {
        const int page = block_table[(int64_t)s * max_pages + p / page_size];
        if (which == 0)  // K: dim-major pages
            pool[(((int64_t)page * nkv + kvh) * hd + d) * page_size + (p % page_size)] = v;
        else
            pool[(((int64_t)page * nkv + kvh) * page_size + (p % page_size)) * hd + d] = v;
    }
}

void launch_synth_kv(fb_ctx *ctx, void *pool, int layer, int which, int nctx, int nkv, int hd, int page_size,
                     const int32_t *block_table, int max_pages, int slots, uint64_t seed, float scale, int kv_head0) {
    const int64_t n = (int64_t)nctx * nkv * hd;
    if (n == 0) return;
    k_synth_kv<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(
        (__half *)pool, layer, which, nctx, nkv, hd, page_size, block_table, max_pages, slots, kv_mix64_host(seed),
        scale * 1.7320508f, kv_head0 * hd);
    FB_CUDA(cudaGetLastError());
}

}  // namespace fb
