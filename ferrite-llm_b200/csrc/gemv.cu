// Decode GEMV for GGUF Q4_K / Q6_K weights against Q8_K activations
// (batch m = 1..16): y[m, n] = x[m, k] . W[n, k]^T.
//
// Arithmetic = candle-core 0.8.4 CPU QMatMul (crates/ferrite-wasm-host/src/
// adapter.rs:61-70 -> QMatMul::forward): activations quantized to Q8_K, then
// per super-block the integer sums  sum_j sc_j * (q_w . q_x)_j  (and for Q4_K
// sum_j m_j * bsum_j) combined in f32 with the fp16 super-block scales.  The
// reference's GPU kernels for the same op are the dp4a MMVQ kernels
// mul_mat_vec_q{4,6}_K_q8_1 (ptx-kernels/kernels/candle/quantized.cu:2627-3344).
//
// B200 design: the op is HBM-bound (0.5625 / 0.8203 weight bytes per MAC at
// m = 1), so every weight byte is read exactly once with 16-byte streaming
// loads that bypass L1.  The integer dot of each 32-value (Q4_K) or 16-value
// (Q6_K) sub-block runs on the tensor pipe as mma.m16n8k32.s8 (16 weight rows
// x 8 activation rows per instruction), which keeps the ALU budget per weight
// byte flat from m = 1 to m = 16; integer partials are exact, so the
// per-sub-block scales are applied in int32 exactly as the CPU path does, and
// the per-super-block float combine runs in binary64 with one rounding to f32
// (bit-identical to the CPU oracle whatever the block summation order).
// The device weight layouts (see fb_qtensor) put each MMA quad lane's bytes
// contiguously, and the Q8_K activation layout (see Q8Act) matches the MMA B
// fragment, so no shuffles or shared-memory staging are needed.
//
// CTA = 8 warps on one 16-row tile; warp w takes super-blocks w, w+8, ...;
// partial sums are reduced across warps through shared memory (fixed order,
// deterministic).  Thread (gid = lane/4, tig = lane%4) owns weight rows gid
// and gid+8 and output columns 2*tig, 2*tig+1 of each 8-wide n-tile.
#include "fb_internal.h"
#include "kq_common.cuh"

namespace fb {

constexpr int GEMV_WARPS = 8;

template <int NT>
struct ActBlock {
    uint32_t b[NT][16];  // B fragments: sub-block s uses (b[2s], b[2s+1])
};

// Loads the B fragments of super-block `blk` for the NT n-tiles (columns
// nt*8 + gid); columns >= m read as zero.
template <int NT>
__device__ __forceinline__ void load_act(const Q8Act &a, int m, int64_t blk, int gid, int tig, ActBlock<NT> &ab) {
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const int col = nt * 8 + gid;
        if (col < m) {
            const int8_t *p = a.qs + (int64_t)col * a.k + blk * QK + 64 * tig;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                uint4 v = ld_act16(p + 16 * i);
                ab.b[nt][4 * i + 0] = v.x;
                ab.b[nt][4 * i + 1] = v.y;
                ab.b[nt][4 * i + 2] = v.z;
                ab.b[nt][4 * i + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; i++) ab.b[nt][i] = 0u;
        }
    }
}

__device__ __forceinline__ float act_d(const Q8Act &a, int m, int col, int64_t blk, int64_t nbk) {
    return col < m ? a.d[(int64_t)col * nbk + blk] : 0.f;
}

template <int NT, bool DOTS>
__device__ __forceinline__ void write_out(double (&acc)[NT][4], double *red, int warp, int gid, int tig, int64_t row0,
                                          int64_t n, int m, float *y, int64_t ldy) {
    constexpr int C = 8 * NT;
    // red[w][r][c] with a padded row to keep the stores conflict-light
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int r = gid + 8 * (i >> 1), c = nt * 8 + 2 * tig + (i & 1);
            red[(warp * 16 + r) * (C + 1) + c] = acc[nt][i];
        }
    __syncthreads();
    for (int o = threadIdx.x; o < 16 * C; o += blockDim.x) {
        const int r = o / C, c = o % C;
        double s = 0.0;
#pragma unroll
        for (int w = 0; w < GEMV_WARPS; w++) s = __dadd_rn(s, red[(w * 16 + r) * (C + 1) + c]);
        const int64_t row = row0 + r;
        if (row < n && c < m) y[(int64_t)c * ldy + row] = __double2float_rn(s);
    }
}

// ---------------------------------------------------------------- Q4_K ---
template <int NT, bool DOTS>
__global__ void __launch_bounds__(256) k_gemv_q4k(const uint8_t *__restrict__ W, int64_t n, int nb, Q8Act a, int m,
                                                  float *__restrict__ y, int64_t ldy, int32_t *__restrict__ dots_sc,
                                                  int32_t *__restrict__ dots_min) {
    __shared__ double red[GEMV_WARPS * 16 * (8 * NT + 1)];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const int64_t row0 = (int64_t)blockIdx.x * 16;
    const int64_t r0 = min(row0 + gid, n - 1), r1 = min(row0 + gid + 8, n - 1);
    const uint8_t *w0 = W + r0 * nb * 144;
    const uint8_t *w1 = W + r1 * nb * 144;

    double acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[nt][i] = 0.0;

    // Weights do not depend on the previous kernel: issue the first loads
    // before waiting on it.
    int b = warp;
    uint4 h0, h1, q0a, q0b, q1a, q1b;
    if (b < nb) {
        h0 = ld_stream16(w0 + b * 144);
        h1 = ld_stream16(w1 + b * 144);
        q0a = ld_stream16(w0 + b * 144 + 16 + 32 * tig);
        q0b = ld_stream16(w0 + b * 144 + 32 + 32 * tig);
        q1a = ld_stream16(w1 + b * 144 + 16 + 32 * tig);
        q1b = ld_stream16(w1 + b * 144 + 32 + 32 * tig);
    }
    pdl_wait();
    const int64_t nbk = nb;
    for (; b < nb; b += GEMV_WARPS) {
        ActBlock<NT> ab;
        load_act<NT>(a, m, b, gid, tig, ab);
        uint4 bs[NT][2];
        float dy[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int col = nt * 8 + 2 * tig + j;
                bs[nt][j] = col < m ? ld_act16(a.bs32 + (int64_t)col * (a.k / 32) + b * 8) : make_uint4(0, 0, 0, 0);
                dy[nt][j] = act_d(a, m, col, b, nbk);
            }
        const Q4Scales s0 = q4k_unpack_scales(h0.y, h0.z, h0.w);
        const Q4Scales s1 = q4k_unpack_scales(h1.y, h1.z, h1.w);
        const float dw0 = h2f(h0.x & 0xFFFF), dm0 = h2f(h0.x >> 16);
        const float dw1 = h2f(h1.x & 0xFFFF), dm1 = h2f(h1.x >> 16);
        const uint32_t W0[8] = {q0a.x, q0a.y, q0a.z, q0a.w, q0b.x, q0b.y, q0b.z, q0b.w};
        const uint32_t W1[8] = {q1a.x, q1a.y, q1a.z, q1a.w, q1b.x, q1b.y, q1b.z, q1b.w};

        // prefetch the next super-block of this warp
        const int bn = b + GEMV_WARPS;
        if (bn < nb) {
            h0 = ld_stream16(w0 + bn * 144);
            h1 = ld_stream16(w1 + bn * 144);
            q0a = ld_stream16(w0 + bn * 144 + 16 + 32 * tig);
            q0b = ld_stream16(w0 + bn * 144 + 32 + 32 * tig);
            q1a = ld_stream16(w1 + bn * 144 + 16 + 32 * tig);
            q1b = ld_stream16(w1 + bn * 144 + 32 + 32 * tig);
        }

        int isum[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) isum[nt][i] = 0;
#pragma unroll
        for (int s = 0; s < 8; s++) {
            const int g = s >> 1, sh = 4 * (s & 1);
            const uint32_t a0 = (W0[2 * g] >> sh) & 0x0F0F0F0Fu;
            const uint32_t a2 = (W0[2 * g + 1] >> sh) & 0x0F0F0F0Fu;
            const uint32_t a1 = (W1[2 * g] >> sh) & 0x0F0F0F0Fu;
            const uint32_t a3 = (W1[2 * g + 1] >> sh) & 0x0F0F0F0Fu;
            const int sc0 = byte_of(s < 4 ? s0.sc_lo : s0.sc_hi, s & 3);
            const int sc1 = byte_of(s < 4 ? s1.sc_lo : s1.sc_hi, s & 3);
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                int c[4] = {0, 0, 0, 0};
                mma_k32(c, a0, a1, a2, a3, ab.b[nt][2 * s], ab.b[nt][2 * s + 1]);
                isum[nt][0] += sc0 * c[0];
                isum[nt][1] += sc0 * c[1];
                isum[nt][2] += sc1 * c[2];
                isum[nt][3] += sc1 * c[3];
            }
        }
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int j = i & 1;
                const Q4Scales &sr = (i < 2) ? s0 : s1;
                const uint4 q = bs[nt][j];
                int msum = __dp2a_lo((int)q.x, (int)sr.mn_lo, 0);
                msum = __dp2a_hi((int)q.y, (int)sr.mn_lo, msum);
                msum = __dp2a_lo((int)q.z, (int)sr.mn_hi, msum);
                msum = __dp2a_hi((int)q.w, (int)sr.mn_hi, msum);
                if (DOTS) {
                    // integer partials for column 0 only
                    if (nt == 0 && tig == 0 && j == 0) {
                        const int64_t row = row0 + gid + 8 * (i >> 1);
                        if (row < n) {
                            dots_sc[row * nb + b] = isum[nt][i];
                            dots_min[row * nb + b] = msum;
                        }
                    }
                } else if (nt * 8 + 2 * tig + j < m) {
                    // binary64 combine: ((d * dy) * isum) - ((dmin * dy) * msum)
                    const double dw = (i < 2) ? dw0 : dw1, dm = (i < 2) ? dm0 : dm1;
                    const double yd = dy[nt][j];
                    acc[nt][i] = __dadd_rn(acc[nt][i], __dmul_rn(__dmul_rn(dw, yd), (double)isum[nt][i]));
                    acc[nt][i] = __dsub_rn(acc[nt][i], __dmul_rn(__dmul_rn(dm, yd), (double)msum));
                }
            }
    }
    pdl_launch();
    if (!DOTS) write_out<NT, DOTS>(acc, red, warp, gid, tig, row0, n, m, y, ldy);
}

// ---------------------------------------------------------------- Q6_K ---
// Each 32-value part (half h, part p) spans two 16-value scale groups; lanes
// with tig < 2 hold the first group's values and tig >= 2 the second's, so
// two MMAs with the B fragment masked by lane group separate them.
template <int NT, bool DOTS>
__global__ void __launch_bounds__(256) k_gemv_q6k(const uint8_t *__restrict__ W, const uint16_t *__restrict__ Wd,
                                                  int64_t n, int nb, Q8Act a, int m, float *__restrict__ y, int64_t ldy,
                                                  int32_t *__restrict__ dots_sc) {
    __shared__ double red[GEMV_WARPS * 16 * (8 * NT + 1)];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const uint32_t mlo = tig < 2 ? 0xFFFFFFFFu : 0u;
    const int64_t row0 = (int64_t)blockIdx.x * 16;
    const int64_t r0 = min(row0 + gid, n - 1), r1 = min(row0 + gid + 8, n - 1);
    const uint8_t *w0 = W + r0 * nb * 208;
    const uint8_t *w1 = W + r1 * nb * 208;
    const uint16_t *d0p = Wd + r0 * nb;
    const uint16_t *d1p = Wd + r1 * nb;

    double acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[nt][i] = 0.0;

    int b = warp;
    uint4 x0[3], x1[3], sc0v, sc1v;
    uint16_t dd0 = 0, dd1 = 0;
    if (b < nb) {
#pragma unroll
        for (int i = 0; i < 3; i++) {
            x0[i] = ld_stream16(w0 + b * 208 + 48 * tig + 16 * i);
            x1[i] = ld_stream16(w1 + b * 208 + 48 * tig + 16 * i);
        }
        sc0v = ld_stream16(w0 + b * 208 + 192);
        sc1v = ld_stream16(w1 + b * 208 + 192);
        dd0 = ld_stream_u16(d0p + b);
        dd1 = ld_stream_u16(d1p + b);
    }
    pdl_wait();
    for (; b < nb; b += GEMV_WARPS) {
        ActBlock<NT> ab;
        load_act<NT>(a, m, b, gid, tig, ab);
        uint4 bsa[NT][2], bsb[NT][2];  // bs16 of the two columns: groups 0..7, 8..15
        float dy[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int col = nt * 8 + 2 * tig + j;
                if (col < m) {
                    const int16_t *p = a.bs16 + (int64_t)col * (a.k / 16) + b * 16;
                    bsa[nt][j] = ld_act16(p);
                    bsb[nt][j] = ld_act16(p + 8);
                } else {
                    bsa[nt][j] = make_uint4(0, 0, 0, 0);
                    bsb[nt][j] = make_uint4(0, 0, 0, 0);
                }
                dy[nt][j] = act_d(a, m, col, b, nb);
            }
        const uint32_t Q0[12] = {x0[0].x, x0[0].y, x0[0].z, x0[0].w, x0[1].x, x0[1].y,
                                 x0[1].z, x0[1].w, x0[2].x, x0[2].y, x0[2].z, x0[2].w};
        const uint32_t Q1[12] = {x1[0].x, x1[0].y, x1[0].z, x1[0].w, x1[1].x, x1[1].y,
                                 x1[1].z, x1[1].w, x1[2].x, x1[2].y, x1[2].z, x1[2].w};
        const uint32_t S0[4] = {sc0v.x, sc0v.y, sc0v.z, sc0v.w};
        const uint32_t S1[4] = {sc1v.x, sc1v.y, sc1v.z, sc1v.w};
        const float dw0 = h2f(dd0), dw1 = h2f(dd1);

        const int bn = b + GEMV_WARPS;
        if (bn < nb) {
#pragma unroll
            for (int i = 0; i < 3; i++) {
                x0[i] = ld_stream16(w0 + bn * 208 + 48 * tig + 16 * i);
                x1[i] = ld_stream16(w1 + bn * 208 + 48 * tig + 16 * i);
            }
            sc0v = ld_stream16(w0 + bn * 208 + 192);
            sc1v = ld_stream16(w1 + bn * 208 + 192);
            dd0 = ld_stream_u16(d0p + bn);
            dd1 = ld_stream_u16(d1p + bn);
        }

        int isum[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) isum[nt][i] = 0;
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int p = 0; p < 4; p++) {
                const int s = 4 * h + p;
                const int lw = 4 * h + 2 * (p & 1), ls = 4 * (p >> 1);
                const int hw = 8 + 2 * h;
                // 6-bit quants (0..63) of values 8*tig + 4x + e of the part
                auto q6 = [&](const uint32_t *Q, int x) -> uint32_t {
                    const uint32_t lo = (Q[lw + x] >> ls) & 0x0F0F0F0Fu;
                    const uint32_t hi = (2 * p <= 4) ? ((Q[hw + x] << (4 - 2 * p)) & 0x30303030u)
                                                     : ((Q[hw + x] >> (2 * p - 4)) & 0x30303030u);
                    return lo | hi;
                };
                const uint32_t a0 = q6(Q0, 0), a2 = q6(Q0, 1), a1 = q6(Q1, 0), a3 = q6(Q1, 1);
                const int G = 8 * h + 2 * p;  // groups G (tig < 2) and G + 1
                const int s0a = sbyte_of(S0[G >> 2], G & 3), s0b = sbyte_of(S0[G >> 2], (G & 3) + 1);
                const int s1a = sbyte_of(S1[G >> 2], G & 3), s1b = sbyte_of(S1[G >> 2], (G & 3) + 1);
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    const uint32_t b0 = ab.b[nt][2 * s], b1 = ab.b[nt][2 * s + 1];
                    int ca[4] = {0, 0, 0, 0}, cb[4] = {0, 0, 0, 0};
                    mma_k32(ca, a0, a1, a2, a3, b0 & mlo, b1 & mlo);
                    mma_k32(cb, a0, a1, a2, a3, b0 & ~mlo, b1 & ~mlo);
                    isum[nt][0] += s0a * ca[0] + s0b * cb[0];
                    isum[nt][1] += s0a * ca[1] + s0b * cb[1];
                    isum[nt][2] += s1a * ca[2] + s1b * cb[2];
                    isum[nt][3] += s1a * ca[3] + s1b * cb[3];
                }
            }
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int j = i & 1;
                const uint32_t *S = (i < 2) ? S0 : S1;
                // sum_G sc_G * bsum16_G (quants are offset by +32)
                const uint4 qa = bsa[nt][j], qb = bsb[nt][j];
                int cs = __dp2a_lo((int)qa.x, (int)S[0], 0);
                cs = __dp2a_hi((int)qa.y, (int)S[0], cs);
                cs = __dp2a_lo((int)qa.z, (int)S[1], cs);
                cs = __dp2a_hi((int)qa.w, (int)S[1], cs);
                cs = __dp2a_lo((int)qb.x, (int)S[2], cs);
                cs = __dp2a_hi((int)qb.y, (int)S[2], cs);
                cs = __dp2a_lo((int)qb.z, (int)S[3], cs);
                cs = __dp2a_hi((int)qb.w, (int)S[3], cs);
                const int tot = isum[nt][i] - 32 * cs;
                if (DOTS) {
                    if (nt == 0 && tig == 0 && j == 0) {
                        const int64_t row = row0 + gid + 8 * (i >> 1);
                        if (row < n) dots_sc[row * nb + b] = tot;
                    }
                } else if (nt * 8 + 2 * tig + j < m) {
                    const double dw = (i < 2) ? dw0 : dw1;
                    acc[nt][i] = __dadd_rn(acc[nt][i], __dmul_rn(__dmul_rn(dw, (double)dy[nt][j]), (double)tot));
                }
            }
    }
    pdl_launch();
    if (!DOTS) write_out<NT, DOTS>(acc, red, warp, gid, tig, row0, n, m, y, ldy);
}

template <typename K, typename... Args>
static void launch_pdl(fb_ctx *ctx, K kernel, unsigned grid, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = ctx->pdl ? 1 : 0;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GEMV_WARPS * 32);
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    FB_CUDA(cudaLaunchKernelEx(&cfg, kernel, args...));
}

void launch_gemv(fb_ctx *ctx, const fb_qtensor *w, const Q8Act &a, int m, float *y, int64_t ldy) {
    FB_REQUIRE(m >= 1 && m <= 16, "gemv: m must be in 1..16");
    const unsigned grid = (unsigned)((w->n + 15) / 16);
    const int nb = (int)w->nb();
    if (w->dtype == FB_Q4_K) {
        if (m <= 8)
            launch_pdl(ctx, k_gemv_q4k<1, false>, grid, w->main(), w->n, nb, a, m, y, ldy, (int32_t *)nullptr,
                       (int32_t *)nullptr);
        else
            launch_pdl(ctx, k_gemv_q4k<2, false>, grid, w->main(), w->n, nb, a, m, y, ldy, (int32_t *)nullptr,
                       (int32_t *)nullptr);
    } else if (w->dtype == FB_Q6_K) {
        if (m <= 8)
            launch_pdl(ctx, k_gemv_q6k<1, false>, grid, w->main(), w->q6_d(), w->n, nb, a, m, y, ldy,
                       (int32_t *)nullptr);
        else
            launch_pdl(ctx, k_gemv_q6k<2, false>, grid, w->main(), w->q6_d(), w->n, nb, a, m, y, ldy,
                       (int32_t *)nullptr);
    } else {
        fail(FB_ERR_INVALID, "gemv: weight dtype must be Q4_K or Q6_K");
    }
}

void launch_block_dots(fb_ctx *ctx, const fb_qtensor *w, const Q8Act &a, int32_t *out_sc, int32_t *out_min) {
    const unsigned grid = (unsigned)((w->n + 15) / 16);
    const int nb = (int)w->nb();
    if (w->dtype == FB_Q4_K) {
        launch_pdl(ctx, k_gemv_q4k<1, true>, grid, w->main(), w->n, nb, a, 1, (float *)nullptr, (int64_t)0, out_sc,
                   out_min);
    } else if (w->dtype == FB_Q6_K) {
        FB_CUDA(cudaMemsetAsync(out_min, 0, (size_t)(w->n * nb) * 4, ctx->stream));
        launch_pdl(ctx, k_gemv_q6k<1, true>, grid, w->main(), w->q6_d(), w->n, nb, a, 1, (float *)nullptr, (int64_t)0,
                   out_sc);
    } else {
        fail(FB_ERR_INVALID, "block_dots: weight dtype must be Q4_K or Q6_K");
    }
}

}  // namespace fb
