// Decode GEMV for GGUF Q4_K / Q6_K weights against Q8_K activations
// (batch m = 1..16): y[m, n] = x[m, k] . W[n, k]^T.
//
// Arithmetic = candle-core 0.8.4 CPU QMatMul (crates/ferrite-wasm-host/src/
// adapter.rs:61-70 -> QMatMul::forward): activations quantized to Q8_K, then
// per super-block the integer sums  sum_j sc_j * (q_w . q_x)_j  (and for Q4_K
// sum_j m_j * bsum_j) combined with the fp16 super-block scales.  The
// reference's GPU kernels for the same op are the dp4a MMVQ kernels
// mul_mat_vec_q{4,6}_K_q8_1 (ptx-kernels/kernels/candle/quantized.cu:2627-3344).
//
// B200 design: the op is HBM-bound (0.5625 / 0.8203 weight bytes per MAC at
// m = 1), so the kernel's job is to keep enough weight bytes in flight.
//  * Persistent CTAs of KS warps loop over 16-row tiles; warp w owns a fixed
//    slice of the super-blocks of every tile.  Each warp streams its (tile,
//    super-block) records -- one contiguous record per 16 rows in the
//    tile-major device layout -- through its own DEPTH-stage shared-memory
//    ring with cp.async.bulk (TMA, no multicast) and per-stage mbarriers;
//    lane 0 refills a stage as soon as the warp has consumed it, so each SM
//    keeps ~150 KB of weights in flight without spending registers on them.
//  * The first DEPTH stages are issued before griddepcontrol.wait: weights do
//    not depend on the previous kernel, so they stream in while it finishes.
//  * The integer dot of each 32-value sub-block runs on the tensor pipe as
//    mma.m16n8k32.s8 (16 weight rows x 8 activation rows per instruction,
//    exact int32); per-sub-block scales are applied in int32 exactly as the
//    CPU path does, and the per-super-block combine runs in binary64 with one
//    rounding to f32 (bit-identical to the CPU oracle whatever the order).
//  * Q6_K: each 32-value part spans two 16-value scale groups; lanes with
//    tig < 2 hold the first group's values and tig >= 2 the second's, so two
//    MMAs with the B fragment masked by lane group separate them.
// Thread (gid = lane/4, tig = lane%4) owns weight rows gid and gid+8 of the
// tile and output columns 2*tig, 2*tig+1 of each 8-wide n-tile; the KS warps'
// partial sums of a tile are reduced through shared memory in fixed order.
// mbarrier waits are bounded; on timeout the kernel raises
// ERRBIT_WAIT_TIMEOUT, drains its outstanding copies (bounded) and exits.
#include "fb_internal.h"
#include "gemv_dp4a.cuh"
#include "kq_common.cuh"

#include <algorithm>
#include <map>
#include <mutex>

namespace fb {


template <int DT> struct QRec;
template <> struct QRec<4> { static constexpr int bytes = Q4K_REC; };
template <> struct QRec<6> { static constexpr int bytes = Q6K_REC; };

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
                const uint4 v = ld_act16(p + 16 * i);
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

// ---------------------------------------------------------- Q4_K block ---
// One (tile, super-block) record in shared memory; accumulates the rows
// gid / gid+8 x columns (2tig, 2tig+1) of every n-tile into acc (binary64),
// or (DOTS) writes the integer partials of column 0.
template <int NT, bool DOTS>
__device__ __forceinline__ void q4k_block(const uint8_t *rec, const Q8Act &a, int m, int b, int nb, int gid, int tig,
                                          int64_t row0, int64_t n, double (&acc)[NT][4], int32_t *dots_sc,
                                          int32_t *dots_min) {
    const uint8_t *r0 = rec + gid * 144, *r1 = rec + (gid + 8) * 144;
    const uint4 h0 = *reinterpret_cast<const uint4 *>(r0), h1 = *reinterpret_cast<const uint4 *>(r1);
    const uint4 q0a = *reinterpret_cast<const uint4 *>(r0 + 16 + 32 * tig);
    const uint4 q0b = *reinterpret_cast<const uint4 *>(r0 + 32 + 32 * tig);
    const uint4 q1a = *reinterpret_cast<const uint4 *>(r1 + 16 + 32 * tig);
    const uint4 q1b = *reinterpret_cast<const uint4 *>(r1 + 32 + 32 * tig);
    ActBlock<NT> ab;
    load_act<NT>(a, m, b, gid, tig, ab);
    uint4 bs[NT][2];
    float dy[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const int col = nt * 8 + 2 * tig + j;
            const bool v = col < m;
            bs[nt][j] = v ? ld_act16(a.bs32 + (int64_t)col * (a.k / 32) + (int64_t)b * 8) : make_uint4(0, 0, 0, 0);
            dy[nt][j] = v ? a.d[(int64_t)col * nb + b] : 0.f;
        }
    const Q4Scales s0 = q4k_unpack_scales(h0.y, h0.z, h0.w);
    const Q4Scales s1 = q4k_unpack_scales(h1.y, h1.z, h1.w);
    const uint32_t W0[8] = {q0a.x, q0a.y, q0a.z, q0a.w, q0b.x, q0b.y, q0b.z, q0b.w};
    const uint32_t W1[8] = {q1a.x, q1a.y, q1a.z, q1a.w, q1b.x, q1b.y, q1b.z, q1b.w};
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
    const double dw0 = h2f(h0.x & 0xFFFF), dm0 = h2f(h0.x >> 16);
    const double dw1 = h2f(h1.x & 0xFFFF), dm1 = h2f(h1.x >> 16);
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int j = i & 1;
            if (nt * 8 + 2 * tig + j >= m) continue;
            const Q4Scales &sr = (i < 2) ? s0 : s1;
            const uint4 q = bs[nt][j];
            int msum = __dp2a_lo((int)q.x, (int)sr.mn_lo, 0);
            msum = __dp2a_hi((int)q.y, (int)sr.mn_lo, msum);
            msum = __dp2a_lo((int)q.z, (int)sr.mn_hi, msum);
            msum = __dp2a_hi((int)q.w, (int)sr.mn_hi, msum);
            if (DOTS) {
                const int64_t row = row0 + gid + 8 * (i >> 1);
                if (nt == 0 && j == 0 && row < n) {
                    dots_sc[row * nb + b] = isum[nt][i];
                    dots_min[row * nb + b] = msum;
                }
            } else {
                // binary64 combine: ((d * dy) * isum) - ((dmin * dy) * msum)
                const double dw = (i < 2) ? dw0 : dw1, dm = (i < 2) ? dm0 : dm1;
                const double yd = dy[nt][j];
                acc[nt][i] = __dadd_rn(acc[nt][i], __dmul_rn(__dmul_rn(dw, yd), (double)isum[nt][i]));
                acc[nt][i] = __dsub_rn(acc[nt][i], __dmul_rn(__dmul_rn(dm, yd), (double)msum));
            }
        }
}

// ---------------------------------------------------------- Q6_K block ---
template <int NT, bool DOTS>
__device__ __forceinline__ void q6k_block(const uint8_t *rec, const Q8Act &a, int m, int b, int nb, int gid, int tig,
                                          int64_t row0, int64_t n, double (&acc)[NT][4], int32_t *dots_sc) {
    const uint32_t mlo = tig < 2 ? 0xFFFFFFFFu : 0u;
    const uint8_t *r0 = rec + gid * 208, *r1 = rec + (gid + 8) * 208;
    uint32_t Q0[12], Q1[12];
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const uint4 v0 = *reinterpret_cast<const uint4 *>(r0 + 48 * tig + 16 * i);
        const uint4 v1 = *reinterpret_cast<const uint4 *>(r1 + 48 * tig + 16 * i);
        Q0[4 * i] = v0.x, Q0[4 * i + 1] = v0.y, Q0[4 * i + 2] = v0.z, Q0[4 * i + 3] = v0.w;
        Q1[4 * i] = v1.x, Q1[4 * i + 1] = v1.y, Q1[4 * i + 2] = v1.z, Q1[4 * i + 3] = v1.w;
    }
    const uint4 sc0v = *reinterpret_cast<const uint4 *>(r0 + 192);
    const uint4 sc1v = *reinterpret_cast<const uint4 *>(r1 + 192);
    const uint32_t S0[4] = {sc0v.x, sc0v.y, sc0v.z, sc0v.w};
    const uint32_t S1[4] = {sc1v.x, sc1v.y, sc1v.z, sc1v.w};
    const double dw0 = h2f(*reinterpret_cast<const uint16_t *>(rec + 3328 + 2 * gid));
    const double dw1 = h2f(*reinterpret_cast<const uint16_t *>(rec + 3328 + 2 * (gid + 8)));
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
                const int16_t *p = a.bs16 + (int64_t)col * (a.k / 16) + (int64_t)b * 16;
                bsa[nt][j] = ld_act16(p);
                bsb[nt][j] = ld_act16(p + 8);
                dy[nt][j] = a.d[(int64_t)col * nb + b];
            } else {
                bsa[nt][j] = make_uint4(0, 0, 0, 0);
                bsb[nt][j] = make_uint4(0, 0, 0, 0);
                dy[nt][j] = 0.f;
            }
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
            if (nt * 8 + 2 * tig + j >= m) continue;
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
                const int64_t row = row0 + gid + 8 * (i >> 1);
                if (nt == 0 && j == 0 && row < n) dots_sc[row * nb + b] = tot;
            } else {
                const double dw = (i < 2) ? dw0 : dw1;
                acc[nt][i] = __dadd_rn(acc[nt][i], __dmul_rn(__dmul_rn(dw, (double)dy[nt][j]), (double)tot));
            }
        }
}

// ----------------------------------------------------------- pipeline ---
// Bytes of the shared-memory copy of M activation rows of length k (dp4a
// path): qs [M][k] | d [M][k/256] f32 | bs16 [M][k/16] | bs32 [M][k/32].
__host__ __device__ inline size_t r16(size_t x) { return (x + 15) & ~(size_t)15; }
__host__ __device__ inline size_t act_smem_bytes(int M, int64_t k) {
    return r16((size_t)M * k) + r16((size_t)M * (k / 256) * 4) + r16((size_t)M * (k / 16) * 2) +
           r16((size_t)M * (k / 32) * 2);
}

// NT > 0: MMA consumer with NT 8-wide n-tiles (m <= 8*NT); NT < 0: dp4a
// consumer for exactly M = -NT activation rows, whose Q8_K rows are first
// copied to shared memory.  KS warps per CTA, `depth` ring stages per warp.
template <int DT, int NT, bool DOTS, int KS>
__global__ void __launch_bounds__(KS * 32) k_gemv(const uint8_t *__restrict__ W, int64_t n, int nb, int n_tiles,
                                                  Q8Act a, int m, float *__restrict__ y, int64_t ldy,
                                                  int32_t *__restrict__ dots_sc, int32_t *__restrict__ dots_min,
                                                  uint32_t *err, int depth, const __grid_constant__ PeerOut po) {
    constexpr int REC = QRec<DT>::bytes;
    const int DEPTH = depth;
    constexpr bool DP4A = NT < 0;
    constexpr int M = DP4A ? -NT : 1;
    constexpr int C = DP4A ? M : 8 * NT;
    constexpr int NTA = DP4A ? 1 : NT;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bars[KS * 8];
    __shared__ uint64_t actbar;
    __shared__ double red[KS * 16 * (C + 1)];
    __shared__ int s_abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const int bpw = (nb + KS - 1) / KS;
    const int bbeg = min(nb, warp * bpw), nmine = min(nb, bbeg + bpw) - bbeg;
    const int ntl = (int)blockIdx.x < n_tiles ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int total = ntl * nmine;  // records this warp streams
    const size_t act_bytes = DP4A ? (act_smem_bytes(M, a.k) + 127) & ~(size_t)127 : 0;
    uint8_t *ring = smem + act_bytes + (size_t)warp * DEPTH * REC;
    uint64_t *wbar = bars + warp * 8;
    if (lane == 0) {
        for (int i = 0; i < DEPTH; i++) mbar_init(&wbar[i], 1);
        mbar_fence_init();
    }
    if (threadIdx.x == 0) {
        s_abort = 0;
        if (DP4A) {
            mbar_init(&actbar, 1);
            mbar_fence_init();
        }
    }
    __syncthreads();
    // producer (lane 0): records issued, and the next record's stage and
    // global address, advanced incrementally (record c = tile c / nmine,
    // super-block bbeg + c % nmine of that tile, stage c % DEPTH; a runtime
    // division per record measurably slows the decode step)
    int issued = 0, p_slot = 0, p_bl = 0;
    const uint8_t *p_src = W + ((size_t)blockIdx.x * nb + bbeg) * REC;
    const size_t tile_step = ((size_t)gridDim.x * nb - (size_t)nmine) * REC;  // last record of a tile -> first of the next
    const uint64_t wpol = l2_evict_first_policy();  // weights are read once per step
    auto issue = [&]() {
        mbar_expect_tx(&wbar[p_slot], REC);
        bulk_g2s_stream(ring + (size_t)p_slot * REC, p_src, REC, &wbar[p_slot], wpol);
        issued++;
        if (++p_slot == DEPTH) p_slot = 0;
        p_src += REC;
        if (++p_bl == nmine) {
            p_bl = 0;
            p_src += tile_step;
        }
    };
    // weights do not depend on the previous kernel: start streaming them now
    if (lane == 0)
        while (issued < DEPTH && issued < total) issue();
    pdl_wait();
    pdl_launch();  // let the next kernel start streaming its weights
    // row-parallel shard: the sequence number tagging this exchange's words
    const uint32_t seq = po.world ? (*po.epoch - 1u) * (uint32_t)po.nx + (uint32_t)po.xi + 1u : 0u;
    Q8Act act = a;
    bool ok = true;
    if constexpr (DP4A) {
        // the activation rows are read by every record: four bulk copies
        // (one round trip) bring them into shared memory.  Regions are
        // rounded up to 16 bytes; the global arrays are padded to 256 bytes
        // (q8act_view), so the rounded copies stay inside them.
        const int64_t k = a.k;
        const size_t bq = r16((size_t)M * k), bd = r16((size_t)M * (k / 256) * 4), b16 = r16((size_t)M * (k / 16) * 2),
                     b32 = r16((size_t)M * (k / 32) * 2);
        uint8_t *sq = smem;
        float *sd = reinterpret_cast<float *>(smem + bq);
        int16_t *s16 = reinterpret_cast<int16_t *>(smem + bq + bd);
        int16_t *s32 = reinterpret_cast<int16_t *>(smem + bq + bd + b16);
        if (threadIdx.x == 0) {
            mbar_expect_tx(&actbar, (uint32_t)(bq + bd + b16 + b32));
            bulk_g2s(sq, a.qs, (uint32_t)bq, &actbar);
            bulk_g2s(sd, a.d, (uint32_t)bd, &actbar);
            bulk_g2s(s16, a.bs16, (uint32_t)b16, &actbar);
            bulk_g2s(s32, a.bs32, (uint32_t)b32, &actbar);
        }
        ok = mbar_wait_bounded(&actbar, 0);
        act = Q8Act{reinterpret_cast<int8_t *>(sq), sd, s16, s32, k};
    }
    const bool act_ok = ok;
    int c = 0, waited = 0;  // records visited / records whose copy has landed
    int slot = 0;           // c % DEPTH
    uint32_t par = 0;       // (c / DEPTH) & 1
    for (int ti = 0; ti < ntl; ti++) {
        const int64_t row0 = ((int64_t)blockIdx.x + (int64_t)ti * gridDim.x) * 16;
        double acc[NTA][4];
        double accd[M];
#pragma unroll
        for (int nt = 0; nt < NTA; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) acc[nt][i] = 0.0;
#pragma unroll
        for (int c2 = 0; c2 < M; c2++) accd[c2] = 0.0;
        for (int bl = 0; bl < nmine; bl++, c++) {
            if (ok) {
                ok = mbar_wait_bounded(&wbar[slot], par);
                if (ok) waited = c + 1;
            }
            if (ok) {
                const uint8_t *rec = ring + (size_t)slot * REC;
                if constexpr (DP4A) {
                    if constexpr (DT == 4)
                        q4k_block_dp4a<M, DOTS>(rec, act, bbeg + bl, nb, lane, row0, n, accd, dots_sc, dots_min);
                    else
                        q6k_block_dp4a<M, DOTS>(rec, act, bbeg + bl, nb, lane, row0, n, accd, dots_sc);
                } else {
                    if constexpr (DT == 4)
                        q4k_block<NTA, DOTS>(rec, a, m, bbeg + bl, nb, gid, tig, row0, n, acc, dots_sc, dots_min);
                    else
                        q6k_block<NTA, DOTS>(rec, a, m, bbeg + bl, nb, gid, tig, row0, n, acc, dots_sc);
                }
            }
            __syncwarp();
            if (lane == 0 && ok && issued < total) {
                fence_proxy_async_smem();  // our reads of this stage precede the refill
                issue();
            }
            if (++slot == DEPTH) {
                slot = 0;
                par ^= 1u;
            }
        }
        if (!ok && lane == 0) {
            s_abort = 1;
            atomicOr(err, ERRBIT_WAIT_TIMEOUT);
        }
        if (!DOTS) {
            if constexpr (DP4A) {
                if (lane < 16)
#pragma unroll
                    for (int c2 = 0; c2 < M; c2++) red[(warp * 16 + lane) * (C + 1) + c2] = accd[c2];
            } else {
#pragma unroll
                for (int nt = 0; nt < NTA; nt++)
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int r = gid + 8 * (i >> 1), col = nt * 8 + 2 * tig + (i & 1);
                        red[(warp * 16 + r) * (C + 1) + col] = acc[nt][i];
                    }
            }
        }
        __syncthreads();
        if (!DOTS && !s_abort) {
            for (int o = threadIdx.x; o < 16 * C; o += blockDim.x) {
                const int r = o / C, col = o % C;
                double sum = 0.0;
#pragma unroll
                for (int w = 0; w < KS; w++) sum = __dadd_rn(sum, red[(w * 16 + r) * (C + 1) + col]);
                const int64_t row = row0 + r;
                if (row < n && col < m) {
                    if (po.world) {  // row-parallel shard: binary64 partials to every rank's inbox
                        const uint64_t bits = (uint64_t)__double_as_longlong(sum);
                        const uint64_t w0 = ((uint64_t)seq << 32) | (bits & 0xffffffffull);
                        const uint64_t w1 = ((uint64_t)seq << 32) | (bits >> 32);
                        const int64_t wi = 2 * ((int64_t)col * po.ld + row);
                        for (int p = 0; p < po.world; p++) {
                            st_relaxed_sys_u64(po.dst[p] + wi, w0);
                            st_relaxed_sys_u64(po.dst[p] + wi + 1, w1);
                        }
                    } else {
                        y[(int64_t)col * ldy + row] = __double2float_rn(sum);
                    }
                }
            }
        }
        __syncthreads();
        if (s_abort) break;
    }
    if (!ok && lane == 0) {
        // let the copies still in flight land before shared memory is released
        for (int k = waited; k < issued; k++) mbar_wait_bounded(&wbar[k % DEPTH], (uint32_t)(k / DEPTH) & 1u);
        if (DP4A && !act_ok && threadIdx.x == 0) mbar_wait_bounded(&actbar, 0);
    }
    pdl_launch();
}

template <int DT, int NT, bool DOTS, int KS>
static void launch_gemv_k(fb_ctx *ctx, const fb_qtensor *w, const Q8Act &a, int m, float *y, int64_t ldy,
                          int32_t *dsc, int32_t *dmn, const PeerOut &po) {
    constexpr int REC = QRec<DT>::bytes;
    constexpr int M = NT < 0 ? -NT : 0;
    const size_t act = M ? (act_smem_bytes(M, w->k) + 127) & ~(size_t)127 : 0;
    // ring depth: as deep as fits next to the staged activations in 40 KB
    // (4-warp CTAs: three stages of Q4_K or Q6_K records) or 112 KB (8-warp
    // CTAs), 3..8 stages per warp.  In the decode step, deeper 4-warp rings
    // (56 KB: five stages, 72 KB) and shallower 8-warp ones measured slower.
    const size_t budget = (size_t)(KS == 4 ? 40 : 112) * 1024;
    int depth = (int)std::min<size_t>(8, (budget - std::min(act, budget / 2)) / ((size_t)KS * REC));
    depth = std::max(depth, 3);
    const size_t smem = act + (size_t)KS * depth * REC;
    auto kernel = k_gemv<DT, NT, DOTS, KS>;
    // the shared-memory attribute and the occupancy query cost more host time
    // than a small GEMV's device time: the attribute only ever grows (to the
    // largest size this kernel has been launched with on the device) and the
    // occupancy is cached per (device, size)
    static std::mutex mu;
    static std::map<std::pair<int, size_t>, int> occ_cache;
    static std::map<int, size_t> smem_max;
    int occ = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = occ_cache.find({ctx->device, smem});
        if (it != occ_cache.end()) {
            occ = it->second;
        } else {
            size_t &mx = smem_max[ctx->device];
            if (smem > mx) {
                FB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
                mx = smem;
            }
            FB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, KS * 32, smem));
            occ_cache[{ctx->device, smem}] = occ;
        }
    }
    FB_REQUIRE(occ > 0, "gemv: configuration does not fit on an SM");
    const int n_tiles = (int)w->n_tiles();
    const int grid = std::min(n_tiles, occ * ctx->num_sms);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = ctx->pdl ? 1 : 0;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(KS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    FB_CUDA(cudaLaunchKernelEx(&cfg, kernel, w->main(), w->n, (int)w->nb(), n_tiles, a, m, y, ldy, dsc, dmn,
                               ctx->err_word, depth, po));
}

// Few tiles (fewer than two per SM; for the dp4a consumer, m <= 4, fewer
// than three): 8-warp CTAs so each SM still runs enough warps; otherwise
// 4-warp CTAs.  (Measured in the decode step: the b = 1 qkv projection, 384
// tiles, is faster with 8-warp CTAs, the b = 16 one with 4-warp CTAs.)
template <int DT, int NT, bool DOTS>
static void launch_gemv_t(fb_ctx *ctx, const fb_qtensor *w, const Q8Act &a, int m, float *y, int64_t ldy,
                          int32_t *dsc, int32_t *dmn, const PeerOut &po) {
    if (w->n_tiles() < (NT < 0 ? 3 : 2) * ctx->num_sms && w->nb() >= 16)
        launch_gemv_k<DT, NT, DOTS, 8>(ctx, w, a, m, y, ldy, dsc, dmn, po);
    else
        launch_gemv_k<DT, NT, DOTS, 4>(ctx, w, a, m, y, ldy, dsc, dmn, po);
}

template <int DT>
static void launch_gemv_dt(fb_ctx *ctx, const fb_qtensor *w, const Q8Act &a, int m, float *y, int64_t ldy,
                           const PeerOut &po) {
    switch (m) {
    case 1: launch_gemv_t<DT, -1, false>(ctx, w, a, m, y, ldy, nullptr, nullptr, po); break;
    case 2: launch_gemv_t<DT, -2, false>(ctx, w, a, m, y, ldy, nullptr, nullptr, po); break;
    case 3: launch_gemv_t<DT, -3, false>(ctx, w, a, m, y, ldy, nullptr, nullptr, po); break;
    case 4: launch_gemv_t<DT, -4, false>(ctx, w, a, m, y, ldy, nullptr, nullptr, po); break;
    default:
        if (m <= 8) launch_gemv_t<DT, 1, false>(ctx, w, a, m, y, ldy, nullptr, nullptr, po);
        else if (m <= 16) launch_gemv_t<DT, 2, false>(ctx, w, a, m, y, ldy, nullptr, nullptr, po);
        else launch_gemv_t<DT, 4, false>(ctx, w, a, m, y, ldy, nullptr, nullptr, po);
    }
}

static void gemv_any(fb_ctx *ctx, const fb_qtensor *w, const Q8Act &a, int m, float *y, int64_t ldy,
                     const PeerOut &po) {
    FB_REQUIRE(m >= 1 && m <= 32, "gemv: m must be in 1..32");
    if (w->dtype == FB_Q4_K) launch_gemv_dt<4>(ctx, w, a, m, y, ldy, po);
    else if (w->dtype == FB_Q6_K) launch_gemv_dt<6>(ctx, w, a, m, y, ldy, po);
    else fail(FB_ERR_INVALID, "gemv: weight dtype must be Q4_K or Q6_K");
}

void launch_gemv(fb_ctx *ctx, const fb_qtensor *w, const Q8Act &a, int m, float *y, int64_t ldy) {
    gemv_any(ctx, w, a, m, y, ldy, PeerOut{});
}

void launch_gemv_peer(fb_ctx *ctx, const fb_qtensor *w, const Q8Act &a, int m, const PeerOut &po) {
    FB_REQUIRE(po.world >= 1 && po.world <= FB_TP_MAX, "gemv: bad peer count");
    gemv_any(ctx, w, a, m, nullptr, 0, po);
}

void launch_block_dots(fb_ctx *ctx, const fb_qtensor *w, const Q8Act &a, int32_t *out_sc, int32_t *out_min) {
    if (w->dtype == FB_Q4_K) {
        launch_gemv_t<4, -1, true>(ctx, w, a, 1, nullptr, 0, out_sc, out_min, PeerOut{});
    } else if (w->dtype == FB_Q6_K) {
        FB_CUDA(cudaMemsetAsync(out_min, 0, (size_t)(w->n * w->nb()) * 4, ctx->stream));
        launch_gemv_t<6, -1, true>(ctx, w, a, 1, nullptr, 0, out_sc, nullptr, PeerOut{});
    } else {
        fail(FB_ERR_INVALID, "block_dots: weight dtype must be Q4_K or Q6_K");
    }
}

}  // namespace fb
