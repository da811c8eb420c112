// Q4_K / Q6_K x Q8_K integer block consumers of the decode GEMV for a few
// activation rows (dp4a on CUDA cores), shared by the standalone GEMV kernel
// (gemv.cu) and the persistent decode-step kernel (decode_step.cu).
#pragma once

#include "fb_internal.h"
#include "kq_common.cuh"

namespace fb {

// ------------------------------------------------ dp4a consumers (m <= 4) ---
// For a handful of activation rows the 16x8 MMA tile is mostly padding, so
// small batches use CUDA-core dp4a instead: lane (r = lane & 15, h = lane >> 4)
// takes row r of the record and half h of the super-block (four 32-value
// sub-blocks), which keeps every lane busy and the shared-memory reads
// bank-conflict-free.  Both halves' integer partials are added with one
// shuffle before the binary64 combine.
__device__ __forceinline__ int dp4(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }
// Unsigned bytes of a times signed bytes of b: with a = w & 0xF0F0F0F0 the
// high nibbles enter as 16 * q without a shift; the sum is then an exact
// multiple of 16 and one arithmetic shift recovers the nibble dot.
__device__ __forceinline__ int dp4us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

template <int M, bool DOTS>
__device__ __forceinline__ void q4k_block_dp4a(const uint8_t *rec, const Q8Act &a, int b, int nb, int lane,
                                               int64_t row0, int64_t n, double (&acc)[M], int32_t *dots_sc,
                                               int32_t *dots_min) {
    const int r = lane & 15, h = lane >> 4;
    const uint8_t *rp = rec + r * 144;
    const uint4 hd = *reinterpret_cast<const uint4 *>(rp);
    uint4 wq[4];
#pragma unroll
    for (int t = 0; t < 4; t++) wq[t] = *reinterpret_cast<const uint4 *>(rp + 16 + 32 * t + 16 * h);
    const Q4Scales sc = q4k_unpack_scales(hd.y, hd.z, hd.w);
    // this half's sub-blocks 4h..4h+3: scales / mins are bytes of the lo or hi word
    const uint32_t scw = h ? sc.sc_hi : sc.sc_lo, mnw = h ? sc.mn_hi : sc.mn_lo;
    const double dw = h2f(hd.x & 0xFFFF), dm = h2f(hd.x >> 16);
#pragma unroll
    for (int c = 0; c < M; c++) {
        const int8_t *qa = a.qs + (int64_t)c * a.k + (int64_t)b * QK + 32 * h;
        int dot[4] = {0, 0, 0, 0};
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint4 a0 = *reinterpret_cast<const uint4 *>(qa + 64 * t);
            const uint4 a1 = *reinterpret_cast<const uint4 *>(qa + 64 * t + 16);
            const uint4 w = wq[t];
            dot[0] = dp4(w.x & 0x0F0F0F0Fu, a0.x, dot[0]);
            dot[0] = dp4(w.y & 0x0F0F0F0Fu, a0.y, dot[0]);
            dot[1] = dp4us(w.x & 0xF0F0F0F0u, a0.z, dot[1]);  // 16 x (high-nibble dot)
            dot[1] = dp4us(w.y & 0xF0F0F0F0u, a0.w, dot[1]);
            dot[2] = dp4(w.z & 0x0F0F0F0Fu, a1.x, dot[2]);
            dot[2] = dp4(w.w & 0x0F0F0F0Fu, a1.y, dot[2]);
            dot[3] = dp4us(w.z & 0xF0F0F0F0u, a1.z, dot[3]);
            dot[3] = dp4us(w.w & 0xF0F0F0F0u, a1.w, dot[3]);
        }
        // |16 x dot| <= 4 * 8 * 240 * 128 < 2^31: exact, a multiple of 16
        dot[1] >>= 4;
        dot[3] >>= 4;
        int isum = byte_of(scw, 0) * dot[0] + byte_of(scw, 1) * dot[1] + byte_of(scw, 2) * dot[2] +
                   byte_of(scw, 3) * dot[3];
        // mins: bs32 of sub-blocks 4h..4h+3 (two int16 pairs)
        const int32_t *bsp = reinterpret_cast<const int32_t *>(a.bs32 + (int64_t)c * (a.k / 32) + (int64_t)b * 8 + 4 * h);
        int msum = __dp2a_lo(bsp[0], (int)mnw, 0);
        msum = __dp2a_hi(bsp[1], (int)mnw, msum);
        isum += __shfl_xor_sync(0xffffffffu, isum, 16);
        msum += __shfl_xor_sync(0xffffffffu, msum, 16);
        if (h == 0) {
            if (DOTS) {
                const int64_t row = row0 + r;
                if (c == 0 && row < n) {
                    dots_sc[row * nb + b] = isum;
                    dots_min[row * nb + b] = msum;
                }
            } else {
                const double yd = a.d[(int64_t)c * nb + b];
                acc[c] = __dadd_rn(acc[c], __dmul_rn(__dmul_rn(dw, yd), (double)isum));
                acc[c] = __dsub_rn(acc[c], __dmul_rn(__dmul_rn(dm, yd), (double)msum));
            }
        }
    }
}

template <int M, bool DOTS>
__device__ __forceinline__ void q6k_block_dp4a(const uint8_t *rec, const Q8Act &a, int b, int nb, int lane,
                                               int64_t row0, int64_t n, double (&acc)[M], int32_t *dots_sc) {
    const int r = lane & 15, h = lane >> 4;
    const uint8_t *rp = rec + r * 208;
    uint4 ql[4];
    uint2 qh[4];
#pragma unroll
    for (int t = 0; t < 4; t++) {
        ql[t] = *reinterpret_cast<const uint4 *>(rp + 48 * t + 16 * h);
        qh[t] = *reinterpret_cast<const uint2 *>(rp + 48 * t + 32 + 8 * h);
    }
    const uint2 scv = *reinterpret_cast<const uint2 *>(rp + 192 + 8 * h);  // scales of groups 8h..8h+7
    const double dw = h2f(*reinterpret_cast<const uint16_t *>(rec + 3328 + 2 * r));
#pragma unroll
    for (int c = 0; c < M; c++) {
        const int8_t *qa = a.qs + (int64_t)c * a.k + (int64_t)b * QK + 32 * h;
        int dg[4][2] = {{0, 0}, {0, 0}, {0, 0}, {0, 0}};  // [part p][t >> 1]: group 8h + 2p + (t >> 1)
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const uint4 a0 = *reinterpret_cast<const uint4 *>(qa + 64 * t);
            const uint4 a1 = *reinterpret_cast<const uint4 *>(qa + 64 * t + 16);
            const uint32_t av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const uint32_t qlw[4] = {ql[t].x, ql[t].y, ql[t].z, ql[t].w};  // index 2j + x
            const uint32_t qhw[2] = {qh[t].x, qh[t].y};                        // index x
#pragma unroll
            for (int p = 0; p < 4; p++)
#pragma unroll
                for (int x = 0; x < 2; x++) {
                    const uint32_t lo = (qlw[2 * (p & 1) + x] >> (4 * (p >> 1))) & 0x0F0F0F0Fu;
                    const uint32_t hi = (2 * p <= 4) ? ((qhw[x] << (4 - 2 * p)) & 0x30303030u)
                                                     : ((qhw[x] >> (2 * p - 4)) & 0x30303030u);
                    dg[p][t >> 1] = dp4(lo | hi, av[2 * p + x], dg[p][t >> 1]);
                }
        }
        int isum = 0;
#pragma unroll
        for (int p = 0; p < 4; p++)
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int G = 2 * p + u;  // group within this half
                isum += sbyte_of(G < 4 ? scv.x : scv.y, G & 3) * dg[p][u];
            }
        // -32 offset of the 6-bit quants: sum_G sc_G * bsum16_G over the half's 8 groups
        const int32_t *bsp = reinterpret_cast<const int32_t *>(a.bs16 + (int64_t)c * (a.k / 16) + (int64_t)b * 16 + 8 * h);
        int cs = __dp2a_lo(bsp[0], (int)scv.x, 0);
        cs = __dp2a_hi(bsp[1], (int)scv.x, cs);
        cs = __dp2a_lo(bsp[2], (int)scv.y, cs);
        cs = __dp2a_hi(bsp[3], (int)scv.y, cs);
        int tot = isum - 32 * cs;
        tot += __shfl_xor_sync(0xffffffffu, tot, 16);
        if (h == 0) {
            if (DOTS) {
                const int64_t row = row0 + r;
                if (c == 0 && row < n) dots_sc[row * nb + b] = tot;
            } else {
                const double yd = a.d[(int64_t)c * nb + b];
                acc[c] = __dadd_rn(acc[c], __dmul_rn(__dmul_rn(dw, yd), (double)tot));
            }
        }
    }
}

}  // namespace fb
