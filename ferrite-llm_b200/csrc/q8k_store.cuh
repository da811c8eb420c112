// Q8_K quantization of values already in registers (shared by the fused
// decode-step kernels: norm, SwiGLU, the GEMV tails) and the binary64 block
// sum of the RMSNorm kernels.
#pragma once

#include "fb_internal.h"
#include "kq_common.cuh"

namespace fb {

// Q8_K quantization helpers shared with quant.cu are re-stated here for
// values already in registers (one warp per 256-value block, lane l owns
// values 8l..8l+7).
__device__ __forceinline__ void q8k_store_warp(const float (&v)[8], int lane, const Q8Act &a, int64_t row,
                                               int64_t blk) {
    float amax = 0.f, piv = 0.f;
    int idx = 1 << 30;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        float av = fabsf(v[e]);
        if (amax < av) {
            amax = av;
            piv = v[e];
            idx = 8 * lane + e;
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        float oa = __shfl_xor_sync(0xffffffffu, amax, off);
        float op = __shfl_xor_sync(0xffffffffu, piv, off);
        int oi = __shfl_xor_sync(0xffffffffu, idx, off);
        if (oa > amax || (oa == amax && oi < idx)) {
            amax = oa;
            piv = op;
            idx = oi;
        }
    }
    uint32_t w0 = 0, w1 = 0;
    int s = 0;
    float d = 0.f;
    if (amax != 0.f) {
        const float iscale = __fdiv_rn(-128.f, piv);
#pragma unroll
        for (int e = 0; e < 8; e++) {
            int q = (int)roundf(__fmul_rn(iscale, v[e]));
            q = q > 127 ? 127 : q;
            s += q;
            if (e < 4) w0 |= ((uint32_t)(uint8_t)q) << (8 * e);
            else w1 |= ((uint32_t)(uint8_t)q) << (8 * (e - 4));
        }
        d = __fdiv_rn(1.f, iscale);
    }
    const int s16 = s + __shfl_xor_sync(0xffffffffu, s, 1);
    const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 2);
    const int64_t k = a.k;
    *reinterpret_cast<uint2 *>(a.qs + row * k + blk * QK + 64 * (lane & 3) + 8 * (lane >> 2)) = make_uint2(w0, w1);
    if ((lane & 1) == 0) a.bs16[row * (k / 16) + blk * 16 + (lane >> 1)] = (int16_t)s16;
    if ((lane & 3) == 0) a.bs32[row * (k / 32) + blk * 8 + (lane >> 2)] = (int16_t)s32;
    if (lane == 0) a.d[row * (k / QK) + blk] = d;
}

// The same Q8_K quantization of one 256-value block by a CTA of 256 threads,
// one value per thread (index t = threadIdx.x in the block): the pivot (the
// value of largest magnitude, first index on ties), iscale = -128 / pivot,
// q = min(127, round(iscale * v)), the 16- and 32-value sums and
// d = 1 / iscale -- identical results to q8k_store_warp, without the
// per-lane loops over eight values.
__device__ __forceinline__ void q8k_store_block(float v, const Q8Act &a, int64_t row, int64_t blk, float *shv,
                                                int *shi) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float amax = fabsf(v), piv = v;
    int idx = t;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, off);
        const float op = __shfl_xor_sync(0xffffffffu, piv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
        if (oa > amax || (oa == amax && oi < idx)) {
            amax = oa;
            piv = op;
            idx = oi;
        }
    }
    if (lane == 0) {
        shv[2 * warp] = amax;
        shv[2 * warp + 1] = piv;
        shi[warp] = idx;
    }
    __syncthreads();
    amax = shv[0];
    piv = shv[1];
    idx = shi[0];
#pragma unroll
    for (int w = 1; w < QK / 32; w++) {
        const float oa = shv[2 * w];
        if (oa > amax || (oa == amax && shi[w] < idx)) {
            amax = oa;
            piv = shv[2 * w + 1];
            idx = shi[w];
        }
    }
    int q = 0;
    float iscale = 0.f;
    if (amax != 0.f) {
        iscale = __fdiv_rn(-128.f, piv);
        q = (int)roundf(__fmul_rn(iscale, v));
        q = q > 127 ? 127 : q;
    }
    // 16- and 32-value sums (the block's values 32w .. 32w + 31 are warp w's lanes)
    int s16 = q;
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, off);
    const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 16);
    const int64_t k = a.k;
    // permuted byte position: value 8l + e -> 64 (l & 3) + 8 (l >> 2) + e; four
    // consecutive values form one 32-bit word
    const uint32_t b0 = (uint32_t)(uint8_t)q;
    const uint32_t b1 = __shfl_down_sync(0xffffffffu, b0, 1), b2 = __shfl_down_sync(0xffffffffu, b0, 2),
                   b3 = __shfl_down_sync(0xffffffffu, b0, 3);
    if ((t & 3) == 0) {
        const int l = t >> 3, e = t & 7;
        *reinterpret_cast<uint32_t *>(a.qs + row * k + blk * QK + 64 * (l & 3) + 8 * (l >> 2) + e) =
            b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
    }
    if ((t & 15) == 0) a.bs16[row * (k / 16) + blk * 16 + (t >> 4)] = (int16_t)s16;
    if (lane == 0) a.bs32[row * (k / 32) + blk * 8 + warp] = (int16_t)s32;
    if (t == 0) a.d[row * (k / QK) + blk] = amax != 0.f ? __fdiv_rn(1.f, iscale) : 0.f;
}

// Block sum in binary64 (RMSNorm sums of squares: each f32 square is exact
// in binary64, so the result is independent of the summation order up to
// binary64 rounding, and rounds to the same f32 as the oracle's).
template <int NW>
__device__ __forceinline__ double block_sum64(double v, double *sh) {
    v = warp_sum64(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < NW; w++) t = __dadd_rn(t, sh[w]);
    return t;
}

}  // namespace fb
