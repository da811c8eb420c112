// The softmax partial of one 16-token unit of decode attention and its fold
// into a warp's running state, shared by the decode attention kernel
// (attention.cu) and the persistent decode step (decode_step.cu).
//
// Numerics (restated by the CPU oracle, oracle/model.c): for the unit's
// tokens t (positions 16u .. 16u + nt - 1) and each of the G query heads,
//   m_u = max s_t,  p_t = f32(exp64(s_t - m_u)),
//   l_u = pairwise sum of the 16 slots (absent tokens count 0),
//   o_u = FMA chain of p_t v_t in token order (f32),
// then, in binary64, the running (m, l, o) and (m_u, l_u, o_u) are added
// with the side of the smaller max weighted by exp64 of the difference.  The
// unit partials do not depend on how units are spread over warps and CTAs.
#pragma once

#include <cuda_fp16.h>

#include "kq_common.cuh"

namespace fb {

// ssw: the unit's scores [16][G] (f32, shared memory, slots >= nt unused);
// pbw: [16][G] f32 scratch of this warp; vrow: V of the unit's first token
// at this lane's dims [4 lane, 4 lane + 4) (token stride 128 values);
// mx: the unit's max per head (warp-uniform, finite: nt >= 1).
template <int G>
__device__ __forceinline__ void att_unit_fold(const float *ssw, float *pbw, const __half *vrow, int nt,
                                              const float (&mx)[G], int lane, float (&m_run)[G], double (&Lw)[G],
                                              double (&o)[G][4]) {
    constexpr unsigned FULL = 0xffffffffu;
    constexpr int GH = G >= 2 ? G / 2 : 1;
    // p and the pairwise l_u: lane (t = lane & 15) takes the heads of parity
    // lane >> 4; the xor shuffles stay inside each half of the warp
    float lu[G];
    {
        const int t = lane & 15, hp = lane >> 4;
        float ls[GH];
#pragma unroll
        for (int k = 0; k < GH; k++) {
            const int g = G >= 2 ? 2 * k + hp : 0;
            const float mg = G >= 2 ? (hp ? mx[G >= 2 ? 2 * k + 1 : 0] : mx[2 * k]) : mx[0];
            float p = 0.f;
            if ((G >= 2 || hp == 0) && t < nt) p = __double2float_rn(exp64(__dsub_rn((double)ssw[t * G + g], (double)mg)));
            if (G >= 2 || hp == 0) pbw[t * G + g] = p;
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) p = __fadd_rn(p, __shfl_xor_sync(FULL, p, off));
            ls[k] = p;
        }
#pragma unroll
        for (int g = 0; g < G; g++) lu[g] = __shfl_sync(FULL, ls[G >= 2 ? g >> 1 : 0], G >= 2 ? 16 * (g & 1) : 0);
    }
    __syncwarp();
    float oa[G][4];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < 4; e++) oa[g][e] = 0.f;
#pragma unroll 4
    for (int t = 0; t < nt; t++) {
        const uint2 vr = *reinterpret_cast<const uint2 *>(vrow + (size_t)t * 128);
        const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vr.x));
        const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vr.y));
        const float vf[4] = {v01.x, v01.y, v23.x, v23.y};
        float pg[G];
        if constexpr (G % 4 == 0) {
#pragma unroll
            for (int g = 0; g < G; g += 4) {
                const float4 x = *reinterpret_cast<const float4 *>(pbw + t * G + g);
                pg[g] = x.x;
                pg[g + 1] = x.y;
                pg[g + 2] = x.z;
                pg[g + 3] = x.w;
            }
        } else {
#pragma unroll
            for (int g = 0; g < G; g++) pg[g] = pbw[t * G + g];
        }
#pragma unroll
        for (int g = 0; g < G; g++)
#pragma unroll
            for (int e = 0; e < 4; e++) oa[g][e] = __fmaf_rn(pg[g], vf[e], oa[g][e]);
    }
    // fold: of the two weights one is 1 (exp64(0) = 1 exactly); lane j
    // evaluates the other one for head j % G
    double ef;
    {
        float mr = m_run[0], mu = mx[0];
#pragma unroll
        for (int g = 1; g < G; g++)
            if (lane % G == g) {
                mr = m_run[g];
                mu = mx[g];
            }
        const float hi = fmaxf(mr, mu), lo = fminf(mr, mu);
        ef = lo == -INFINITY ? 0.0 : exp64(__dsub_rn((double)lo, (double)hi));
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
        const double f = __shfl_sync(FULL, ef, g);
        if (mx[g] > m_run[g]) {  // warp-uniform: the running state is rescaled
#pragma unroll
            for (int e = 0; e < 4; e++) o[g][e] = __fma_rn(o[g][e], f, (double)oa[g][e]);
            Lw[g] = __fma_rn(Lw[g], f, (double)lu[g]);
            m_run[g] = mx[g];
        } else {
#pragma unroll
            for (int e = 0; e < 4; e++) o[g][e] = __fma_rn(f, (double)oa[g][e], o[g][e]);
            Lw[g] = __fma_rn(f, (double)lu[g], Lw[g]);
        }
    }
}

}  // namespace fb
