// Causal attention for a batched prefill: T new queries of one sequence
// (positions pos0 .. pos0 + T - 1) against its paged fp16 KV cache, which
// the prologue kernel has already extended with the T new keys/values.
//
// Replaces the prompt pass of candle-transformers 0.8.4 quantized_llama's
// attention (softmax(q.k^T / sqrt(hd) + causal mask) . v over the
// concatenated KV cache; called from crates/ferrite-wasm-host/src/
// adapter.rs:61-70 with all prompt tokens at once) -- the reference itself
// feeds the prompt token by token (crates/ferrite-core/src/chat_session.rs:
// 417-424), which this path replaces.
//
// Design (tensor cores through mma.sync.m16n8k16, f32 accumulation):
//  * one CTA of 4 warps per (64-query block, query head); warp w owns
//    queries 16w .. 16w + 15 of the block;
//  * key blocks of 64 = one KV page: its K (dim-major, 16 KB) and V
//    (token-major, 16 KB) stream into padded shared memory with cp.async
//    (double-buffered: block kb + 1 loads while kb is processed) and reach
//    the MMAs through ldmatrix.trans (both operands are K-major that way);
//  * precision: q and the softmax probabilities are split into fp16 hi + lo
//    parts (two MMAs each), so S = q.k and O = P.V carry ~22 bits of the
//    f32 operands; K and V are fp16 in the cache already (exact);
//  * online softmax per query row in f32 (running max, rescale by
//    exp(m_old - m_new)), causal mask on key > query position.
#include <math.h>

#include "fb_internal.h"
#include "kq_common.cuh"

namespace fb {

constexpr int PA_Q = 64;                 // queries per CTA
constexpr int PA_KB = 64;                // keys per block (one page)
constexpr int PA_HD = 128;
constexpr int PA_KP = PA_KB * 2 + 16;    // K smem row pitch (dims are rows): 144 B
constexpr int PA_VP = PA_HD * 2 + 16;    // V smem row pitch (keys are rows): 272 B
constexpr int PA_K_BYTES = PA_HD * PA_KP;  // 18432
constexpr int PA_V_BYTES = PA_KB * PA_VP;  // 17408
constexpr int PA_STAGE = PA_K_BYTES + PA_V_BYTES;
constexpr int PA_SMEM = 2 * PA_STAGE;  // 71680

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// (hi, lo) fp16 pair of two f32 values: hi = fp16(x), lo = fp16(x - hi)
__device__ __forceinline__ void split_h2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(__fsub_rn(x0, hf.x), __fsub_rn(x1, hf.y));
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

// grid (ceil(T / 64), n_heads), 128 threads.
__global__ void __launch_bounds__(128) k_attn_prefill(const float *__restrict__ q, const __half *__restrict__ kpool,
                                                      const __half *__restrict__ vpool,
                                                      const int32_t *__restrict__ bt, int max_pages, int num_pages,
                                                      int pos0, int T, int n_heads, int n_kv, float scale,
                                                      float *__restrict__ out, uint32_t *err) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int q0 = blockIdx.x * PA_Q, h = blockIdx.y, kvh = h / (n_heads / n_kv);
    const int qlast = min(T, q0 + PA_Q) - 1;  // last query of the CTA
    const int nkb = (pos0 + qlast) / PA_KB + 1;

    // q fragments of this warp's 16 queries (A operand, row-major 16 x 128),
    // hi and lo parts; rows past T read zeros
    uint32_t qa[8][4], qb[8][4];
    {
        const int r0 = q0 + 16 * warp + g, r1 = r0 + 8;
        const float *p0 = q + ((int64_t)min(r0, T - 1) * n_heads + h) * PA_HD;
        const float *p1 = q + ((int64_t)min(r1, T - 1) * n_heads + h) * PA_HD;
        const bool v0 = r0 < T, v1 = r1 < T;
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
#pragma unroll
            for (int half = 0; half < 2; half++) {  // columns 2c (+8 for half 1)
                const int col = 16 * kk + 2 * c + 8 * half;
                const float2 a = v0 ? *reinterpret_cast<const float2 *>(p0 + col) : make_float2(0.f, 0.f);
                const float2 b = v1 ? *reinterpret_cast<const float2 *>(p1 + col) : make_float2(0.f, 0.f);
                split_h2(a.x, a.y, qa[kk][2 * half], qb[kk][2 * half]);
                split_h2(b.x, b.y, qa[kk][2 * half + 1], qb[kk][2 * half + 1]);
            }
        }
    }
    const int qpos0 = pos0 + q0 + 16 * warp + g, qpos1 = qpos0 + 8;  // positions of this thread's two rows

    // stage loader: K page-head [128 dims][64 keys] and V page-head [64 keys][128 dims]
    const uint32_t sbase = smem_u32(smem);
    auto load = [&](int kb, int st) {
        int page = kb < max_pages ? bt[kb] : -1;
        if (page < 0 || page >= num_pages) {
            if (threadIdx.x == 0) atomicOr(err, ERRBIT_BAD_PAGE);
            page = 0;
        }
        const size_t off = ((size_t)page * n_kv + kvh) * (size_t)(PA_HD * PA_KB);
        const uint8_t *ks = reinterpret_cast<const uint8_t *>(kpool + off);
        const uint8_t *vs = reinterpret_cast<const uint8_t *>(vpool + off);
        const uint32_t kd = sbase + st * PA_STAGE, vd = kd + PA_K_BYTES;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int ch = threadIdx.x + 128 * i;  // 1024 chunks of 16 bytes each
            cp_async16(kd + (ch >> 3) * PA_KP + (ch & 7) * 16, ks + ch * 16);
            cp_async16(vd + (ch >> 4) * PA_VP + (ch & 15) * 16, vs + ch * 16);
        }
        cp_async_commit();
    };

    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    load(0, 0);
    for (int kb = 0; kb < nkb; kb++) {
        const int st = kb & 1;
        if (kb + 1 < nkb) {
            load(kb + 1, st ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const uint32_t kd = sbase + st * PA_STAGE, vd = kd + PA_K_BYTES;
        // ---- S = q . k^T for 16 queries x 64 keys (8 n-tiles of 8 keys)
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; i++) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
#pragma unroll
            for (int np = 0; np < 4; np++) {  // n-tile pairs (2np, 2np + 1)
                // matrices: dims 16kk + {0..7, 8..15} x keys 8(2np) .. / 8(2np+1) ..
                const int mi = lane >> 3, rr = lane & 7;
                const int dim = 16 * kk + (mi & 1) * 8 + rr, key = 8 * (2 * np + (mi >> 1));
                uint32_t b[4];
                ldsm_x4_trans(b, kd + dim * PA_KP + key * 2);
                mma16816(s[2 * np], qa[kk], b[0], b[1]);
                mma16816(s[2 * np], qb[kk], b[0], b[1]);
                mma16816(s[2 * np + 1], qa[kk], b[2], b[3]);
                mma16816(s[2 * np + 1], qb[kk], b[2], b[3]);
            }
        }
        // ---- scale, causal mask, online softmax (rows g and g + 8 of the warp)
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int key = kb * PA_KB + 8 * nt + 2 * c + e;
                s[nt][e] = key <= qpos0 ? __fmul_rn(s[nt][e], scale) : -INFINITY;
                s[nt][2 + e] = key <= qpos1 ? __fmul_rn(s[nt][2 + e], scale) : -INFINITY;
                mx0 = fmaxf(mx0, s[nt][e]);
                mx1 = fmaxf(mx1, s[nt][2 + e]);
            }
        }
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
        }
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        // rows with no visible key yet keep zero weight (mn = -inf)
        const float al0 = mn0 == -INFINITY ? 1.f : expf(m0 - mn0);
        const float al1 = mn1 == -INFINITY ? 1.f : expf(m1 - mn1);
        m0 = mn0;
        m1 = mn1;
        float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                s[nt][e] = mn0 == -INFINITY ? 0.f : expf(s[nt][e] - mn0);
                s[nt][2 + e] = mn1 == -INFINITY ? 0.f : expf(s[nt][2 + e] - mn1);
                ps0 += s[nt][e];
                ps1 += s[nt][2 + e];
            }
        }
        l0 = l0 * al0 + ps0;
        l1 = l1 * al1 + ps1;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            o[i][0] *= al0;
            o[i][1] *= al0;
            o[i][2] *= al1;
            o[i][3] *= al1;
        }
        // ---- O += P . V: k-steps of 16 keys (n-tiles 2j, 2j + 1 of S), 16 dim n-tiles
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint32_t pa[4], pb[4];
            split_h2(s[2 * j][0], s[2 * j][1], pa[0], pb[0]);
            split_h2(s[2 * j][2], s[2 * j][3], pa[1], pb[1]);
            split_h2(s[2 * j + 1][0], s[2 * j + 1][1], pa[2], pb[2]);
            split_h2(s[2 * j + 1][2], s[2 * j + 1][3], pa[3], pb[3]);
#pragma unroll
            for (int dp = 0; dp < 8; dp++) {  // dim n-tile pairs (2dp, 2dp + 1)
                const int mi = lane >> 3, rr = lane & 7;
                const int key = 16 * j + (mi & 1) * 8 + rr, dim = 8 * (2 * dp + (mi >> 1));
                uint32_t b[4];
                ldsm_x4_trans(b, vd + key * PA_VP + dim * 2);
                mma16816(o[2 * dp], pa, b[0], b[1]);
                mma16816(o[2 * dp], pb, b[0], b[1]);
                mma16816(o[2 * dp + 1], pa, b[2], b[3]);
                mma16816(o[2 * dp + 1], pb, b[2], b[3]);
            }
        }
        __syncthreads();  // stage st is refilled by the next iteration's load
    }
    // ---- normalise and store
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, off);
        l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    const int r0 = q0 + 16 * warp + g, r1 = r0 + 8;
    const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
    for (int dn = 0; dn < 16; dn++) {
        const int dim = 8 * dn + 2 * c;
        if (r0 < T)
            *reinterpret_cast<float2 *>(out + ((int64_t)r0 * n_heads + h) * PA_HD + dim) =
                make_float2(o[dn][0] * i0, o[dn][1] * i0);
        if (r1 < T)
            *reinterpret_cast<float2 *>(out + ((int64_t)r1 * n_heads + h) * PA_HD + dim) =
                make_float2(o[dn][2] * i1, o[dn][3] * i1);
    }
}

void launch_attn_prefill(fb_ctx *ctx, const float *q, const void *kpool, const void *vpool, const int32_t *bt,
                         int max_pages, int num_pages, int pos0, int T, int n_heads, int n_kv, float scale,
                         float *out) {
    FB_REQUIRE(T >= 1 && pos0 >= 0 && n_heads % n_kv == 0, "attn_prefill: bad shape");
    FB_REQUIRE((pos0 + T + PA_KB - 1) / PA_KB <= max_pages, "attn_prefill: positions exceed the block table");
    FB_CUDA(cudaFuncSetAttribute(k_attn_prefill, cudaFuncAttributeMaxDynamicSharedMemorySize, PA_SMEM));
    dim3 grid((unsigned)((T + PA_Q - 1) / PA_Q), (unsigned)n_heads);
    k_attn_prefill<<<grid, 128, PA_SMEM, ctx->stream>>>(q, (const __half *)kpool, (const __half *)vpool, bt, max_pages,
                                                         num_pages, pos0, T, n_heads, n_kv, scale, out,
                                                         ctx->err_word);
    FB_CUDA(cudaGetLastError());
}

}  // namespace fb
