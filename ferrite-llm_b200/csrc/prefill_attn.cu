// Causal attention for a batched prefill: T new queries of one sequence
// (positions pos0 .. pos0 + T - 1) against its paged fp16 KV cache, which
// the prologue kernel has already extended with the T new keys/values.
//
// Replaces the prompt pass of candle-transformers 0.8.4 quantized_llama's
// attention (softmax(q.k^T / sqrt(hd) + causal mask) . v over the
// concatenated KV cache; called from crates/ferrite-wasm-host/src/
// adapter.rs:61-70 with all prompt tokens at once) -- the reference itself
// feeds the prompt token by token (crates/ferrite-core/src/chat_session.rs:
// 417-424), which this path replaces.  The reference's own flash-attention
// kernel (crates/ferrite-core/kernels/flash_attention.cu:166-225) is an f32
// stub that is never launched.
//
// B200 design (5th-generation tensor cores; tensor-bound at long prompts):
//  * one CTA per (128 queries, query head); 10 warps: warps 0..7 run the
//    softmax (warp w: TMEM lane quarter w % 4, i.e. query rows 32 (w % 4) ..
//    +31, and key columns 32 (w / 4) .. +31 of each block; both warps of a
//    row read all 64 scores for the row max), warp 8 issues the TMA
//    copies, warp 9 allocates tensor memory and issues tcgen05.mma from one
//    thread;
//  * key blocks of 64 = one KV page.  The dim-major K page [128 dims][64
//    keys] and the token-major V page [64 keys][128 dims] are copied by TMA
//    with 128-byte swizzle straight into the MN-major layouts of the B
//    operands (no transposes); K runs three stages ahead (a stage frees as
//    soon as S of its block completes), V two (freed by O of its block);
//  * S = Q K^T (M = 128, N = 64, K = 128) into one of two TMEM buffers, so
//    the MMA of block j + 1 overlaps the softmax of block j; O += P V (M =
//    128, N = 128, K = 64) accumulates in TMEM for the whole key range;
//  * precision: q and the probabilities enter the MMAs as fp16 hi + lo
//    parts (two MMAs each, ~22 bits of the f32 operands); K and V are fp16 in
//    the cache already; products accumulate in f32;
//  * softmax in log2 units with a lazy reference max: O and the row sum are
//    rescaled (tcgen05.ld / st) only when a row's max grows by more than 8,
//    so p stays below 256 and most blocks never touch the accumulator;
//  * every mbarrier wait is bounded; a timeout raises ERRBIT_WAIT_TIMEOUT and
//    the roles stop.
#include <math.h>

#include "fb_internal.h"
#include "kq_common.cuh"
#include "tc_common.cuh"

namespace fb {

constexpr int TA_Q = 128;        // queries per CTA (MMA M)
constexpr int TA_KB = 64;        // keys per block (one page)
constexpr int TA_HD = 128;
constexpr int TA_KS = 3;         // K stages (freed when S of their block completes)
constexpr int TA_VS = 2;         // V stages (freed when O += P V of their block completes)
constexpr int TA_THREADS = 320;  // warps 0..7 softmax, 8 TMA, 9 MMA
constexpr uint32_t TA_Q_BYTES = TA_Q * TA_HD * 2;   // two 64-dim slabs of [128 rows][128 B], K-major
constexpr uint32_t TA_K_BYTES = TA_HD * TA_KB * 2;  // [128 dims][64 keys]: MN-major B of S
constexpr uint32_t TA_V_BYTES = TA_KB * TA_HD * 2;  // two [64 keys][64 dims] halves: MN-major B of O
constexpr uint32_t TA_P_BYTES = TA_Q * TA_KB * 2;   // [128 rows][64 keys], K-major A of O
constexpr size_t TA_SMEM = 1024 + 2 * (size_t)TA_Q_BYTES + TA_KS * (size_t)TA_K_BYTES + TA_VS * (size_t)TA_V_BYTES +
                           4 * (size_t)TA_P_BYTES;
constexpr uint32_t TA_TMEM_COLS = 256;  // S buffers at columns 0 and 64, O at 128
constexpr uint32_t TA_O_COL = 128;
constexpr uint32_t TA_IDESC_S = umma_idesc_f16(TA_Q, TA_KB, false, true);
constexpr uint32_t TA_IDESC_O = umma_idesc_f16(TA_Q, TA_HD, false, true);
static_assert(TA_SMEM <= 227 * 1024, "prefill attention stages must fit");

// Byte offset of 16-byte chunk c of row r in a K-major, 128-byte-swizzled
// [rows][128 B] slab (8-row atoms of 1024 bytes, the TMA SWIZZLE_128B pattern).
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// 2^x (the SFU's approximation: relative error about 2^-22).
__device__ __forceinline__ float exp2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Eight f32 as fp16 hi parts and fp16 lo parts (x - hi).
__device__ __forceinline__ void split8(const float (&x)[8], uint4 &hi, uint4 &lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const __half2 a = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
        const float2 af = __half22float2(a);
        const __half2 b = __floats2half2_rn(__fsub_rn(x[2 * i], af.x), __fsub_rn(x[2 * i + 1], af.y));
        h[i] = *reinterpret_cast<const uint32_t *>(&a);
        l[i] = *reinterpret_cast<const uint32_t *>(&b);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// grid (ceil(T / 128), n_heads), TA_THREADS threads, TA_SMEM dynamic shared memory.
// kmap: the K pool as rows of 64 keys ([num_pages * n_kv * 128] x 64 fp16),
// vmap: the V pool as rows of 128 dims ([num_pages * n_kv * 64] x 128 fp16).
__global__ void __launch_bounds__(TA_THREADS, 1)
    k_attn_prefill_tc(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                      const float *__restrict__ q, const int32_t *__restrict__ bt, int max_pages, int num_pages,
                      int pos0, int T, int n_heads, int n_kv, float scale, float *__restrict__ out, uint32_t *err) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t k_full[TA_KS], k_empty[TA_KS], v_full[TA_VS], v_empty[TA_VS], s_full[2], s_free[2], p_full[2],
        p_free[2], o_done, fin;
    __shared__ uint32_t s_tmem;
    __shared__ float s_l[2][TA_Q];  // [column half][row]: the halves' row sums
    __shared__ uint64_t l_bar[4];   // the two warps of a lane quarter exchanged them
    __shared__ int s_abort_raw;
    volatile int &s_abort = s_abort_raw;
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sQh = sm, *sQl = sm + TA_Q_BYTES;
    uint8_t *sK = sQl + TA_Q_BYTES;         // [stage] K page
    uint8_t *sV = sK + TA_KS * TA_K_BYTES;  // [stage] V page (dims 0..63, then 64..127)
    uint8_t *sP = sV + TA_VS * TA_V_BYTES;  // [buffer][hi, lo] probabilities
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // query tiles in reverse order: the long (late, causal) tiles start first
    const int q0 = (gridDim.x - 1 - blockIdx.x) * TA_Q, h = blockIdx.y, kvh = h / (n_heads / n_kv);
    const int qlast = min(T, q0 + TA_Q) - 1;
    const int nkb = (pos0 + qlast) / TA_KB + 1;  // key blocks up to the CTA's last query
    if (threadIdx.x == 0) {
        for (int i = 0; i < TA_KS; i++) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
        }
        for (int i = 0; i < TA_VS; i++) {
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 8);
            mbar_init(&p_full[i], 8);
            mbar_init(&p_free[i], 1);
        }
        mbar_init(&o_done, 1);
        mbar_init(&fin, 1);
        for (int i = 0; i < 4; i++) {
            mbar_init(&l_bar[i], 64);
        }
        mbar_fence_init();
        s_abort = 0;
    }
    if (warp == 9) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(TA_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (warp < 8) {
        // q rows as fp16 hi / lo A operands (rows past T repeat the last
        // query; their results are not stored); thread: row, 64-dim half
        const int r = threadIdx.x & 127;
        const float *qr = q + ((int64_t)min(q0 + r, T - 1) * n_heads + h) * TA_HD;
#pragma unroll 4
        for (int c = 8 * (threadIdx.x >> 7); c < 8 * (threadIdx.x >> 7) + 8; c++) {
            const float4 a = *reinterpret_cast<const float4 *>(qr + 8 * c);
            const float4 b = *reinterpret_cast<const float4 *>(qr + 8 * c + 4);
            const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
            uint4 hi, lo;
            split8(x, hi, lo);
            const uint32_t off = (uint32_t)(c >> 3) * (TA_Q * 128) + sw128_off(r, c & 7);
            *reinterpret_cast<uint4 *>(sQh + off) = hi;
            *reinterpret_cast<uint4 *>(sQl + off) = lo;
        }
        fence_proxy_async_smem();  // the tensor core reads them through the async proxy
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == 8) {
        // ---- TMA, in the order the MMAs consume the pages: K_0, then per
        // block j K_{j+1} and V_j; block-table ids are read one block ahead
        if (lane == 0) {
            auto page_of = [&](int j) {
                int page = j < max_pages ? bt[j] : -1;
                if (page < 0 || page >= num_pages) {
                    atomicOr(err, ERRBIT_BAD_PAGE);
                    page = 0;
                }
                return page * n_kv + kvh;
            };
            int nk = 0, nv = 0;  // copies issued
            auto issue_k = [&](int j, int pk) -> bool {
                const int st = j % TA_KS;
                if (j >= TA_KS && !mbar_wait_bounded(&k_empty[st], (uint32_t)((j / TA_KS) - 1) & 1u)) return false;
                mbar_expect_tx(&k_full[st], TA_K_BYTES);
                tma_load_2d(sK + st * TA_K_BYTES, &kmap, 0, pk * TA_HD, &k_full[st]);
                nk = j + 1;
                return true;
            };
            auto issue_v = [&](int j, int pk) -> bool {
                const int st = j % TA_VS;
                if (j >= TA_VS && !mbar_wait_bounded(&v_empty[st], (uint32_t)((j / TA_VS) - 1) & 1u)) return false;
                mbar_expect_tx(&v_full[st], TA_V_BYTES);
                tma_load_2d(sV + st * TA_V_BYTES, &vmap, 0, pk * TA_KB, &v_full[st]);
                tma_load_2d(sV + st * TA_V_BYTES + TA_V_BYTES / 2, &vmap, 64, pk * TA_KB, &v_full[st]);
                nv = j + 1;
                return true;
            };
            int pg_cur = page_of(0), pg_nxt = nkb > 1 ? page_of(1) : 0;
            bool okp = issue_k(0, pg_cur);
            for (int j = 0; okp && j < nkb && !s_abort; j++) {
                const int pg_nn = j + 2 < nkb ? page_of(j + 2) : 0;
                if (j + 1 < nkb) okp = issue_k(j + 1, pg_nxt);
                if (okp) okp = issue_v(j, pg_cur);
                pg_cur = pg_nxt;
                pg_nxt = pg_nn;
            }
            if (!okp) s_abort = 1;
            // copies in flight land before shared memory is released
            for (int k = nk > TA_KS ? nk - TA_KS : 0; k < nk; k++)
                mbar_wait_bounded(&k_full[k % TA_KS], (uint32_t)(k / TA_KS) & 1u);
            for (int k = nv > TA_VS ? nv - TA_VS : 0; k < nv; k++)
                mbar_wait_bounded(&v_full[k % TA_VS], (uint32_t)(k / TA_VS) & 1u);
        }
    } else if (warp == 9) {
        // ---- MMA issue: S_{j+1} is issued before O_j so it overlaps block j's softmax
        if (lane == 0) {
            const uint32_t aQh = smem_u32(sQh), aQl = smem_u32(sQl), aK = smem_u32(sK), aV = smem_u32(sV),
                           aP = smem_u32(sP);
            auto issue_s = [&](int j) -> bool {
                const int st = j % TA_KS, sb = j & 1;
                if (!mbar_wait_bounded(&k_full[st], (uint32_t)(j / TA_KS) & 1u)) return false;
                if (j >= 2 && !mbar_wait_bounded(&s_free[sb], (uint32_t)((j >> 1) - 1) & 1u)) return false;
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < TA_HD / 16; ks++) {  // 16 dims: 16 K rows of the MN-major page
                    const uint32_t qo = (uint32_t)(ks >> 2) * (TA_Q * 128) + (uint32_t)(ks & 3) * 32;
                    const uint64_t db = umma_desc_mn_sw128(aK + st * TA_K_BYTES + ks * 2048, TA_K_BYTES, 1024);
                    umma_f16_desc(tmem + sb * TA_KB, umma_desc_sw128(aQh + qo), db, TA_IDESC_S, ks > 0 ? 1u : 0u);
                    umma_f16_desc(tmem + sb * TA_KB, umma_desc_sw128(aQl + qo), db, TA_IDESC_S, 1u);
                }
                umma_commit(&s_full[sb]);
                umma_commit(&k_empty[st]);
                return true;
            };
            auto issue_o = [&](int j) -> bool {
                const int st = j % TA_VS, pb = j & 1;
                if (!mbar_wait_bounded(&p_full[pb], (uint32_t)(j >> 1) & 1u)) return false;
                if (!mbar_wait_bounded(&v_full[st], (uint32_t)(j / TA_VS) & 1u)) return false;
                tc_fence_after();
                const uint32_t ph = aP + pb * 2 * TA_P_BYTES, pl = ph + TA_P_BYTES;
#pragma unroll
                for (int ks = 0; ks < TA_KB / 16; ks++) {  // 16 keys: 16 K rows of both V halves
                    const uint64_t db = umma_desc_mn_sw128(aV + st * TA_V_BYTES + ks * 2048, TA_V_BYTES / 2, 1024);
                    umma_f16_desc(tmem + TA_O_COL, umma_desc_sw128(ph + ks * 32), db, TA_IDESC_O,
                                  (j > 0 || ks > 0) ? 1u : 0u);
                    umma_f16_desc(tmem + TA_O_COL, umma_desc_sw128(pl + ks * 32), db, TA_IDESC_O, 1u);
                }
                umma_commit(&v_empty[st]);
                umma_commit(&p_free[pb]);
                umma_commit(&o_done);
                return true;
            };
            bool okm = issue_s(0);
            for (int j = 0; okm && j < nkb && !s_abort; j++) {
                if (j + 1 < nkb) okm = issue_s(j + 1);
                if (okm) okm = issue_o(j);
            }
            if (!okm) s_abort = 1;
            umma_commit(&fin);  // every MMA issued has completed before TMEM is released
            mbar_wait_bounded(&fin, 0);
        }
    } else {
        // ---- softmax: thread = query row r (TMEM lane) x 32 key columns
        constexpr unsigned FULL = 0xffffffffu;
        const int qd = warp & 3, ch = warp >> 2;
        const int r = 32 * qd + lane;
        const int qpos = pos0 + min(q0 + r, T - 1);
        const int qpos_min = pos0 + q0;  // no mask before the CTA's first query
        const uint32_t lt = tmem + ((uint32_t)(32 * qd) << 16);
        const float sl2 = __fmul_rn(scale, 1.4426950408889634f);  // scores in log2 units
        float m = -INFINITY, l = 0.f;  // reference max (log2 units), this half's row sum
        bool okw = true;
        for (int j = 0; j < nkb && okw; j++) {
            const int sb = j & 1;
            if (!(okw = mbar_wait_bounded(&s_full[sb], (uint32_t)(j >> 1) & 1u))) break;
            tc_fence_after();
            uint32_t sv[32], so[32];  // this warp's 32 columns and the other half (row max only)
            tmem_ld32(lt + sb * TA_KB + 32 * ch, sv);
            tmem_ld32(lt + sb * TA_KB + 32 * (ch ^ 1), so);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[sb]);  // the MMA of block j + 2 may overwrite it
            // scale, causal mask (keys after the query's position), row max
            const int key0 = j * TA_KB + 32 * ch, keyo = j * TA_KB + 32 * (ch ^ 1);
            float x[32];
            float bm = -INFINITY;
            if (j * TA_KB + TA_KB - 1 <= qpos_min) {
#pragma unroll
                for (int t = 0; t < 32; t++) {
                    x[t] = __fmul_rn(__uint_as_float(sv[t]), sl2);
                    bm = fmaxf(bm, fmaxf(x[t], __fmul_rn(__uint_as_float(so[t]), sl2)));
                }
            } else {
#pragma unroll
                for (int t = 0; t < 32; t++) {
                    x[t] = key0 + t <= qpos ? __fmul_rn(__uint_as_float(sv[t]), sl2) : -INFINITY;
                    const float xo = keyo + t <= qpos ? __fmul_rn(__uint_as_float(so[t]), sl2) : -INFINITY;
                    bm = fmaxf(bm, fmaxf(x[t], xo));
                }
            }
            const float mn = fmaxf(m, bm);  // finite: key 0 precedes every query
            const bool need = j > 0 && mn > m + 8.f;
            if (__any_sync(FULL, need)) {
                // rescale this warp's half of the accumulator rows once O += P_{j-1} V_{j-1} has landed
                if (!(okw = mbar_wait_bounded(&o_done, (uint32_t)(j - 1) & 1u))) break;
                tc_fence_after();
                const float al = need ? exp2_approx(__fsub_rn(m, mn)) : 1.f;
#pragma unroll 1
                for (int c = 0; c < 2; c++) {
                    uint32_t ov[32];
                    tmem_ld32(lt + TA_O_COL + 64 * ch + 32 * c, ov);
#pragma unroll
                    for (int i = 0; i < 32; i++) ov[i] = __float_as_uint(__fmul_rn(__uint_as_float(ov[i]), al));
                    tmem_st32(lt + TA_O_COL + 64 * ch + 32 * c, ov);
                }
                tc_fence_before();
                if (need) {
                    l = __fmul_rn(l, al);
                    m = mn;
                }
            }
            if (j == 0) m = mn;
            // p = 2^(x - m) (<= 256), written as fp16 hi / lo A operands
            if (j >= 2 && !(okw = mbar_wait_bounded(&p_free[sb], (uint32_t)((j >> 1) - 1) & 1u))) break;
            uint8_t *ph = sP + sb * 2 * TA_P_BYTES, *pl = ph + TA_P_BYTES;
            float ls = 0.f;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                float p[8];
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    p[e] = exp2_approx(__fsub_rn(x[8 * c + e], m));
                    ls = __fadd_rn(ls, p[e]);
                }
                uint4 hi, lo;
                split8(p, hi, lo);
                *reinterpret_cast<uint4 *>(ph + sw128_off(r, 4 * ch + c)) = hi;
                *reinterpret_cast<uint4 *>(pl + sw128_off(r, 4 * ch + c)) = lo;
            }
            l = __fadd_rn(l, ls);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[sb]);
        }
        // ---- O / l once the last P V has landed (l = the two halves' sums)
        if (okw) okw = mbar_wait_bounded(&o_done, (uint32_t)(nkb - 1) & 1u);
        if (okw) {
            s_l[ch][r] = l;
            mbar_arrive(&l_bar[qd]);
            okw = mbar_wait_bounded(&l_bar[qd], 0);
            l = __fadd_rn(s_l[0][r], s_l[1][r]);
        }
        if (okw) {
            tc_fence_after();
            const float inv = l > 0.f ? __fdiv_rn(1.f, l) : 0.f;
            float *orow = out + ((int64_t)(q0 + r) * n_heads + h) * TA_HD + 64 * ch;
#pragma unroll 1
            for (int c = 0; c < 2; c++) {
                uint32_t ov[32];
                tmem_ld32(lt + TA_O_COL + 64 * ch + 32 * c, ov);
                if (q0 + r < T)
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4 *>(orow + 32 * c + i) =
                            make_float4(__fmul_rn(__uint_as_float(ov[i]), inv), __fmul_rn(__uint_as_float(ov[i + 1]), inv),
                                        __fmul_rn(__uint_as_float(ov[i + 2]), inv),
                                        __fmul_rn(__uint_as_float(ov[i + 3]), inv));
            }
        } else {
            s_abort = 1;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (s_abort && threadIdx.x == 0) atomicOr(err, ERRBIT_WAIT_TIMEOUT);
    if (warp == 9) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TA_TMEM_COLS)
                     : "memory");
    }
}

}  // namespace fb

namespace fb {

// fp16 pool viewed as rows of `inner` values, boxes of 64 values x box_rows
// rows, 128-byte swizzle (the MN-major B layouts above).
static CUtensorMap pool_map(const void *pool, int64_t rows, int64_t inner, uint32_t box_rows) {
    auto encode = tensor_map_encoder();
    FB_REQUIRE(encode != nullptr, "attn_prefill: cuTensorMapEncodeTiled is unavailable");
    FB_REQUIRE(((uintptr_t)pool & 15) == 0, "attn_prefill: KV pools must be 16-byte aligned");
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult cr = encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(pool), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    FB_REQUIRE(cr == CUDA_SUCCESS, "attn_prefill: tensor map encoding failed");
    return map;
}

void launch_attn_prefill(fb_ctx *ctx, const float *q, const void *kpool, const void *vpool, const int32_t *bt,
                         int max_pages, int num_pages, int pos0, int T, int n_heads, int n_kv, float scale,
                         float *out) {
    FB_REQUIRE(T >= 1 && pos0 >= 0 && n_kv >= 1 && n_heads % n_kv == 0, "attn_prefill: bad shape");
    FB_REQUIRE((pos0 + T + TA_KB - 1) / TA_KB <= max_pages, "attn_prefill: positions exceed the block table");
    FB_REQUIRE((int64_t)num_pages * n_kv * TA_HD < ((int64_t)1 << 31), "attn_prefill: KV pool too large");
    const CUtensorMap kmap = pool_map(kpool, (int64_t)num_pages * n_kv * TA_HD, TA_KB, TA_HD);
    const CUtensorMap vmap = pool_map(vpool, (int64_t)num_pages * n_kv * TA_KB, TA_HD, TA_KB);
    FB_CUDA(cudaFuncSetAttribute(k_attn_prefill_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TA_SMEM));
    dim3 grid((unsigned)((T + TA_Q - 1) / TA_Q), (unsigned)n_heads);
    k_attn_prefill_tc<<<grid, TA_THREADS, TA_SMEM, ctx->stream>>>(kmap, vmap, q, bt, max_pages, num_pages, pos0, T,
                                                                   n_heads, n_kv, scale, out, ctx->err_word);
    FB_CUDA(cudaGetLastError());
}

}  // namespace fb
