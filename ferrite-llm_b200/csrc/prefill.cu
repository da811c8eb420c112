// Prefill QMatMul on the 5th-generation tensor cores:
//   Y[T, N] = X[T, K] . dequant(W)[N, K]^T     (T >= 17 rows, Q4_K / Q6_K W)
//
// Replaces candle's large-m QMatMul (quantized_llama's prompt forward; the
// reference's CUDA build runs MMQ `mul_mat_q4_K` at ferrite-os/crates/
// internal/ptx-kernels/kernels/candle/quantized.cu:4297 or dequantize + GEMM).
// Arithmetic: W is dequantized in fp16 with candle's `to_float` factors
// (w = fp16(fp16(d*sc) * q - fp16(dmin*m)), see dequant_slice_*); X is
// scaled per row by an exact power of two that keeps |x| below 32768 and
// rounded to fp16; the products accumulate in f32 in tensor memory; the row
// scale is applied in the epilogue.
//
// B200 design (tensor-bound: 2 T N K flops):
//  * one CTA per 256 x 128 output tile (256 tokens, 128 weight rows) as two
//    cta_group::1 MMAs of M = 128 sharing each dequantized B slice, so the
//    dequantization -- the CTA's CUDA-core work -- is amortized over 256
//    token rows; 10 warps: warp 0 feeds the pipeline (TMA tensor loads of
//    fp16 X tiles with 128-byte swizzle; cp.async.bulk of the tile-major
//    weight records, one contiguous 16-row x 256-column record per copy),
//    warp 1 allocates tensor memory (two 128-column f32 accumulators) and
//    issues tcgen05.mma from one thread, warps 2..9 (two threads per weight
//    row) dequantize each 64-column slice of the weight records into the
//    K-major, 128-byte-swizzled fp16 B operand and then drain the
//    accumulators with tcgen05.ld;
//  * 3 smem stages of (A 32 KB + B 16 KB) plus two record buffers;
//    mbarriers between the roles, every wait bounded (a timeout raises
//    ERRBIT_WAIT_TIMEOUT and all roles stop).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "fb_internal.h"
#include "kq_common.cuh"
#include "tc_common.cuh"

namespace fb {

constexpr int PF_BM = 256, PF_BN = 128, PF_BK = 64;  // tile; K step = one 128-byte swizzle row of fp16
constexpr int PF_MH = 128;                            // rows of one MMA (accumulator half of the tile)
constexpr int PF_STAGES = 3;
constexpr int PF_DQ_WARPS = 8;                        // dequant / epilogue warps (two per weight row)
constexpr int PF_THREADS = 64 + 32 * PF_DQ_WARPS;
constexpr uint32_t PF_A_BYTES = PF_BM * PF_BK * 2, PF_B_BYTES = PF_BN * PF_BK * 2;  // 32 KB, 16 KB
constexpr uint32_t PF_TMEM_COLS = 2 * PF_BN;  // two f32 accumulators of 128 columns
constexpr int PF_TILES_N = PF_BN / 16;                                              // weight row tiles per CTA

template <int DT> struct PfRec;
template <> struct PfRec<4> { static constexpr int bytes = Q4K_REC; };
template <> struct PfRec<6> { static constexpr int bytes = Q6K_REC; };

template <int DT>
constexpr size_t pf_smem_bytes() {
    return 1024 /* alignment slack */ + (size_t)PF_STAGES * (PF_A_BYTES + PF_B_BYTES) +
           2 * (size_t)PF_TILES_N * PfRec<DT>::bytes;
}

// ---- tcgen05 / TMA helpers -------------------------------------------------
// kind::f16 instruction descriptor: A = B = fp16, D = f32, both K-major,
// M = 128, N = 128
constexpr uint32_t PF_IDESC = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(PF_BN >> 3) << 17) |
                              ((uint32_t)(PF_MH >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(PF_IDESC), "r"(accumulate)
        : "memory");
}

// Packed fp16 dequantization (two weights per instruction).  A weight's
// integer code q goes into an fp16 exactly as 1024 + q (bits 0x6400 | q) and
// 1024 is subtracted; the factors are fp16 roundings of the exact f32
// products d * sc (and dmin * m):  w = fp16(fp16(d*sc) * q - fp16(dmin*m))
// for Q4_K (one fused multiply-add, one rounding) and
// w = fp16(fp16(d*sc) * (q - 32)) for Q6_K.
__device__ __forceinline__ __half2 h2_bits(uint32_t v) { return *reinterpret_cast<const __half2 *>(&v); }
__device__ __forceinline__ uint32_t bits_h2(__half2 v) { return *reinterpret_cast<const uint32_t *>(&v); }
__device__ __forceinline__ __half half_of_small_uint(uint32_t v) {  // 0 <= v < 1024, exact
    return __hsub(__ushort_as_half((unsigned short)(0x6400u | v)), __ushort_as_half((unsigned short)0x6400u));
}

// Half hf (0, 1) of the 64-column slice c (0..3) of one weight row's
// super-block (row r of the 16-row tile record `rec`) -> 4 chunks of 8 fp16
// weights (uint4 each): chunks 4 hf .. 4 hf + 3 (k = 8q .. 8q+7 of the slice).
__device__ __forceinline__ void dequant_slice_q4k(const uint8_t *rec, int r, int c, int hf, uint4 (&out)[4]) {
    const uint8_t *blk = rec + r * 144;
    const uint4 hd = *reinterpret_cast<const uint4 *>(blk);
    const Q4Scales s = q4k_unpack_scales(hd.y, hd.z, hd.w);
    // group g = c: sub-block 2c (low nibbles, chunks 0..3) or 2c + 1 (high nibbles, chunks 4..7)
    const int j = 2 * c + hf;
    const uint32_t sc = (uint32_t)byte_of(j < 4 ? s.sc_lo : s.sc_hi, j & 3);
    const uint32_t mn = (uint32_t)byte_of(j < 4 ? s.mn_lo : s.mn_hi, j & 3);
    const __half d1 = __hmul(__ushort_as_half((unsigned short)(hd.x & 0xFFFF)), half_of_small_uint(sc));
    const __half m1 = __hmul(__ushort_as_half((unsigned short)(hd.x >> 16)), half_of_small_uint(mn));
    const __half2 d12 = __halves2half2(d1, d1), nm12 = __halves2half2(__hneg(m1), __hneg(m1));
    const __half2 k1024 = h2_bits(0x64006400u);
#pragma unroll
    for (int t = 0; t < 4; t++) {
        const uint2 q = *reinterpret_cast<const uint2 *>(blk + 16 + 32 * t + 8 * c);
        uint32_t w[4];
#pragma unroll
        for (int pr = 0; pr < 4; pr++) {  // bytes (2pr, 2pr + 1) of the 8
            const uint32_t word = pr < 2 ? q.x : q.y;
            uint32_t p = __byte_perm(word, 0u, (pr & 1) ? 0x4342u : 0x4140u);  // byte pair -> halves
            if (hf) p >>= 4;
            const __half2 nib = __hsub2(h2_bits((p & 0x000F000Fu) | 0x64006400u), k1024);
            w[pr] = bits_h2(__hfma2(d12, nib, nm12));
        }
        out[t] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__device__ __forceinline__ void dequant_slice_q6k(const uint8_t *rec, int r, int c, int hf, uint4 (&out)[4]) {
    const uint32_t *blk = reinterpret_cast<const uint32_t *>(rec + r * 208);
    const __half d = __ushort_as_half(*reinterpret_cast<const uint16_t *>(rec + 3328 + 2 * r));
    const int h = c >> 1;
    const __half2 k1056 = h2_bits(0x64206420u);  // 1024 + 32
#pragma unroll
    for (int qq = 0; qq < 4; qq++) {
        const int q = 4 * hf + qq;
        const int p = 2 * (c & 1) + (q >> 2), t = q & 3;
        const int sc = sbyte_of(blk[48 + c], q >> 1);  // int8
        const __half ds = __hmul(d, __hsub(half_of_small_uint((uint32_t)(sc + 128)),
                                           __ushort_as_half((unsigned short)0x5800u)));  // sc exactly (128 = 0x5800)
        const __half2 ds2 = __halves2half2(ds, ds);
        uint32_t w[4];
#pragma unroll
        for (int pr = 0; pr < 4; pr++) {  // weights (2pr, 2pr + 1) of the chunk
            const int x = pr >> 1;
            const uint32_t sel = (pr & 1) ? 0x4342u : 0x4140u;
            const uint32_t lo = (__byte_perm(blk[12 * t + 4 * h + 2 * (p & 1) + x], 0u, sel) >> (4 * (p >> 1))) & 0x000F000Fu;
            const uint32_t hi = (__byte_perm(blk[12 * t + 8 + 2 * h + x], 0u, sel) >> (2 * p)) & 0x00030003u;
            const __half2 qc = __hsub2(h2_bits(lo | (hi << 4) | 0x64006400u), k1056);  // q6 - 32, exact
            w[pr] = bits_h2(__hmul2(ds2, qc));
        }
        out[qq] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// grid (N / 128, ceil(T / 256)), PF_THREADS threads.
template <int DT>
__global__ void __launch_bounds__(PF_THREADS, 1)
    k_prefill_gemm(const __grid_constant__ CUtensorMap xmap, const uint8_t *__restrict__ W, int64_t nb, int T,
                   int64_t N, const float *__restrict__ rowscale, float *__restrict__ Y, uint32_t *err) {
    constexpr int REC = PfRec<DT>::bytes;
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t a_full[PF_STAGES], b_full[PF_STAGES], empty[PF_STAGES], rec_full[2], rec_empty[2], acc_full;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort_raw;
    volatile int &s_abort = s_abort_raw;  // set by any role that gives up; polled by the others
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sA = smem, *sB = smem + PF_STAGES * PF_A_BYTES;
    uint8_t *sRec = sB + PF_STAGES * PF_B_BYTES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tile = blockIdx.x, m0 = blockIdx.y * PF_BM;
    const int ksteps = (int)nb * 4;

    if (threadIdx.x == 0) {
        for (int i = 0; i < PF_STAGES; i++) {
            mbar_init(&a_full[i], 1);
            mbar_init(&b_full[i], PF_DQ_WARPS);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&rec_full[i], 1);
            mbar_init(&rec_empty[i], PF_DQ_WARPS);
        }
        mbar_init(&acc_full, 1);
        mbar_fence_init();
        s_abort = 0;
    }
    if (warp == 1) {
        // two accumulators (token rows m0.. and m0+128..) of 128 f32 columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(PF_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            const uint8_t *wtiles = W + (size_t)n_tile * PF_TILES_N * nb * REC;
            for (int s = 0; s < ksteps && !s_abort; s++) {
                const int st = s % PF_STAGES;
                if (s >= PF_STAGES && !mbar_wait_bounded(&empty[st], (uint32_t)((s / PF_STAGES) - 1) & 1u)) {
                    s_abort = 1;
                    break;
                }
                mbar_expect_tx(&a_full[st], PF_A_BYTES);
                tma_load_2d(sA + st * PF_A_BYTES, &xmap, s * PF_BK, m0, &a_full[st]);
                if (s % 4 == 0) {
                    const int sb = s / 4, rb = sb & 1;
                    if (sb >= 2 && !mbar_wait_bounded(&rec_empty[rb], (uint32_t)((sb >> 1) - 1) & 1u)) {
                        s_abort = 1;
                        break;
                    }
                    mbar_expect_tx(&rec_full[rb], PF_TILES_N * REC);
                    for (int tt = 0; tt < PF_TILES_N; tt++)
                        bulk_g2s(sRec + ((size_t)rb * PF_TILES_N + tt) * REC,
                                 wtiles + ((size_t)tt * nb + sb) * REC, REC, &rec_full[rb]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t aBase = smem_u32(sA), bBase = smem_u32(sB);
            for (int s = 0; s < ksteps && !s_abort; s++) {
                const int st = s % PF_STAGES;
                const uint32_t par = (uint32_t)(s / PF_STAGES) & 1u;
                if (!mbar_wait_bounded(&a_full[st], par) || !mbar_wait_bounded(&b_full[st], par)) {
                    s_abort = 1;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < PF_BK / 16; kk++) {
                    const uint64_t db = umma_desc_sw128(bBase + st * PF_B_BYTES + kk * 32);
#pragma unroll
                    for (int h = 0; h < 2; h++) {  // token rows 128h .. 128h + 127 of the tile
                        const uint64_t da = umma_desc_sw128(aBase + st * PF_A_BYTES + h * (PF_MH * 128) + kk * 32);
                        umma_f16(tmem + h * PF_BN, da, db, (s > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                umma_commit(&empty[st]);  // frees the stage once these MMAs have read it
            }
            umma_commit(&acc_full);
        }
    } else {
        // warps 2..9: dequantize (thread = weight row x half slice), then
        // drain the accumulator (warp quarter x column half)
        const int tid = threadIdx.x - 64;        // 0..255
        const int row = tid & 127, hf = tid >> 7;  // weight row of the tile, half of the slice
        const int tt = row >> 4, r = row & 15;
        for (int s = 0; s < ksteps && !s_abort; s++) {
            const int st = s % PF_STAGES, sb = s >> 2, rb = sb & 1, c = s & 3;
            if (c == 0 && !mbar_wait_bounded(&rec_full[rb], (uint32_t)(sb >> 1) & 1u)) {
                s_abort = 1;
                break;
            }
            if (s >= PF_STAGES && !mbar_wait_bounded(&empty[st], (uint32_t)((s / PF_STAGES) - 1) & 1u)) {
                s_abort = 1;
                break;
            }
            uint4 ch[4];
            const uint8_t *rec = sRec + ((size_t)rb * PF_TILES_N + tt) * REC;
            if constexpr (DT == 4) dequant_slice_q4k(rec, r, c, hf, ch);
            else dequant_slice_q6k(rec, r, c, hf, ch);
            uint8_t *brow = sB + st * PF_B_BYTES + row * 128;
#pragma unroll
            for (int qq = 0; qq < 4; qq++) {
                const int q = 4 * hf + qq;
                *reinterpret_cast<uint4 *>(brow + ((q ^ (row & 7)) << 4)) = ch[qq];
            }
            fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor cores
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&b_full[st]);
                if (c == 3) mbar_arrive(&rec_empty[rb]);
            }
        }
        if (!s_abort && mbar_wait_bounded(&acc_full, 0)) {
            tc_fence_after();
            const int q = warp & 3;                  // TMEM lane quarter of this warp
            const int h = (warp - 2) >> 2;           // accumulator: warps 2..5 -> rows 0..127, 6..9 -> 128..255
            const int orow = m0 + PF_MH * h + 32 * q + lane;
            const float sc = orow < T ? rowscale[orow] : 0.f;
#pragma unroll 1
            for (int cc = 0; cc < PF_BN / 32; cc++) {
                uint32_t v[32];
                tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + h * PF_BN + 32 * cc, v);
                if (orow < T) {
                    float *dst = Y + (int64_t)orow * N + (int64_t)n_tile * PF_BN + 32 * cc;
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4 *>(dst + i) =
                            make_float4(__fmul_rn(__uint_as_float(v[i]), sc), __fmul_rn(__uint_as_float(v[i + 1]), sc),
                                        __fmul_rn(__uint_as_float(v[i + 2]), sc),
                                        __fmul_rn(__uint_as_float(v[i + 3]), sc));
                }
            }
        } else {
            s_abort = 1;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (s_abort && threadIdx.x == 0) atomicOr(err, ERRBIT_WAIT_TIMEOUT);
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PF_TMEM_COLS)
                     : "memory");
    }
    pdl_launch();
}

// ---------------------------------------------------------------------------
// Two-pass form for long prompts.  The fused kernel above dequantizes each
// weight slice once per 256-token tile, i.e. T / 256 times per prompt; from
// T = 512 rows on, the weights are instead dequantized once (per chunk of
// rows, k_dequant_rows_f16: the same fp16 values dequant_slice_* feed the
// fused kernel's B operand) and multiplied by a plain fp16 tensor-core GEMM
// with TMA on both operands (k_gemm_f16).  Same operands, same MMA shape and
// k order: the two forms give the same bits.

// Wh[r][k] fp16 (r < rows, weight rows row0 + r) from the tile-major records.
// Thread (row, super-block b, 64-column slice c, half hf) writes 32 columns.
template <int DT>
__global__ void __launch_bounds__(256) k_dequant_rows_f16(const uint8_t *__restrict__ W, int64_t nb, int64_t row0,
                                                          int64_t rows, __half *__restrict__ Wh) {
    constexpr int REC = PfRec<DT>::bytes;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * nb * 8) return;
    const int hf = (int)(i & 1), c = (int)((i >> 1) & 3);
    const int64_t b = (i >> 3) % nb, rr = (i >> 3) / nb;
    const int64_t row = row0 + rr;
    const uint8_t *rec = W + ((size_t)(row >> 4) * nb + b) * REC;
    uint4 ch[4];
    if constexpr (DT == 4) dequant_slice_q4k(rec, (int)(row & 15), c, hf, ch);
    else dequant_slice_q6k(rec, (int)(row & 15), c, hf, ch);
    uint4 *dst = reinterpret_cast<uint4 *>(Wh + rr * (nb * 256) + b * 256 + 64 * c + 32 * hf);
#pragma unroll
    for (int qq = 0; qq < 4; qq++) dst[qq] = ch[qq];
}

constexpr int GM_BM = 256, GM_BK = 64;
constexpr uint32_t GM_A_BYTES = GM_BM * GM_BK * 2;  // 32 KB
constexpr int GM_EPI_WARPS = 4;
constexpr int GM_THREADS = 64 + 32 * GM_EPI_WARPS;
constexpr uint32_t GM_TMEM_COLS = 512;
// BN = 128: 4 stages of 48 KB, two accumulator sets (the epilogue of tile i
// overlaps the mainloop of tile i + 1); BN = 256: 3 stages of 64 KB, one
// accumulator set filling TMEM, half the L2 re-reads of X per output.
template <int BN> struct GmCfg {
    static constexpr uint32_t B_BYTES = BN * GM_BK * 2;
    static constexpr int STAGES = BN == 128 ? 4 : 3;
    static constexpr int NACC = (int)GM_TMEM_COLS / (2 * BN);
    static constexpr size_t SMEM = 1024 + (size_t)STAGES * (GM_A_BYTES + B_BYTES);
    // kind::f16 instruction descriptor: fp16 A / B, f32 D, K-major, M = 128, N = BN
    static constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(PF_MH >> 4) << 24);
};
static_assert(GmCfg<128>::SMEM <= 227 * 1024 && GmCfg<256>::SMEM <= 227 * 1024, "gemm stages must fit");


// Y[t, n_base + n] = rowscale[t] * sum_k Xh[t, k] Wh[n, k] for the chunk's
// rows n < BN * tiles_n.  Persistent: CTA b takes tiles b, b + grid, ...
// (tile = (n tile) * tiles_m + (m tile)); warp 0 issues the TMA loads of
// both operands into the stage ring, warp 1 the MMAs (two M = 128 halves of
// the 256-row tile per 16-wide k step) into TMEM, warps 2..5 drain a finished
// accumulator set (tcgen05.ld, row scale, f32 stores).  Every wait is bounded.
template <int BN>
__global__ void __launch_bounds__(GM_THREADS, 1)
    k_gemm_f16(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap, int T,
               int64_t ldy, int64_t n_base, int tiles_m, int tiles_n, int ksteps, const float *__restrict__ rowscale,
               float *__restrict__ Y, uint32_t *err) {
    using Cfg = GmCfg<BN>;
    constexpr int ST_N = Cfg::STAGES, NACC = Cfg::NACC;
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t full[ST_N], empty[ST_N], acc_full[NACC], acc_empty[NACC];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort_raw;
    volatile int &s_abort = s_abort_raw;
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sA = smem, *sB = smem + ST_N * GM_A_BYTES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = tiles_m * tiles_n;
    if (threadIdx.x == 0) {
        for (int i = 0; i < ST_N; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < NACC; i++) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], GM_EPI_WARPS);
        }
        mbar_fence_init();
        s_abort = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(GM_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == 0) {
        if (lane == 0) {
            long long s = 0;
            for (int t = blockIdx.x; t < tiles && !s_abort; t += gridDim.x) {
                const int m0 = (t % tiles_m) * GM_BM, n0 = (t / tiles_m) * BN;
                for (int k = 0; k < ksteps; k++, s++) {
                    const int st = (int)(s % ST_N);
                    if (s >= ST_N && !mbar_wait_bounded(&empty[st], (uint32_t)((s / ST_N) - 1) & 1u)) {
                        s_abort = 1;
                        break;
                    }
                    mbar_expect_tx(&full[st], GM_A_BYTES + Cfg::B_BYTES);
                    tma_load_2d(sA + st * GM_A_BYTES, &xmap, k * GM_BK, m0, &full[st]);
                    tma_load_2d(sB + st * Cfg::B_BYTES, &wmap, k * GM_BK, n0, &full[st]);
                }
            }
            // copies in flight land before shared memory is released
            for (long long k = s > ST_N ? s - ST_N : 0; k < s; k++)
                mbar_wait_bounded(&full[k % ST_N], (uint32_t)(k / ST_N) & 1u);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t aBase = smem_u32(sA), bBase = smem_u32(sB);
            long long s = 0;
            int li = 0;
            for (int t = blockIdx.x; t < tiles && !s_abort; t += gridDim.x, li++) {
                const int a = li % NACC;
                if (li >= NACC && !mbar_wait_bounded(&acc_empty[a], (uint32_t)((li / NACC) - 1) & 1u)) {
                    s_abort = 1;
                    break;
                }
                tc_fence_after();
                for (int k = 0; k < ksteps; k++, s++) {
                    const int st = (int)(s % ST_N);
                    if (!mbar_wait_bounded(&full[st], (uint32_t)(s / ST_N) & 1u)) {
                        s_abort = 1;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < GM_BK / 16; kk++) {
                        const uint64_t db = umma_desc_sw128(bBase + st * Cfg::B_BYTES + kk * 32);
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const uint64_t da = umma_desc_sw128(aBase + st * GM_A_BYTES + h * (PF_MH * 128) + kk * 32);
                            umma_f16_desc(tmem + a * (2 * BN) + h * BN, da, db, Cfg::IDESC, (k > 0 || kk > 0) ? 1u : 0u);
                        }
                    }
                    umma_commit(&empty[st]);  // frees the stage once these MMAs have read it
                }
                if (s_abort) break;
                umma_commit(&acc_full[a]);
            }
        }
    } else {
        // warps 2..5: TMEM lane quarter q = warp % 4 holds tile rows 32 q .. 32 q + 31 of each half
        const int q = warp & 3;
        int li = 0;
        for (int t = blockIdx.x; t < tiles && !s_abort; t += gridDim.x, li++) {
            const int a = li % NACC;
            const int m0 = (t % tiles_m) * GM_BM, n0 = (t / tiles_m) * BN;
            if (!mbar_wait_bounded(&acc_full[a], (uint32_t)(li / NACC) & 1u)) {
                s_abort = 1;
                break;
            }
            tc_fence_after();
#pragma unroll 1
            for (int h = 0; h < 2; h++) {
                const int orow = m0 + PF_MH * h + 32 * q + lane;
                const float sc = orow < T ? rowscale[orow] : 0.f;
#pragma unroll 1
                for (int cc = 0; cc < BN / 32; cc++) {
                    uint32_t v[32];
                    tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + a * (2 * BN) + h * BN + 32 * cc, v);
                    if (orow < T) {
                        float *dst = Y + (int64_t)orow * ldy + n_base + n0 + 32 * cc;
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4 *>(dst + i) = make_float4(
                                __fmul_rn(__uint_as_float(v[i]), sc), __fmul_rn(__uint_as_float(v[i + 1]), sc),
                                __fmul_rn(__uint_as_float(v[i + 2]), sc), __fmul_rn(__uint_as_float(v[i + 3]), sc));
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[a]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (s_abort && threadIdx.x == 0) atomicOr(err, ERRBIT_WAIT_TIMEOUT);
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(GM_TMEM_COLS)
                     : "memory");
    }
}

// X [T, K] f32 -> fp16 with a per-row power-of-two scale s (|x / s| <= 32768):
// one warp per row.
__global__ void __launch_bounds__(256) k_x_to_f16(const float *__restrict__ x, __half *__restrict__ xh,
                                                  float *__restrict__ rowscale, int T, int64_t K) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= T) return;
    const float *xr = x + (int64_t)row * K;
    float amax = 0.f;
#pragma unroll 4  // several row loads in flight per lane
    for (int64_t i = 4 * lane; i < K; i += 128) {
        const float4 v = *reinterpret_cast<const float4 *>(xr + i);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    int e = 0;  // smallest e >= 0 with amax / 2^e <= 32768
    while (e < 120 && amax > ldexpf(32768.f, e)) e++;
    const float inv = ldexpf(1.f, -e);
    if (lane == 0) rowscale[row] = ldexpf(1.f, e);
    __half *hr = xh + (int64_t)row * K;
#pragma unroll 4
    for (int64_t i = 4 * lane; i < K; i += 128) {
        const float4 v = *reinterpret_cast<const float4 *>(xr + i);
        const __half2 a = __floats2half2_rn(__fmul_rn(v.x, inv), __fmul_rn(v.y, inv));
        const __half2 b = __floats2half2_rn(__fmul_rn(v.z, inv), __fmul_rn(v.w, inv));
        *reinterpret_cast<uint2 *>(hr + i) =
            make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
    }
}


bool prefill_gemm_supported(const fb_qtensor *w, int64_t m) {
    return (w->dtype == FB_Q4_K || w->dtype == FB_Q6_K) && m >= 17 && w->n % PF_BN == 0 && w->k % QK == 0 &&
           m <= 0x7fffffff;
}

template <int DT>
static void launch_prefill_dt(fb_ctx *ctx, const fb_qtensor *w, const CUtensorMap &map, const float *rowscale,
                              float *y, int T) {
    const size_t smem = pf_smem_bytes<DT>();
    FB_CUDA(cudaFuncSetAttribute(k_prefill_gemm<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)(w->n / PF_BN), (unsigned)((T + PF_BM - 1) / PF_BM));
    k_prefill_gemm<DT><<<grid, PF_THREADS, smem, ctx->stream>>>(map, w->main(), w->nb(), T, w->n, rowscale, y,
                                                                 ctx->err_word);
    FB_CUDA(cudaGetLastError());
}

// fp16 row-major [rows][K] tensor map, boxes of 64 columns x box_rows rows, 128-byte swizzle.
static CUtensorMap f16_map(const __half *p, int64_t rows, int64_t K, uint32_t box_rows) {
    auto encode = tensor_map_encoder();
    FB_REQUIRE(encode != nullptr, "prefill gemm: cuTensorMapEncodeTiled is unavailable");
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {PF_BK, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult cr = encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(p), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    FB_REQUIRE(cr == CUDA_SUCCESS, "prefill gemm: tensor map encoding failed");
    return map;
}

// From this many rows on, the weights are dequantized once per prompt chunk
// (two-pass form) instead of once per 256-row tile.
constexpr int64_t PF_TWO_PASS_MIN_ROWS = 512;
// Weight rows dequantized per pass: at most 256 MB of fp16 (a whole Qwen3-8B
// projection; Llama-3-70B's gate/up in four passes), a multiple of 256.  (32
// MB passes, which stay in L2, left the Q6_K down projection 80 tiles for
// 148 SMs: slower.)
static int64_t two_pass_chunk_rows(int64_t n, int64_t K) {
    int64_t r = ((int64_t)256 << 20) / (K * 2);
    r = std::max<int64_t>(256, r / 256 * 256);
    return std::min(n, r);
}

// Y[m, n] = X[m, k] . W^T on the tensor cores (prefill_gemm_supported(w, m)).
// The fp16 copy of W kept for later prompt passes (prefill weight cache), made
// on the first long pass while max(16 GiB, a quarter of the device) stays
// free; null when the cache is off or the memory is not there.
static const __half *prefill_weight_cache(fb_ctx *ctx, const fb_qtensor *w) {
    fb_qtensor *mw = const_cast<fb_qtensor *>(w);  // the cache is a derived copy, not the tensor's value
    if (!ctx->prefill_cache) return nullptr;
    if (!mw->f16_tried) {
        mw->f16_tried = true;
        size_t free_b = 0, total_b = 0;
        FB_CUDA(cudaMemGetInfo(&free_b, &total_b));
        const size_t need = (size_t)w->n * w->k * 2;
        const size_t keep = std::max((size_t)16 << 30, total_b / 4);
        if (free_b > need && free_b - need > keep) {
            mw->f16.alloc(need);
            const int64_t nthr = w->n * w->nb() * 8;
            if (w->dtype == FB_Q4_K)
                k_dequant_rows_f16<4><<<(unsigned)((nthr + 255) / 256), 256, 0, ctx->stream>>>(
                    w->main(), w->nb(), 0, w->n, mw->f16.as<__half>());
            else
                k_dequant_rows_f16<6><<<(unsigned)((nthr + 255) / 256), 256, 0, ctx->stream>>>(
                    w->main(), w->nb(), 0, w->n, mw->f16.as<__half>());
            FB_CUDA(cudaGetLastError());
        }
    }
    return mw->f16.ptr ? mw->f16.as<__half>() : nullptr;
}

// Y = rowscale * (Xh . Wh^T) from fp16 rows Xh [m][K] and their power-of-two
// scales; wtmp: scratch for the weights' fp16 chunk (null: taken from the
// context's workspace, which must then not hold Xh).
static void prefill_gemm_impl(fb_ctx *ctx, const fb_qtensor *w, const __half *xh, const float *rowscale, float *y,
                              int64_t m, __half *wtmp) {
    const int64_t K = w->k, N = w->n;
    const bool two_pass = m >= PF_TWO_PASS_MIN_ROWS;
    const __half *wcache = two_pass ? prefill_weight_cache(ctx, w) : nullptr;
    const int64_t chunk = two_pass ? (wcache ? N : two_pass_chunk_rows(N, K)) : 0;
    if (two_pass && !wcache && !wtmp)
        wtmp = static_cast<__half *>(ctx->ensure_scratch((size_t)chunk * K * 2));
    if (!two_pass) {
        const CUtensorMap map = f16_map(xh, m, K, PF_BM);
        if (w->dtype == FB_Q4_K) launch_prefill_dt<4>(ctx, w, map, rowscale, y, (int)m);
        else launch_prefill_dt<6>(ctx, w, map, rowscale, y, (int)m);
        return;
    }
    __half *wh = wtmp;
    const CUtensorMap xmap = f16_map(xh, m, K, GM_BM);
    static std::once_flag once;
    std::call_once(once, [] {
        FB_CUDA(cudaFuncSetAttribute(k_gemm_f16<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)GmCfg<128>::SMEM));
        FB_CUDA(cudaFuncSetAttribute(k_gemm_f16<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)GmCfg<256>::SMEM));
    });
    const int tiles_m = (int)((m + GM_BM - 1) / GM_BM);
    for (int64_t r0 = 0; r0 < N; r0 += chunk) {
        const int64_t rows = std::min(chunk, N - r0);
        const int64_t nthr = rows * w->nb() * 8;
        if (wcache) {
            wh = const_cast<__half *>(wcache);  // (chunk = N: one pass over the cached copy)
        } else {
            if (w->dtype == FB_Q4_K)
                k_dequant_rows_f16<4><<<(unsigned)((nthr + 255) / 256), 256, 0, ctx->stream>>>(w->main(), w->nb(),
                                                                                              r0, rows, wh);
            else
                k_dequant_rows_f16<6><<<(unsigned)((nthr + 255) / 256), 256, 0, ctx->stream>>>(w->main(), w->nb(),
                                                                                              r0, rows, wh);
            FB_CUDA(cudaGetLastError());
        }
        // 256-column tiles (half the L2 re-reads of X per output) or 128-column
        // ones, whichever needs less time in whole waves of one tile per SM;
        // a 256-column tile is counted as 1.8 of the narrow ones (measured:
        // 948 vs ~700 TFLOP/s per tile-time on the Qwen3-8B gate/up shape)
        const int64_t waves128 = ((int64_t)tiles_m * (rows / 128) + ctx->num_sms - 1) / ctx->num_sms;
        const int64_t waves256 = ((int64_t)tiles_m * (rows / 256) + ctx->num_sms - 1) / ctx->num_sms;
        const bool wide = rows % 256 == 0 && 18 * waves256 < 10 * waves128;
        if (wide) {
            const CUtensorMap wmap = f16_map(wh, rows, K, 256);
            const int tiles_n = (int)(rows / 256);
            const int grid = std::min(tiles_m * tiles_n, ctx->num_sms);
            k_gemm_f16<256><<<grid, GM_THREADS, GmCfg<256>::SMEM, ctx->stream>>>(
                xmap, wmap, (int)m, N, r0, tiles_m, tiles_n, (int)(K / GM_BK), rowscale, y, ctx->err_word);
        } else {
            const CUtensorMap wmap = f16_map(wh, rows, K, 128);
            const int tiles_n = (int)(rows / 128);
            const int grid = std::min(tiles_m * tiles_n, ctx->num_sms);
            k_gemm_f16<128><<<grid, GM_THREADS, GmCfg<128>::SMEM, ctx->stream>>>(
                xmap, wmap, (int)m, N, r0, tiles_m, tiles_n, (int)(K / GM_BK), rowscale, y, ctx->err_word);
        }
        FB_CUDA(cudaGetLastError());
    }
}

void prefill_gemm(fb_ctx *ctx, const fb_qtensor *w, const float *x, float *y, int64_t m) {
    FB_REQUIRE(prefill_gemm_supported(w, m), "prefill gemm: unsupported shape");
    const int64_t K = w->k, N = w->n;
    const bool two_pass = m >= PF_TWO_PASS_MIN_ROWS;
    // the fp16 chunk of the weights shares the workspace with Xh: reserve it
    // unless a cached copy exists (a copy made by this call is allocated on
    // its own and leaves the reserved chunk unused)
    const bool cached = two_pass && ctx->prefill_cache && w->f16.ptr;
    const int64_t chunk = two_pass && !cached ? two_pass_chunk_rows(N, K) : 0;
    const size_t xh_bytes = ((size_t)m * K * 2 + 255) & ~(size_t)255;
    const size_t rs_bytes = ((size_t)m * 4 + 255) & ~(size_t)255;
    uint8_t *scratch = static_cast<uint8_t *>(ctx->ensure_scratch(xh_bytes + rs_bytes + (size_t)chunk * K * 2));
    __half *xh = reinterpret_cast<__half *>(scratch);
    float *rowscale = reinterpret_cast<float *>(scratch + xh_bytes);
    launch_x_to_f16(ctx, x, xh, rowscale, m, K);
    prefill_gemm_impl(ctx, w, xh, rowscale, y, m,
                      chunk ? reinterpret_cast<__half *>(scratch + xh_bytes + rs_bytes) : nullptr);
}

void prefill_gemm_x16(fb_ctx *ctx, const fb_qtensor *w, const __half *xh, const float *rowscale, float *y,
                      int64_t m) {
    FB_REQUIRE(prefill_gemm_supported(w, m), "prefill gemm: unsupported shape");
    prefill_gemm_impl(ctx, w, xh, rowscale, y, m, nullptr);
}

void launch_x_to_f16(fb_ctx *ctx, const float *x, __half *xh, float *rowscale, int64_t m, int64_t K) {
    k_x_to_f16<<<(unsigned)((m + 7) / 8), 256, 0, ctx->stream>>>(x, xh, rowscale, (int)m, K);
    FB_CUDA(cudaGetLastError());
}

}  // namespace fb
