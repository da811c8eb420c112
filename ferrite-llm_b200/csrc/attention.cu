// GQA flash-decode attention over a paged fp16 KV cache.
//
// Replaces the attention inside candle-transformers 0.8.4 quantized_llama
// (q.k^T / sqrt(hd) -> softmax_last_dim -> .v over an f32 KV cache that grows
// by concatenation; called from crates/ferrite-wasm-host/src/adapter.rs:
// 61-70) and the reference's own stub kernel
// crates/ferrite-core/kernels/flash_attention.cu:166-225 (f32, hd <= 64,
// never launched).
//
// B200 design (HBM-bound: 2 * ctx * n_kv * hd * 2 bytes per layer and token):
//  * split-K: CTA (kv head, split of 2 pages, sequence); every CTA of the
//    grid issues its K and V page copies at once with cp.async.bulk (TMA,
//    one 16 KB copy per page, no multicast) onto per-page mbarriers, so each
//    SM keeps >64 KB in flight;
//  * the G = n_heads / n_kv query heads of the kv head share each K/V row
//    read from shared memory;
//  * scores: lane owns 4 dims of hd, a 32-value butterfly reduce-scatter
//    turns (32/G tokens x G heads) per-lane partials into one full dot per
//    lane (31 shuffles per 32 dots);
//  * partial (max, sum, o) per split go to a scratch buffer; a combine kernel
//    merges the splits (log-sum-exp) and, fused into the model path,
//    quantizes the result to Q8_K for the output projection;
//  * dots, exponentials and sums run in binary64 with one rounding to f32
//    at the end, so the result equals the CPU oracle's single-pass softmax
//    bit for bit whatever the split layout.
// All mbarrier waits are bounded: on timeout the kernel raises
// ERRBIT_WAIT_TIMEOUT in the context's error word and returns.
#include <math.h>

#include <mutex>

#include "fb_internal.h"
#include "kq_common.cuh"

namespace fb {

constexpr int ATT_HD = 128;
constexpr int ATT_WARPS = 4;

__device__ __forceinline__ int seq_len_of(const AttnArgs &A, int b) {
    return A.seq_lens ? A.seq_lens[b] : A.pos[b] + 1;
}

__device__ __forceinline__ void q8k_store_warp_ext(const float (&v)[8], int lane, const Q8Act &a, int64_t row,
                                                   int64_t blk);

// One CTA per (kv head, page of the sequence, sequence).  Dynamic shared
// memory: K[page][hd] half, V[page][hd] half, q[G][hd] f32, s[G][page] f32,
// p[G][page] f64, red[ATT_WARPS][G][hd] f64.  The last CTA of each (sequence,
// kv head) to finish merges all pages' partials (fixed order) and writes the
// G heads' output (f32 and/or Q8_K); the per-(sequence, kv head) counters
// return to zero afterwards.
//
// Numerics (identical to the CPU oracle up to binary64 rounding):
//   s_t = f32(sum_e q_e * k_te in binary64) * scale
//   per page:  m = max_t s_t, p_t = exp64(s_t - m), l = sum p_t,
//              o = sum p_t v_t              (binary64)
//   merge:     M = max m, w = exp64(m - M), out = f32(sum w*o / sum w*l)
template <int G>
__global__ void __launch_bounds__(ATT_WARPS * 32) k_attn_decode(AttnArgs A, float *__restrict__ out_f32, Q8Act aq,
                                                                int use_q8, int *__restrict__ counters) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bars[2];  // K page, V page
    __shared__ int s_last;
    __shared__ double s_M[G], s_L[G];
    const int kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int P = A.page_size;
    // sequence lengths are inputs of the whole step (written before it began)
    const int len = seq_len_of(A, b);
    const int t0 = split * P;
    if (t0 >= len) {
        pdl_launch();
        return;
    }
    const int nsplit = (len + P - 1) / P;
    const int ntok = min(P, len - t0);
    __half *Ks = reinterpret_cast<__half *>(smem);
    __half *Vs = Ks + (size_t)P * ATT_HD;
    float *qs = reinterpret_cast<float *>(Vs + (size_t)P * ATT_HD);
    float *ss = qs + G * ATT_HD;
    double *ps = reinterpret_cast<double *>(ss + G * P);
    double *red = ps + G * P;
    const uint32_t page_bytes = (uint32_t)P * ATT_HD * 2;
    // the page holding the newest position is written by the preceding kernel
    const bool fresh = t0 + P >= len;
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_fence_init();
    }
    __syncthreads();
    int page = -1;
    if (tid == 0) {
        page = split < A.max_pages ? A.block_table[(int64_t)b * A.max_pages + split] : -1;
        if (page < 0 || page >= A.num_pages) {
            atomicOr(A.err, ERRBIT_BAD_PAGE);
            page = -1;
        }
    }
    auto issue = [&]() {
        if (page >= 0) {
            const size_t off = ((size_t)page * A.n_kv + kvh) * (size_t)P * ATT_HD;
            mbar_expect_tx(&bars[0], page_bytes);
            bulk_g2s(Ks, reinterpret_cast<const __half *>(A.kpool) + off, page_bytes, &bars[0]);
            mbar_expect_tx(&bars[1], page_bytes);
            bulk_g2s(Vs, reinterpret_cast<const __half *>(A.vpool) + off, page_bytes, &bars[1]);
        } else {
            // complete the phases without data (the error word is set)
            mbar_expect_tx(&bars[0], 0);
            mbar_expect_tx(&bars[1], 0);
        }
    };
    if (tid == 0 && !fresh) issue();  // older pages stream in before the wait
    pdl_wait();
    if (tid == 0 && fresh) issue();
    const float *qg = A.q + ((int64_t)b * A.n_heads + (int64_t)kvh * G) * ATT_HD;
    for (int i = tid; i < G * ATT_HD; i += blockDim.x) qs[i] = qg[i];
    __syncthreads();

    // ---- scores: warp w handles tokens [WT*w, WT*w + WT) of the page
    constexpr int TCH = 32 / G;  // tokens per reduce-scatter chunk
    const int WT = P / ATT_WARPS;
    const int tw0 = warp * WT;
    bool waited_ok = true;
    if (tw0 < ntok) {
        waited_ok = mbar_wait_bounded(&bars[0], 0);
        float qv[G][4];
#pragma unroll
        for (int g = 0; g < G; g++)
#pragma unroll
            for (int e = 0; e < 4; e++) qv[g][e] = qs[g * ATT_HD + 4 * lane + e];
        const int nch = WT > TCH ? WT / TCH : 1;
#pragma unroll 1
        for (int c = 0; c < nch; c++) {
            const int tc0 = tw0 + c * TCH;
            double v[32];
#pragma unroll
            for (int t = 0; t < TCH; t++) {
                const int tok = tc0 + t;  // rows past the page are masked below
                const uint2 kr = *reinterpret_cast<const uint2 *>(Ks + (size_t)tok * ATT_HD + 4 * lane);
                const float2 k01 = __half22float2(*reinterpret_cast<const __half2 *>(&kr.x));
                const float2 k23 = __half22float2(*reinterpret_cast<const __half2 *>(&kr.y));
#pragma unroll
                for (int g = 0; g < G; g++) {
                    // f32 x fp16 products are exact in binary64
                    double acc = __dmul_rn((double)qv[g][0], (double)k01.x);
                    acc = __fma_rn((double)qv[g][1], (double)k01.y, acc);
                    acc = __fma_rn((double)qv[g][2], (double)k23.x, acc);
                    acc = __fma_rn((double)qv[g][3], (double)k23.y, acc);
                    v[t * G + g] = acc;
                }
            }
            // butterfly reduce-scatter: lane l ends with the sum of index l
#pragma unroll
            for (int o = 16, n = 32; o > 0; o >>= 1, n >>= 1) {
                const bool up = (lane & o) != 0;
#pragma unroll
                for (int i = 0; i < n / 2; i++) {
                    const double send = up ? v[i] : v[i + n / 2];
                    const double keep = up ? v[i + n / 2] : v[i];
                    v[i] = __dadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
                }
            }
            const int t = lane / G, g = lane % G;
            const int tl = c * TCH + t, tok = tw0 + tl;
            if (tl < WT) ss[g * P + tok] = tok < ntok ? __fmul_rn(__double2float_rn(v[0]), A.scale) : -INFINITY;
        }
    }
    __syncthreads();
    // ---- per-head page max and p_t = exp(s_t - max) (warps take heads)
    double *ml = red;  // [G][2] before the P.V reduction reuses red
    for (int g = warp; g < G; g += ATT_WARPS) {
        float mx = -INFINITY;
        for (int t = lane; t < ntok; t += 32) mx = fmaxf(mx, ss[g * P + t]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        double sum = 0.0;
        for (int t = lane; t < P; t += 32) {
            const double pv = t < ntok ? exp64(__dsub_rn((double)ss[g * P + t], (double)mx)) : 0.0;
            ps[g * P + t] = pv;
            sum = __dadd_rn(sum, pv);
        }
        sum = warp_sum64(sum);
        if (lane == 0) {
            ml[2 * g] = (double)mx;
            ml[2 * g + 1] = sum;
        }
    }
    __syncthreads();
    double mls[G][2];
#pragma unroll
    for (int g = 0; g < G; g++) {
        mls[g][0] = ml[2 * g];
        mls[g][1] = ml[2 * g + 1];
    }
    __syncthreads();
    // ---- o = sum_t p_t * v_t; warp w over its tokens, lane owns 4 dims
    double o[G][4];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < 4; e++) o[g][e] = 0.0;
    if (tw0 < ntok) {
        waited_ok = mbar_wait_bounded(&bars[1], 0) && waited_ok;
        const int tend = min(tw0 + WT, ntok);
        for (int tok = tw0; tok < tend; tok++) {
            const uint2 vr = *reinterpret_cast<const uint2 *>(Vs + (size_t)tok * ATT_HD + 4 * lane);
            const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vr.x));
            const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vr.y));
#pragma unroll
            for (int g = 0; g < G; g++) {
                const double pg = ps[g * P + tok];
                o[g][0] = __dadd_rn(o[g][0], __dmul_rn(pg, (double)v01.x));
                o[g][1] = __dadd_rn(o[g][1], __dmul_rn(pg, (double)v01.y));
                o[g][2] = __dadd_rn(o[g][2], __dmul_rn(pg, (double)v23.x));
                o[g][3] = __dadd_rn(o[g][3], __dmul_rn(pg, (double)v23.y));
            }
        }
    }
    if (!waited_ok) {
        atomicOr(A.err, ERRBIT_WAIT_TIMEOUT);
        // let any copy still in flight land before shared memory is released
        mbar_wait_bounded(&bars[0], 0);
        mbar_wait_bounded(&bars[1], 0);
    }
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < 4; e++) red[(warp * G + g) * ATT_HD + 4 * lane + e] = o[g][e];
    __syncthreads();
    for (int i = tid; i < G * ATT_HD; i += blockDim.x) {
        const int g = i / ATT_HD, d = i % ATT_HD;
        double sum = 0.0;
#pragma unroll
        for (int w = 0; w < ATT_WARPS; w++) sum = __dadd_rn(sum, red[(w * G + g) * ATT_HD + d]);
        const int64_t hrow = ((int64_t)b * A.n_heads + (int64_t)kvh * G + g) * A.nsplit_max + split;
        A.part_o[hrow * ATT_HD + d] = sum;
        if (d == 0) {
            A.part_ml[2 * hrow] = mls[g][0];
            A.part_ml[2 * hrow + 1] = mls[g][1];
        }
    }
    // ---- the last page CTA of this (sequence, kv head) merges all pages
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        int *cnt = counters + (int64_t)b * A.n_kv + kvh;
        const int prev = atomicAdd(cnt, 1);
        s_last = prev == nsplit - 1;
        if (s_last) *cnt = 0;  // ready for the next step
    }
    __syncthreads();
    if (!s_last) {
        pdl_launch();
        return;
    }
    __threadfence();
    const int64_t hb0 = ((int64_t)b * A.n_heads + (int64_t)kvh * G) * A.nsplit_max;
    double *wts = reinterpret_cast<double *>(smem);  // [G][nsplit], reuses the K/V area
    for (int g = warp; g < G; g += ATT_WARPS) {
        const int64_t hb = hb0 + (int64_t)g * A.nsplit_max;
        double M = -INFINITY;
        for (int s2 = lane; s2 < nsplit; s2 += 32) M = fmax(M, __ldcg(&A.part_ml[2 * (hb + s2)]));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M = fmax(M, __shfl_xor_sync(0xffffffffu, M, off));
        double L = 0.0;
        for (int s2 = lane; s2 < nsplit; s2 += 32) {
            const double w = exp64(__dsub_rn(__ldcg(&A.part_ml[2 * (hb + s2)]), M));
            wts[g * nsplit + s2] = w;
            L = __dadd_rn(L, __dmul_rn(__ldcg(&A.part_ml[2 * (hb + s2) + 1]), w));
        }
        L = warp_sum64(L);
        if (lane == 0) {
            s_M[g] = M;
            s_L[g] = L;
        }
    }
    __syncthreads();
    float *vals = qs;  // [G][hd] outputs, reuses the q area
    // each thread owns G outputs (one per head: index tid + 128 g when hd =
    // 128 = blockDim); 16 pages of all G heads are loaded per batch so the L2
    // round trips overlap
    {
        const int d = tid;  // blockDim.x == ATT_HD
        double acc[G];
#pragma unroll
        for (int g = 0; g < G; g++) acc[g] = 0.0;
        constexpr int UB = G >= 8 ? 8 : 16;
        for (int s0 = 0; s0 < nsplit; s0 += UB) {
            double v[G][UB];
#pragma unroll
            for (int g = 0; g < G; g++)
#pragma unroll
                for (int u = 0; u < UB; u++)
                    v[g][u] = s0 + u < nsplit
                                  ? __ldcg(&A.part_o[(hb0 + (int64_t)g * A.nsplit_max + s0 + u) * ATT_HD + d])
                                  : 0.0;
#pragma unroll
            for (int g = 0; g < G; g++)
#pragma unroll
                for (int u = 0; u < UB; u++)
                    if (s0 + u < nsplit) acc[g] = __dadd_rn(acc[g], __dmul_rn(v[g][u], wts[g * nsplit + s0 + u]));
        }
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float val = __double2float_rn(__ddiv_rn(acc[g], s_L[g]));
            vals[g * ATT_HD + d] = val;
            if (out_f32) out_f32[((int64_t)b * A.n_heads + (int64_t)kvh * G + g) * ATT_HD + d] = val;
        }
    }
    if (use_q8) {
        __syncthreads();
        // G*hd values = G/2 Q8_K blocks of the [n_heads*hd] row
        for (int blk = warp; blk < G / 2; blk += ATT_WARPS) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = vals[blk * 256 + 8 * lane + e];
            q8k_store_warp_ext(v, lane, aq, b, (int64_t)kvh * G / 2 + blk);
        }
    }
    pdl_launch();
}

// (same arithmetic as the Q8_K store in ops.cu)
__device__ __forceinline__ void q8k_store_warp_ext(const float (&v)[8], int lane, const Q8Act &a, int64_t row,
                                                   int64_t blk) {
    float amax = 0.f, piv = 0.f;
    int idx = 1 << 30;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const float av = fabsf(v[e]);
        if (amax < av) {
            amax = av;
            piv = v[e];
            idx = 8 * lane + e;
        }
    }
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

size_t attn_smem_bytes(int G, int page_size) {
    const size_t P = (size_t)page_size;
    return 2 * P * ATT_HD * 2 + (size_t)G * ATT_HD * 4 + (size_t)G * P * 4 + (size_t)G * P * 8 +
           (size_t)ATT_WARPS * G * ATT_HD * 8;
}

// Paged decode attention with the page merge fused in.  `counters` holds
// batch * n_kv int32 that are zero on entry and zero again on exit.  out_f32
// and/or (aq != null, needs an even GQA group) receive the result.
void launch_attn_decode(fb_ctx *ctx, const AttnArgs &A, int batch, int max_seq_len, float *out_f32, const Q8Act *aq,
                        int *counters, bool pdl) {
    const int G = A.n_heads / A.n_kv;
    FB_REQUIRE(A.n_heads % A.n_kv == 0, "attn: n_heads must be a multiple of n_kv_heads");
    FB_REQUIRE(A.page_size == 32 || A.page_size == 64, "attn: page_size must be 32 or 64");
    FB_REQUIRE(!aq || G % 2 == 0, "attn: fused Q8_K output needs an even GQA group");
    const int nsplit = (max_seq_len + A.page_size - 1) / A.page_size;
    FB_REQUIRE(nsplit <= A.nsplit_max, "attn: max_seq_len exceeds the split scratch");
    const size_t smem = attn_smem_bytes(G, A.page_size);
    FB_REQUIRE((size_t)G * nsplit * 8 <= (size_t)2 * A.page_size * ATT_HD * 2,
               "attn: max_seq_len too long for the in-kernel page merge");
    dim3 grid(A.n_kv, nsplit, batch);
    Q8Act q = aq ? *aq : Q8Act{nullptr, nullptr, nullptr, nullptr, 0};
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    // older KV pages are read before griddepcontrol.wait: only valid when the
    // preceding kernel is one of this library's (the model's decode step)
    attr[0].val.programmaticStreamSerializationAllowed = (ctx->pdl && pdl) ? 1 : 0;
    cfg.gridDim = grid;
    cfg.blockDim = dim3(ATT_WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (G) {
#define FB_ATT_CASE(GG)                                                                                           \
    case GG:                                                                                                      \
        FB_CUDA(cudaFuncSetAttribute(k_attn_decode<GG>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
        FB_CUDA(cudaLaunchKernelEx(&cfg, k_attn_decode<GG>, A, out_f32, q, aq ? 1 : 0, counters));              \
        break;
        FB_ATT_CASE(1)
        FB_ATT_CASE(2)
        FB_ATT_CASE(4)
        FB_ATT_CASE(8)
#undef FB_ATT_CASE
    default:
        fail(FB_ERR_INVALID, "attn: GQA group size must be 1, 2, 4 or 8");
    }
}

// ---------------------------------------------------------------------------
// Allocation-free decode attention (fb_attn_decode_noalloc).
//
// fb_attn_decode takes its split-K scratch (partial sums and maxima of every
// split) from the context's workspace, which is grown with cudaMalloc and a
// stream synchronisation on first use.  Some callers cannot allow that: code
// running under a caching or pooled device allocator that forbids direct
// cudaMalloc/cudaFree (ferrite-os routes device allocations through its own
// TLSF pool), and latency-critical loops that must never take the implicit
// device synchronisation cudaMalloc/cudaFree may cause.  For them this entry
// point keeps the scratch in a fixed, file-scope device array instead.
//
// The array is a `static __device__` object: every GPU that loads the library
// holds it until the process exits.  Host code cannot use the array's name as
// a device address (it is a host-side stand-in), so its device address is
// looked up per device with cudaGetSymbolAddress, with that device current,
// the first time the entry point runs on it; that first call should therefore
// come before any stream capture.  All calls on a device share the one array:
// calls that overlap on the GPU (two streams, or two contexts of one device)
// race on it.  The partial sums need no clearing (every slot a call reads is
// written by the same call first); the page-merge counters at its start must
// be zero, so each call clears them (cudaMemsetAsync, no allocation).
constexpr size_t kAttnNoAllocScratchBytes = (size_t)4 << 20;  // 4 MiB
static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[kAttnNoAllocScratchBytes];

static void *noalloc_scratch_address(int device) {
    static std::mutex mu;
    static void *addr[128] = {nullptr};
    FB_REQUIRE(device >= 0 && device < 128, "attn_decode_noalloc: device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[device]) {
        int cur = 0;
        FB_CUDA(cudaGetDevice(&cur));
        if (cur != device) FB_CUDA(cudaSetDevice(device));
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
        if (cur != device) cudaSetDevice(cur);
        FB_CUDA(e);
        addr[device] = p;
    }
    return addr[device];
}

}  // namespace fb

extern "C" int fb_attn_decode_noalloc(fb_ctx *ctx, const float *q_dev, const void *k_pages_dev,
                                      const void *v_pages_dev, const int32_t *block_table_dev,
                                      const int32_t *seq_lens_dev, float *out_dev, int batch, int n_heads,
                                      int n_kv_heads, int head_dim, int page_size, int max_pages,
                                      int max_seq_len, float scale) {
    using namespace fb;
    return guarded([&] {
        FB_REQUIRE(ctx && q_dev && k_pages_dev && v_pages_dev && block_table_dev && seq_lens_dev && out_dev,
                   "null argument");
        FB_REQUIRE(head_dim == 128, "head_dim must be 128");
        FB_REQUIRE(page_size == 32 || page_size == 64, "page_size must be 32 or 64");
        FB_REQUIRE(batch >= 1 && n_heads >= 1 && n_kv_heads >= 1 && max_pages >= 1 && max_seq_len >= 1,
                   "bad shape");
        FB_REQUIRE(max_seq_len <= max_pages * page_size, "max_seq_len exceeds the block table");
        const int nsplit = (max_seq_len + page_size - 1) / page_size;
        const size_t cnt_bytes = ((size_t)batch * n_kv_heads * sizeof(int) + 255) & ~(size_t)255;
        const size_t need = (size_t)batch * n_heads * nsplit * (head_dim + 2) * sizeof(double) + cnt_bytes;
        if (need > kAttnNoAllocScratchBytes)
            fail(FB_ERR_INVALID, "attn_decode_noalloc: batch * n_heads * ceil(max_seq_len / page_size) * " +
                                     std::to_string((head_dim + 2) * sizeof(double)) + " bytes = " +
                                     std::to_string(need) + " (with the merge counters) exceeds the fixed " +
                                     std::to_string(kAttnNoAllocScratchBytes) + "-byte scratch");
        uint8_t *raw = static_cast<uint8_t *>(noalloc_scratch_address(ctx->device));
        int *counters = reinterpret_cast<int *>(raw);
        // the merge counters must start at zero; the partials need no clearing
        FB_CUDA(cudaMemsetAsync(counters, 0, cnt_bytes, ctx->stream));
        double *base = reinterpret_cast<double *>(raw + cnt_bytes);
        AttnArgs A{};
        A.q = q_dev;
        A.kpool = k_pages_dev;
        A.vpool = v_pages_dev;
        A.block_table = block_table_dev;
        A.seq_lens = seq_lens_dev;
        A.pos = nullptr;
        A.part_o = base;
        A.part_ml = base + (size_t)batch * n_heads * nsplit * head_dim;
        A.n_heads = n_heads;
        A.n_kv = n_kv_heads;
        A.page_size = page_size;
        A.max_pages = max_pages;
        A.num_pages = 0x7fffffff;
        A.nsplit_max = nsplit;
        A.scale = scale;
        A.err = ctx->err_word;
        launch_attn_decode(ctx, A, batch, max_seq_len, out_dev, nullptr, counters, false);
    });
}
