// Device-side helpers shared by the sm_100a kernels: PDL controls, cache-hinted
// loads, 8-bit integer MMA wrappers and the k-quant field decoders.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace fb {

constexpr int QK = 256;

// Programmatic dependent launch: wait for the preceding grid's results /
// allow the next grid to start its prologue.  Both are no-ops when the
// kernel was launched without the PDL attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Streaming weight loads: read once, keep out of L1.
__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint16_t ld_stream_u16(const void *p) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}
// Activation loads: shared by every warp of the grid, keep in L1.
__device__ __forceinline__ uint4 ld_act16(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// D = A(16x32 s8, row) * B(32x8 s8, col) + C, int32 accumulate.
__device__ __forceinline__ void mma_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---- shared memory, mbarriers and TMA bulk copies (no multicast) ----
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// The same copy, marked evict-first in L2: for data read once per step (the
// weight and KV-cache streams), so that it does not push the kernels' code,
// activations, norm gains and RoPE rows out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void bulk_g2s_stream(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                                uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// One wait attempt; the thread may be suspended in hardware for up to
// `suspend_ns` while the phase is incomplete (it resumes when the phase
// completes), so waiting warps do not compete for issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity, uint32_t suspend_ns = 0) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(suspend_ns)
        : "memory");
    return ok != 0;
}
// Bounded wait (~1 s of SM clock).  Returns false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity, 20000)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity, 100000)) {
        if (clock64() - t0 > 2000000000LL) return false;
    }
    return true;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// System-scope flag handoff between GPUs (tensor-parallel exchanges): the
// writer's release store orders everything that happened before it (the
// producer grid's peer stores included); the reader's acquire load orders
// its later reads after it.
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t *p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// 8-byte system-scope relaxed accesses (single-copy atomic when aligned):
// the words of the tensor-parallel exchange, written over NVLink.
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Waits until the sequence number at p reaches seq (wrap-safe compare);
// gives up after limit_ns and returns false.
template <bool SYS>
__device__ __forceinline__ bool wait_seq(const uint32_t *p, uint32_t seq, uint64_t limit_ns) {
    auto ld = [&] { return SYS ? ld_acquire_sys(p) : ld_acquire_gpu(p); };
    if ((int32_t)(ld() - seq) >= 0) return true;
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld() - seq) < 0) {
        if (globaltimer_ns() - t0 > limit_ns) return false;
        __nanosleep(100);
    }
    return true;
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// subsequent async-proxy (TMA) writes to the same shared memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Q4_K: 8 six-bit scales (sc) and mins (mn) packed as 4 bytes per word:
// sc_lo/hi hold j = 0..3 / 4..7, mn_lo/hi likewise (format of
// get_scale_min_k4 in the GGUF Q4_K block).
struct Q4Scales {
    uint32_t sc_lo, sc_hi, mn_lo, mn_hi;
};
__device__ __forceinline__ Q4Scales q4k_unpack_scales(uint32_t s0, uint32_t s1, uint32_t s2) {
    Q4Scales r;
    r.sc_lo = s0 & 0x3F3F3F3Fu;
    r.mn_lo = s1 & 0x3F3F3F3Fu;
    r.sc_hi = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
    r.mn_hi = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
    return r;
}
__device__ __forceinline__ int byte_of(uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xFFu); }
__device__ __forceinline__ int sbyte_of(uint32_t w, int i) { return (int)(int8_t)((w >> (8 * i)) & 0xFFu); }

// exp(x) in binary64: Cody-Waite reduction x = k ln2 + r (ln2 split into a
// 32-bit head and a tail), the degree-13 Taylor polynomial of e^r evaluated
// by Horner's rule with fused multiply-adds, and the scaling by 2^k done with
// one rounding (as C's ldexp).  The CPU oracle evaluates the same sequence.
__device__ __forceinline__ double exp64_pow2(int n) {  // 2^n, -1022 <= n <= 1023
    return __longlong_as_double((long long)(n + 1023) << 52);
}
__device__ __forceinline__ double exp64(double x) {
    if (x != x) return x;
    if (x > 709.5) return __longlong_as_double(0x7FF0000000000000LL);
    if (x < -745.5) return 0.0;
    const double k = rint(__dmul_rn(x, 1.4426950408889634));
    const double r = __dsub_rn(__dsub_rn(x, __dmul_rn(k, 0.6931471803691238)), __dmul_rn(k, 1.9082149292705877e-10));
    double p = 1.6059043836821613e-10;  // 1/13!
    p = __fma_rn(p, r, 2.08767569878681e-09);
    p = __fma_rn(p, r, 2.505210838544172e-08);
    p = __fma_rn(p, r, 2.755731922398589e-07);
    p = __fma_rn(p, r, 2.7557319223985893e-06);
    p = __fma_rn(p, r, 2.48015873015873e-05);
    p = __fma_rn(p, r, 0.0001984126984126984);
    p = __fma_rn(p, r, 0.001388888888888889);
    p = __fma_rn(p, r, 0.008333333333333333);
    p = __fma_rn(p, r, 0.041666666666666664);
    p = __fma_rn(p, r, 0.16666666666666666);
    p = __fma_rn(p, r, 0.5);
    p = __fma_rn(p, r, 1.0);
    p = __fma_rn(p, r, 1.0);
    const int ki = (int)k;
    if (ki >= -1022 && ki <= 1023) return __dmul_rn(p, exp64_pow2(ki));
    if (ki > 1023) return __dmul_rn(__dmul_rn(p, 2.0), exp64_pow2(ki - 1));
    return __dmul_rn(__dmul_rn(p, exp64_pow2(ki + 64)), 5.421010862427522e-20);  // subnormal: * 2^-64 rounds once
}

// silu(v) = v / (1 + exp(-v)), evaluated in binary64 and rounded once.
__device__ __forceinline__ float silu64(float v) {
    return __double2float_rn(__ddiv_rn((double)v, __dadd_rn(exp64(-(double)v), 1.0)));
}

// 1 / RMS factor of a row: sqrt(mean(x^2) + eps) from a binary64 sum of squares.
__device__ __forceinline__ float rms_of(double ss, int dim, float eps) {
    return __fsqrt_rn(__fadd_rn(__double2float_rn(__ddiv_rn(ss, (double)dim)), eps));
}

// Warp sum in binary64.
__device__ __forceinline__ double warp_sum64(double v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

// One 128-dim attention head held by a warp (lane owns dims 4 lane .. 4 lane
// + 3): optional per-head RMSNorm with gain `gw` (Qwen3 QK-norm), then RoPE
// with the position's cos / sin rows (64 entries): mode 0 rotates adjacent
// pairs (2i, 2i+1), mode 1 rotates (i, i + 64) (partner in lane ^ 16).
// QkHead holds this lane's gains and rotation factors; it depends only on
// weights and the position, so it can be loaded before the grid-dependency
// wait.
struct QkHead {
    float g[4], c[4], s[4];
    bool norm;
};
__device__ __forceinline__ QkHead qk_head_load(int lane, const float *gw, const float *ct, const float *st, int mode) {
    QkHead h;
    h.norm = gw != nullptr;
#pragma unroll
    for (int e = 0; e < 4; e++) {
        h.g[e] = gw ? gw[lane * 4 + e] : 1.f;
        const int d = lane * 4 + e;
        const int i = mode == 0 ? d >> 1 : (d < 64 ? d : d - 64);
        h.c[e] = ct[i];
        h.s[e] = st[i];
    }
    return h;
}
__device__ __forceinline__ void qk_head_apply(float (&v)[4], int lane, const QkHead &h, float eps, int mode) {
    if (h.norm) {
        double ss = 0.0;
#pragma unroll
        for (int e = 0; e < 4; e++) ss = __fma_rn((double)v[e], (double)v[e], ss);
        ss = warp_sum64(ss);
        const float m = rms_of(ss, 128, eps);
#pragma unroll
        for (int e = 0; e < 4; e++) v[e] = __fmul_rn(__fdiv_rn(v[e], m), h.g[e]);
    }
    if (mode == 0) {
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
            const float c = h.c[e], s = h.s[e], x0 = v[e], x1 = v[e + 1];
            v[e] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
            v[e + 1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        }
    } else {
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float other = __shfl_xor_sync(0xffffffffu, v[e], 16);
            const int d = lane * 4 + e;
            const float c = h.c[e], s = h.s[e];
            if (d < 64) v[e] = __fsub_rn(__fmul_rn(v[e], c), __fmul_rn(other, s));
            else v[e] = __fadd_rn(__fmul_rn(other, s), __fmul_rn(v[e], c));
        }
    }
}

}  // namespace fb
