// Format kernels: Q8_K activation quantization, GGUF <-> device re-layout of
// Q4_K / Q6_K weights, on-device random-init generator, and dequantization.
//
// Semantics follow the GGUF k-quant formats as the reference declares them
// (ferrite-os/crates/internal/ptx-kernels/kernels/candle/quantized.cu:388-432)
// and candle-core 0.8.4's CPU path (Q8_K activation quantizer of
// BlockQ8K::from_float; dequantization of quantized.cu:936-1129).  Every
// elementwise float step uses explicit round-to-nearest intrinsics so the
// results are bit-identical to the CPU arithmetic.
#include "fb_internal.h"
#include "kq_common.cuh"

namespace fb {

size_t q8act_bytes(int64_t m, int64_t k) {
    size_t qs = (size_t)(m * k);
    size_t d = (size_t)(m * (k / 256)) * 4;
    size_t b16 = (size_t)(m * (k / 16)) * 2;
    size_t b32 = (size_t)(m * (k / 32)) * 2;
    auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
    return up(qs) + up(d) + up(b16) + up(b32);
}

Q8Act q8act_view(void *base, int64_t m, int64_t k) {
    auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
    uint8_t *p = (uint8_t *)base;
    Q8Act a;
    a.k = k;
    a.qs = (int8_t *)p;
    p += up((size_t)(m * k));
    a.d = (float *)p;
    p += up((size_t)(m * (k / 256)) * 4);
    a.bs16 = (int16_t *)p;
    p += up((size_t)(m * (k / 16)) * 2);
    a.bs32 = (int16_t *)p;
    return a;
}

// ------------------------------------------------------------------------
// Q8_K quantization of one 256-value block by one warp.  Lane l owns values
// 8l..8l+7.  Matches BlockQ8K::from_float: the pivot is the first value of
// largest magnitude, iscale = -128 / pivot, q = min(127, round(iscale * x))
// (round half away from zero), d = 1 / iscale, bsums over groups of 16.
struct Q8Block {
    int8_t q[8];
    float d;
    int bs16;  // valid on even lanes (group of 16 = lanes 2g, 2g+1)
    int bs32;  // valid on lanes 4j (group of 32 = lanes 4j..4j+3)
};

__device__ __forceinline__ Q8Block q8k_warp_block(const float *xb, int lane) {
    float4 v0 = *reinterpret_cast<const float4 *>(xb + 8 * lane);
    float4 v1 = *reinterpret_cast<const float4 *>(xb + 8 * lane + 4);
    float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float amax = 0.f, piv = 0.f;
    int idx = 1 << 30;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        float a = fabsf(v[e]);
        if (amax < a) {
            amax = a;
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
    Q8Block r;
    int s = 0;
    if (amax == 0.f) {
#pragma unroll
        for (int e = 0; e < 8; e++) r.q[e] = 0;
        r.d = 0.f;
    } else {
        float iscale = __fdiv_rn(-128.f, piv);
#pragma unroll
        for (int e = 0; e < 8; e++) {
            int q = (int)roundf(__fmul_rn(iscale, v[e]));
            q = q > 127 ? 127 : q;
            r.q[e] = (int8_t)q;
            s += q;
        }
        r.d = __fdiv_rn(1.f, iscale);
    }
    int s16 = s + __shfl_xor_sync(0xffffffffu, s, 1);
    int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 2);
    r.bs16 = s16;
    r.bs32 = s32;
    return r;
}

__global__ void __launch_bounds__(256) k_quantize_q8k(const float *__restrict__ x, int64_t m, int64_t k,
                                                      Q8Act a) {
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t nbk = k / QK;
    const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (wid < m * nbk) {
        const int64_t row = wid / nbk, blk = wid % nbk;
        Q8Block b = q8k_warp_block(x + row * k + blk * QK, lane);
        // permuted position of values 8l..8l+7: 64*(l&3) + 8*(l>>2)
        int8_t *dst = a.qs + row * k + blk * QK + 64 * (lane & 3) + 8 * (lane >> 2);
        uint2 w;
        w.x = (uint32_t)(uint8_t)b.q[0] | ((uint32_t)(uint8_t)b.q[1] << 8) |
              ((uint32_t)(uint8_t)b.q[2] << 16) | ((uint32_t)(uint8_t)b.q[3] << 24);
        w.y = (uint32_t)(uint8_t)b.q[4] | ((uint32_t)(uint8_t)b.q[5] << 8) |
              ((uint32_t)(uint8_t)b.q[6] << 16) | ((uint32_t)(uint8_t)b.q[7] << 24);
        *reinterpret_cast<uint2 *>(dst) = w;
        if ((lane & 1) == 0) a.bs16[row * (k / 16) + blk * 16 + (lane >> 1)] = (int16_t)b.bs16;
        if ((lane & 3) == 0) a.bs32[row * (k / 32) + blk * 8 + (lane >> 2)] = (int16_t)b.bs32;
        if (lane == 0) a.d[row * nbk + blk] = b.d;
    }
    pdl_launch();
}

// GGUF block_q8_K (292 B: f32 d, int8 qs[256], int16 bsums[16]).
__global__ void __launch_bounds__(256) k_quantize_q8k_gguf(const float *__restrict__ x, int64_t m, int64_t k,
                                                           uint8_t *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t nbk = k / QK;
    const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (wid >= m * nbk) return;
    const int64_t row = wid / nbk, blk = wid % nbk;
    Q8Block b = q8k_warp_block(x + row * k + blk * QK, lane);
    uint8_t *ob = out + (size_t)wid * 292;
#pragma unroll
    for (int e = 0; e < 8; e++) ob[4 + 8 * lane + e] = (uint8_t)b.q[e];
    if ((lane & 1) == 0) {
        int16_t s = (int16_t)b.bs16;
        memcpy(ob + 260 + 2 * (lane >> 1), &s, 2);
    }
    if (lane == 0) memcpy(ob, &b.d, 4);
}

void launch_quantize_q8k(fb_ctx *ctx, const float *x, int64_t m, int64_t k, const Q8Act &a) {
    int64_t warps = m * (k / QK);
    unsigned grid = (unsigned)((warps + 7) / 8);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = ctx->pdl ? 1 : 0;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    FB_CUDA(cudaLaunchKernelEx(&cfg, k_quantize_q8k, x, m, k, a));
}

void launch_quantize_q8k_gguf(fb_ctx *ctx, const float *x, int64_t m, int64_t k, void *out) {
    int64_t warps = m * (k / QK);
    k_quantize_q8k_gguf<<<(unsigned)((warps + 7) / 8), 256, 0, ctx->stream>>>(x, m, k, (uint8_t *)out);
    FB_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------------
// GGUF <-> device re-layout, one thread per (row, super-block).
__global__ void k_repack_q4k(const uint32_t *__restrict__ src, uint8_t *__restrict__ dst, int64_t nblocks, int64_t nb) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    const uint32_t *s = src + i * 36;
    uint32_t *d = reinterpret_cast<uint32_t *>(dst + q4k_offset(i / nb, i % nb, nb));
#pragma unroll
    for (int w = 0; w < 4; w++) d[w] = s[w];
    // device word 4 + 8t + 2g + x  <-  GGUF qs word 8g + 2t + x
#pragma unroll
    for (int t = 0; t < 4; t++)
#pragma unroll
        for (int g = 0; g < 4; g++)
#pragma unroll
            for (int x = 0; x < 2; x++) d[4 + 8 * t + 2 * g + x] = s[4 + 8 * g + 2 * t + x];
}

__global__ void k_unpack_q4k(const uint8_t *__restrict__ src, uint32_t *__restrict__ dst, int64_t nblocks, int64_t nb) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    const uint32_t *s = reinterpret_cast<const uint32_t *>(src + q4k_offset(i / nb, i % nb, nb));
    uint32_t *d = dst + i * 36;
#pragma unroll
    for (int w = 0; w < 4; w++) d[w] = s[w];
#pragma unroll
    for (int t = 0; t < 4; t++)
#pragma unroll
        for (int g = 0; g < 4; g++)
#pragma unroll
            for (int x = 0; x < 2; x++) d[4 + 8 * g + 2 * t + x] = s[4 + 8 * t + 2 * g + x];
}

// Byte offset (within the 210-byte GGUF block) of the 4 bytes that device
// word w of quad lane t holds; w < 8: ql, w >= 8: qh.
__device__ __forceinline__ int q6k_src_off(int t, int w) {
    if (w < 8) {
        int h = w >> 2, j = (w >> 1) & 1, x = w & 1;
        return 64 * h + 32 * j + 8 * t + 4 * x;
    }
    int h = (w - 8) >> 1, x = (w - 8) & 1;
    return 128 + 32 * h + 8 * t + 4 * x;
}

__global__ void k_repack_q6k(const uint8_t *__restrict__ src, uint8_t *__restrict__ dev, int64_t nblocks,
                             int64_t nb) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    const int64_t row = i / nb, b = i % nb;
    const uint8_t *s = src + i * 210;
    uint32_t *d = reinterpret_cast<uint32_t *>(dev + q6k_offset(row, b, nb));
    for (int t = 0; t < 4; t++)
        for (int w = 0; w < 12; w++) {
            const uint8_t *p = s + q6k_src_off(t, w);
            d[12 * t + w] = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
        }
    for (int w = 0; w < 4; w++) {
        const uint8_t *p = s + 192 + 4 * w;
        d[48 + w] = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
    }
    *reinterpret_cast<uint16_t *>(dev + q6k_d_offset(row, b, nb)) = (uint16_t)(s[208] | (s[209] << 8));
}

__global__ void k_unpack_q6k(const uint8_t *__restrict__ dev, uint8_t *__restrict__ dst, int64_t nblocks,
                             int64_t nb) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    const int64_t row = i / nb, b = i % nb;
    uint8_t *o = dst + i * 210;
    const uint32_t *s = reinterpret_cast<const uint32_t *>(dev + q6k_offset(row, b, nb));
    for (int t = 0; t < 4; t++)
        for (int w = 0; w < 12; w++) {
            uint32_t v = s[12 * t + w];
            uint8_t *p = o + q6k_src_off(t, w);
            p[0] = v & 0xFF; p[1] = (v >> 8) & 0xFF; p[2] = (v >> 16) & 0xFF; p[3] = v >> 24;
        }
    for (int w = 0; w < 4; w++) {
        uint32_t v = s[48 + w];
        uint8_t *p = o + 192 + 4 * w;
        p[0] = v & 0xFF; p[1] = (v >> 8) & 0xFF; p[2] = (v >> 16) & 0xFF; p[3] = v >> 24;
    }
    const uint16_t d = *reinterpret_cast<const uint16_t *>(dev + q6k_d_offset(row, b, nb));
    o[208] = d & 0xFF;
    o[209] = d >> 8;
}

void launch_repack(fb_ctx *ctx, int dtype, int64_t n, int64_t k, const void *gguf, void *dev) {
    const int64_t nb = k / QK, nbl = n * nb;
    unsigned grid = (unsigned)((nbl + 255) / 256);
    if (dtype == FB_Q4_K) {
        k_repack_q4k<<<grid, 256, 0, ctx->stream>>>((const uint32_t *)gguf, (uint8_t *)dev, nbl, nb);
    } else if (dtype == FB_Q6_K) {
        k_repack_q6k<<<grid, 256, 0, ctx->stream>>>((const uint8_t *)gguf, (uint8_t *)dev, nbl, nb);
    } else {
        fail(FB_ERR_INVALID, "repack: unsupported dtype");
    }
    FB_CUDA(cudaGetLastError());
}

void launch_unpack(fb_ctx *ctx, int dtype, int64_t n, int64_t k, const void *dev, void *gguf) {
    const int64_t nb = k / QK, nbl = n * nb;
    unsigned grid = (unsigned)((nbl + 255) / 256);
    if (dtype == FB_Q4_K) {
        k_unpack_q4k<<<grid, 256, 0, ctx->stream>>>((const uint8_t *)dev, (uint32_t *)gguf, nbl, nb);
    } else if (dtype == FB_Q6_K) {
        k_unpack_q6k<<<grid, 256, 0, ctx->stream>>>((const uint8_t *)dev, (uint8_t *)gguf, nbl, nb);
    } else {
        fail(FB_ERR_INVALID, "unpack: unsupported dtype");
    }
    FB_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------------
// Random-init generator: splitmix64 finalizer over (seed, index).  The CPU
// oracle restates the same function (oracle/model.c) for parity checks.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t synth_hash(uint64_t seed_mixed, uint64_t idx) { return mix64(seed_mixed ^ idx); }
__device__ __forceinline__ float synth_unit(uint64_t h) { return (float)(h >> 40) * (1.0f / 16777216.0f); }

__global__ void k_synth_q4k(uint32_t *__restrict__ out, int64_t nblocks, uint64_t sm, uint16_t base) {
    int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    uint32_t *o = out + b * 36;
    uint64_t i0 = (uint64_t)b * 32u;
    for (int w = 0; w < 16; w++) {
        uint64_t h = synth_hash(sm, i0 + (uint64_t)w);
        o[4 + 2 * w] = (uint32_t)h;
        o[4 + 2 * w + 1] = (uint32_t)(h >> 32);
    }
    uint64_t hs = synth_hash(sm, i0 + 16u);
    uint8_t sb[12] = {0};
    for (int j = 0; j < 8; j++) {
        uint32_t sc = 32u + (uint32_t)((hs >> (5 * j)) & 31u);
        uint32_t mn = (sc * 15u + 8u) >> 4;
        if (j < 4) {
            sb[j] = (uint8_t)sc;
            sb[j + 4] = (uint8_t)mn;
        } else {
            sb[j + 4] = (uint8_t)((sc & 0x0F) | ((mn & 0x0F) << 4));
            sb[j - 4] |= (uint8_t)((sc >> 4) << 6);
            sb[j] |= (uint8_t)((mn >> 4) << 6);
        }
    }
    uint64_t hd = synth_hash(sm, i0 + 17u);
    uint16_t d = (uint16_t)(base + (uint16_t)(hd & 15u));
    uint16_t dmin = __half_as_ushort(__float2half_rn(__fmul_rn(8.0f, h2f(d))));
    o[0] = (uint32_t)d | ((uint32_t)dmin << 16);
    for (int i = 0; i < 3; i++)
        o[1 + i] = (uint32_t)sb[4 * i] | ((uint32_t)sb[4 * i + 1] << 8) | ((uint32_t)sb[4 * i + 2] << 16) |
                   ((uint32_t)sb[4 * i + 3] << 24);
}

__global__ void k_synth_q6k(uint8_t *__restrict__ out, int64_t nblocks, uint64_t sm, uint16_t base) {
    int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    uint8_t *o = out + b * 210;
    uint64_t i0 = (uint64_t)b * 32u;
    for (int w = 0; w < 24; w++) {  // ql (16 words) then qh (8 words)
        uint64_t h = synth_hash(sm, i0 + (uint64_t)w);
        for (int e = 0; e < 8; e++) o[8 * w + e] = (uint8_t)(h >> (8 * e));
    }
    for (int half = 0; half < 2; half++) {
        uint64_t h = synth_hash(sm, i0 + 24u + (uint64_t)half);
        for (int j = 0; j < 8; j++) o[192 + 8 * half + j] = (uint8_t)(48u + ((h >> (6 * j)) & 63u));
    }
    uint64_t hd = synth_hash(sm, i0 + 26u);
    uint16_t d = (uint16_t)(base + (uint16_t)(hd & 15u));
    o[208] = d & 0xFF;
    o[209] = d >> 8;
}

__global__ void k_synth_f32(float *__restrict__ out, int64_t n, uint64_t sm, float mean, float s3) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float u = synth_unit(synth_hash(sm, (uint64_t)i));
    out[i] = __fadd_rn(mean, __fmul_rn(s3, __fsub_rn(__fmul_rn(2.0f, u), 1.0f)));
}

static uint64_t host_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void launch_synth(fb_ctx *ctx, int dtype, int64_t nblocks, uint64_t seed, float sigma, void *gguf_out) {
    unsigned grid = (unsigned)((nblocks + 255) / 256);
    uint64_t sm = host_mix64(seed);
    if (dtype == FB_Q4_K) {
        uint16_t base = __half_as_ushort(__float2half_rn(sigma / 219.0f));
        k_synth_q4k<<<grid, 256, 0, ctx->stream>>>((uint32_t *)gguf_out, nblocks, sm, base);
    } else if (dtype == FB_Q6_K) {
        uint16_t base = __half_as_ushort(__float2half_rn(sigma / 1468.0f));
        k_synth_q6k<<<grid, 256, 0, ctx->stream>>>((uint8_t *)gguf_out, nblocks, sm, base);
    } else {
        fail(FB_ERR_INVALID, "synth: unsupported dtype");
    }
    FB_CUDA(cudaGetLastError());
}

void launch_synth_f32(fb_ctx *ctx, float *out, int64_t n, uint64_t seed, float mean, float stddev) {
    k_synth_f32<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(out, n, host_mix64(seed), mean,
                                                                        stddev * 1.7320508f);
    FB_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------------
// Dequantization from the device layouts; one warp per super-block, lane l
// produces values 8l..8l+7.
template <typename T> __device__ __forceinline__ T cvt_out(float v);
template <> __device__ __forceinline__ float cvt_out<float>(float v) { return v; }
template <> __device__ __forceinline__ __half cvt_out<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Values 8 lane .. 8 lane + 7 of super-block b of row `row` (f32, exact
// candle `to_float` arithmetic).
__device__ __forceinline__ void dq8_q4k(const uint8_t *__restrict__ w, int64_t row, int64_t b, int64_t nb, int lane,
                                        float (&v)[8]) {
    const uint8_t *blk = w + q4k_offset(row, b, nb);
    const uint32_t *hw = reinterpret_cast<const uint32_t *>(blk);
    Q4Scales s = q4k_unpack_scales(hw[1], hw[2], hw[3]);
    const float d = h2f((uint16_t)(hw[0] & 0xFFFF)), dmin = h2f((uint16_t)(hw[0] >> 16));
    // values 8l..8l+7 live in group g = l >> 3, half hi = (l >> 2) & 1,
    // positions l' = 8*(l & 3) + e inside the 32-value sub-block
    const int g = lane >> 3, hi = (lane >> 2) & 1, t = lane & 3;
    const int j = 2 * g + hi;
    const int sc = byte_of(j < 4 ? s.sc_lo : s.sc_hi, j & 3);
    const int mn = byte_of(j < 4 ? s.mn_lo : s.mn_hi, j & 3);
    const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
    const uint2 q = *reinterpret_cast<const uint2 *>(blk + 16 + 32 * t + 8 * g);
#pragma unroll
    for (int e = 0; e < 8; e++) {
        uint32_t word = e < 4 ? q.x : q.y;
        int nib = (int)((word >> (8 * (e & 3) + 4 * hi)) & 0xF);
        v[e] = __fsub_rn(__fmul_rn(d1, (float)nib), m1);
    }
}

__device__ __forceinline__ void dq8_q6k(const uint8_t *__restrict__ w, int64_t row, int64_t b, int64_t nb, int lane,
                                        float (&v)[8]) {
    const uint32_t *blk = reinterpret_cast<const uint32_t *>(w + q6k_offset(row, b, nb));
    const float d = h2f(*reinterpret_cast<const uint16_t *>(w + q6k_d_offset(row, b, nb)));
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const int i = 8 * lane + e;
        const int h = i >> 7, r = i & 127, p = r >> 5, l = r & 31;
        const int t = l >> 3, x = (l >> 2) & 1, e4 = l & 3;
        const uint32_t qlw = blk[12 * t + 4 * h + 2 * (p & 1) + x];
        const uint32_t qhw = blk[12 * t + 8 + 2 * h + x];
        const int lo = (int)((qlw >> (8 * e4 + 4 * (p >> 1))) & 0xF);
        const int hi2 = (int)((qhw >> (8 * e4 + 2 * p)) & 0x3);
        const int sc = sbyte_of(blk[48 + (i >> 6)], (i >> 4) & 3);
        v[e] = __fmul_rn(__fmul_rn(d, (float)sc), (float)((lo | (hi2 << 4)) - 32));
    }
}

template <typename T>
__global__ void __launch_bounds__(256) k_dequant_q4k(const uint8_t *__restrict__ w, int64_t nblocks, int64_t nb,
                                                     T *__restrict__ y) {
    const int lane = threadIdx.x & 31;
    const int64_t b = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (b >= nblocks) return;
    float v[8];
    dq8_q4k(w, b / nb, b % nb, nb, lane, v);
    T *out = y + b * QK + 8 * lane;
#pragma unroll
    for (int e = 0; e < 8; e++) out[e] = cvt_out<T>(v[e]);
}

template <typename T>
__global__ void __launch_bounds__(256) k_dequant_q6k(const uint8_t *__restrict__ w, int64_t nblocks, int64_t nb,
                                                     T *__restrict__ y) {
    const int lane = threadIdx.x & 31;
    const int64_t b = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (b >= nblocks) return;
    float v[8];
    dq8_q6k(w, b / nb, b % nb, nb, lane, v);
    T *out = y + b * QK + 8 * lane;
#pragma unroll
    for (int e = 0; e < 8; e++) out[e] = cvt_out<T>(v[e]);
}

// y[r] = f32(sum_i W[r, i] * x[i]) with the f32 dequantized weights and a
// binary64 accumulation: the float form of QMatMul for one activation row
// (candle's dequantize + float matmul; the oracle's or_qmatmul_f32).  One
// warp per weight row.
template <int DT>
__global__ void __launch_bounds__(256) k_gemv_float(const uint8_t *__restrict__ w, int64_t n, int64_t nb,
                                                    const float *__restrict__ x, float *__restrict__ y) {
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (r >= n) return;
    double acc8[8] = {0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0};  // one chain per lane value: short FMA chains
    // four super-blocks' small weight loads in flight per warp (the loop is
    // bound by their latency: one warp per row streams the matrix once)
#pragma unroll 4
    for (int64_t b = 0; b < nb; b++) {
        float v[8];
        if constexpr (DT == 4) dq8_q4k(w, r, b, nb, lane, v);
        else dq8_q6k(w, r, b, nb, lane, v);
        const float4 x0 = *reinterpret_cast<const float4 *>(x + b * QK + 8 * lane);
        const float4 x1 = *reinterpret_cast<const float4 *>(x + b * QK + 8 * lane + 4);
        const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int e = 0; e < 8; e++) acc8[e] = __fma_rn((double)v[e], (double)xv[e], acc8[e]);
    }
    double acc = 0.0;
#pragma unroll
    for (int e = 0; e < 8; e++) acc = __dadd_rn(acc, acc8[e]);
    acc = warp_sum64(acc);
    if (lane == 0) y[r] = __double2float_rn(acc);
}

void launch_gemv_float(fb_ctx *ctx, const fb_qtensor *w, const float *x, float *y) {
    const unsigned grid = (unsigned)((w->n + 7) / 8);
    if (w->dtype == FB_Q4_K) k_gemv_float<4><<<grid, 256, 0, ctx->stream>>>(w->main(), w->n, w->nb(), x, y);
    else if (w->dtype == FB_Q6_K) k_gemv_float<6><<<grid, 256, 0, ctx->stream>>>(w->main(), w->n, w->nb(), x, y);
    else fail(FB_ERR_INVALID, "gemv_float: weight dtype must be Q4_K or Q6_K");
    FB_CUDA(cudaGetLastError());
}

void launch_dequantize(fb_ctx *ctx, const fb_qtensor *t, void *out, int out_dtype) {
    const int64_t nb = t->nb(), nbl = t->n * nb;
    unsigned grid = (unsigned)((nbl + 7) / 8);
    cudaStream_t s = ctx->stream;
    if (t->dtype == FB_Q4_K) {
        if (out_dtype == FB_F32) k_dequant_q4k<float><<<grid, 256, 0, s>>>(t->main(), nbl, nb, (float *)out);
        else if (out_dtype == FB_F16) k_dequant_q4k<__half><<<grid, 256, 0, s>>>(t->main(), nbl, nb, (__half *)out);
        else if (out_dtype == FB_BF16)
            k_dequant_q4k<__nv_bfloat16><<<grid, 256, 0, s>>>(t->main(), nbl, nb, (__nv_bfloat16 *)out);
        else fail(FB_ERR_INVALID, "dequantize: out_dtype must be F32, F16 or BF16");
    } else if (t->dtype == FB_Q6_K) {
        if (out_dtype == FB_F32) k_dequant_q6k<float><<<grid, 256, 0, s>>>(t->main(), nbl, nb, (float *)out);
        else if (out_dtype == FB_F16) k_dequant_q6k<__half><<<grid, 256, 0, s>>>(t->main(), nbl, nb, (__half *)out);
        else if (out_dtype == FB_BF16)
            k_dequant_q6k<__nv_bfloat16><<<grid, 256, 0, s>>>(t->main(), nbl, nb, (__nv_bfloat16 *)out);
        else fail(FB_ERR_INVALID, "dequantize: out_dtype must be F32, F16 or BF16");
    } else if (t->dtype == FB_F32) {
        FB_REQUIRE(out_dtype == FB_F32, "dequantize: F32 tensor only to F32");
        FB_CUDA(cudaMemcpyAsync(out, t->main(), (size_t)(t->n * t->k) * 4, cudaMemcpyDeviceToDevice, s));
    } else {
        fail(FB_ERR_INVALID, "dequantize: unsupported tensor dtype");
    }
    FB_CUDA(cudaGetLastError());
}

}  // namespace fb
