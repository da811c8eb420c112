// Persistent decode step: one cooperative kernel runs every layer of a
// batch-1 decode step (the InferenceModel::forward of one token, reference
// crates/ferrite-core/src/generation.rs:187-195 with candle's quantized
// forward at crates/ferrite-wasm-host/src/adapter.rs:60-93) and the lm_head;
// the greedy argmax follows as a separate small kernel.
//
// Why: at batch 1 the step is a chain of ~290 dependent kernels whose
// launch / drain gaps and small latency-bound kernels (norms, SwiGLU, the
// attention's split merge) leave HBM idle for about half of the step.  Here
// one CTA per SM lives for the whole step and the phases of a layer are
// separated by grid barriers, while a producer warp per CTA streams the
// weight records and KV pages the CTA will consume -- in consumption order,
// across phase and layer boundaries -- into a ring of shared-memory stages
// with cp.async.bulk (TMA, no multicast).  Weights and older KV positions do
// not depend on activations, so the producer never waits for a barrier: while
// the consumers wait for one, the ring fills with the next phase's bytes.
//
// Per layer (consumer warps; every arrow is a grid barrier):
//   norm: x += y_down (previous layer; the embedding row at layer 0), RMSNorm
//         with a binary64 sum of squares and Q8_K of the whole row -- computed
//         redundantly by every CTA into its own shared memory
//   QKV GEMV (tile-major Q4_K/Q6_K records x Q8_K, dp4a, binary64 combine)
//   -> attention: (kv head, split) per CTA: QK-norm + RoPE of q and of the new
//         k / v (written into the paged fp16 cache), f32 scores in the fixed
//         slice order, binary64 online softmax and P.V, a fixed-order tree
//         merge of the warps, split partials merged by the last CTA of each
//         kv head into the Q8_K input of the output projection
//   -> O GEMV -> norm (x += y_o, redundant) -> gate/up GEMV
//   -> SwiGLU + Q8_K (one CTA per 256-value block) -> down GEMV ->
// Arithmetic is the multi-kernel decode step's (gemv.cu, attention.cu,
// ops.cu) value for value, so results equal the CPU oracle's.
//
// All waits are bounded: mbarrier waits (~1 s of SM clock) and grid barriers
// (2 s of %globaltimer).  A wait that runs out raises ERRBIT_WAIT_TIMEOUT in
// the context's error word and sets an abort flag that every other wait of
// the launch checks, so all CTAs leave; the producer lets its copies in
// flight land before its CTA exits.
#include <math.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "fb_internal.h"
#include "gemv_dp4a.cuh"
#include "kq_common.cuh"
#include "attn_unit.cuh"
#include "q8k_store.cuh"
#include "decode_step.h"

namespace fb {

constexpr int DS_NC = 8;                  // consumer warps
constexpr int DS_CT = 32 * DS_NC;         // consumer threads (named barrier 1)
constexpr int DS_THREADS = DS_CT + 32;    // + the producer warp
constexpr uint32_t DS_STAGE = 36864;      // ring stage: 16 Q4_K or 10 Q6_K records, or one 64-token KV chunk
constexpr int DS_MAXSTAGE = 6;
constexpr int DS_HD = 128, DS_CHUNK = 64, DS_UNIT = 16;
constexpr int DS_QPAD = 32;                                      // bytes between the staged K quarters
constexpr uint32_t DS_KQS = DS_CHUNK * DS_HD * 2 / 4 + DS_QPAD;  // staged K quarter stride (32 dims)
constexpr uint32_t DS_KREG = 4 * DS_KQS;                         // K part of a KV stage
constexpr uint32_t DS_KROW = 2 * DS_CHUNK;                       // bytes between consecutive dims
constexpr int DS_BT_CAP = 256;                                   // chunks one split may hold
constexpr int DS_SPLITS_MAX = 32;
constexpr int DS_NMAXP = 8;  // float4 of the residual row per consumer thread: hidden <= 8192
constexpr int DS_NMAXB = 4;  // 256-value blocks of the row per consumer warp: hidden <= 8192
static_assert(DS_KREG + DS_CHUNK * DS_HD * 2 <= DS_STAGE, "a KV chunk must fit a stage");
static_assert(16 * 2304 <= DS_STAGE && 10 * 3360 <= DS_STAGE, "records per stage");

// ---------------------------------------------------------------- helpers
__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, %0;" ::"n"(DS_CT) : "memory"); }
__device__ __forceinline__ void red_release_gpu(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ bool aborted(const DsArgs &A) { return *(volatile unsigned *)&A.sync[1] != 0u; }
__device__ __forceinline__ void raise_abort(const DsArgs &A, uint32_t bit) {
    atomicOr(A.err, bit);
    atomicExch(&A.sync[1], 1u);
}
// mbarrier wait bounded like mbar_wait_bounded, giving up early when the launch aborts.
__device__ __forceinline__ bool ds_wait(uint64_t *bar, uint32_t parity, const DsArgs &A) {
    if (mbar_try_wait(bar, parity, 20000)) return true;
    const long long t0 = clock64();
    int it = 0;
    while (!mbar_try_wait(bar, parity, 100000)) {
        if ((++it & 63) == 0 && aborted(A)) return false;
        if (clock64() - t0 > 2000000000LL) return false;
    }
    return true;
}
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void st_release_u32(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Grid barrier k (1-based) among the consumer threads of every CTA: one
// arrival per CTA on a counter; the CTA whose arrival completes barrier k
// publishes k on a separate line (sync[32]) that the others poll, so the
// pollers do not contend with the arrivals.
__device__ __forceinline__ bool grid_barrier(const DsArgs &A, unsigned k, int *s_ok) {
    cons_sync();
    if (threadIdx.x == 0) {
        int ok = 1;
        __threadfence();
        const unsigned old = atom_add_acq_rel(&A.sync[0], 1u);
        if (old == k * gridDim.x - 1) {
            st_release_u32(&A.sync[32], k);
        } else if (ld_acquire_u32(&A.sync[32]) < k) {
            const uint64_t t0 = globaltimer_ns();
            while (ld_acquire_u32(&A.sync[32]) < k) {
                if (aborted(A)) {
                    ok = 0;
                    break;
                }
                if (globaltimer_ns() - t0 > 2000000000ull) {
                    raise_abort(A, ERRBIT_WAIT_TIMEOUT);
                    ok = 0;
                    break;
                }
            }
        }
        *s_ok = ok;
    }
    cons_sync();
    return *s_ok != 0;
}
// binary64 sum over the consumer threads (fixed order: warps 0..NC-1)
__device__ __forceinline__ double cons_sum64(double v, double *sh) {
    v = warp_sum64(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    cons_sync();
    if (lane == 0) sh[warp] = v;
    cons_sync();
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < DS_NC; w++) t = __dadd_rn(t, sh[w]);
    return t;
}
// Q8_K of one 256-value block held one value per consumer thread (the
// arithmetic of q8k_store_block, with the consumer-only barrier).
__device__ __forceinline__ void q8k_store_block_cons(float v, const Q8Act &a, int64_t row, int64_t blk, float *shv,
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
    cons_sync();
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
    int s16 = q;
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, off);
    const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 16);
    const int64_t k = a.k;
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
    cons_sync();  // shv / shi are reused by the next block
}

// ------------------------------------------------- shared-memory layout
__host__ __device__ inline size_t ds_r16(size_t x) { return (x + 15) & ~(size_t)15; }
__host__ __device__ inline size_t ds_act_bytes(int64_t k) {
    return ds_r16((size_t)k) + ds_r16((size_t)(k / 256) * 4) + ds_r16((size_t)(k / 16) * 2) +
           ds_r16((size_t)(k / 32) * 2);
}
__device__ __forceinline__ Q8Act ds_act_view(uint8_t *base, int64_t k) {
    Q8Act a;
    a.qs = reinterpret_cast<int8_t *>(base);
    a.d = reinterpret_cast<float *>(base + ds_r16((size_t)k));
    a.bs16 = reinterpret_cast<int16_t *>(base + ds_r16((size_t)k) + ds_r16((size_t)(k / 256) * 4));
    a.bs32 = reinterpret_cast<int16_t *>(base + ds_r16((size_t)k) + ds_r16((size_t)(k / 256) * 4) +
                                         ds_r16((size_t)(k / 16) * 2));
    a.k = k;
    return a;
}
// attention scratch (G heads per kv head)
__host__ __device__ constexpr int ds_qidx(int d, int g, int G) { return (d + (d >> 5)) * G + g; }
struct DsAttLayout {
    size_t q, ss, pb, tree, mw, lw, wt, wts, wl, mmax, fin, newkv, total;
};
__host__ __device__ inline DsAttLayout ds_att_layout(int G) {
    DsAttLayout L;
    size_t off = 0;
    L.q = off;
    off += ds_r16((size_t)(DS_HD + 4) * G * 4);
    L.ss = off;
    off += ds_r16((size_t)DS_NC * DS_UNIT * G * 4);
    L.pb = off;
    off += ds_r16((size_t)DS_NC * DS_UNIT * G * 8);
    L.tree = off;  // [NC/2][G][hd] f64 + [NC/2][G] f64 sums
    off += ds_r16((size_t)(DS_NC / 2) * G * (DS_HD + 1) * 8);
    L.mw = off;
    off += ds_r16((size_t)DS_NC * G * 8);
    L.lw = off;
    off += ds_r16((size_t)DS_NC * G * 8);
    L.wt = off;
    off += ds_r16((size_t)DS_NC * G * 8);
    L.wts = off;
    off += ds_r16((size_t)G * DS_SPLITS_MAX * 8);
    L.wl = off;
    off += ds_r16((size_t)G * DS_SPLITS_MAX * 8);
    L.mmax = off;
    off += ds_r16((size_t)G * 8);
    L.fin = off;
    off += ds_r16((size_t)G * DS_HD * 4);
    L.newkv = off;
    off += ds_r16((size_t)2 * DS_HD * 2);
    L.total = off;
    return L;
}
struct DsLayout {
    size_t ring, act, uni, red, total;
};
__host__ __device__ inline DsLayout ds_layout(int nstage, int64_t kmax, int H, int G) {
    DsLayout L;
    size_t off = 0;
    L.ring = off;
    off += (size_t)nstage * DS_STAGE;
    L.act = off;
    off += ds_act_bytes(kmax);
    L.uni = off;  // norm: x row [H] f32; attention: DsAttLayout
    const size_t att = ds_att_layout(G).total, nrm = ds_r16((size_t)H * 4);
    off += att > nrm ? att : nrm;
    L.red = off;  // GEMV tile partials [nstage + 1][NC][16] f64
    off += (size_t)(nstage + 1) * DS_NC * 16 * 8;
    L.total = ds_r16(off);
    return L;
}

// -------------------------------------------------------- the schedule
// Both roles walk the same sequence of ring stages: per layer the CTA's
// tiles of the QKV weight (each tile's records in pieces of at most a
// stage), its attention chunks, then its tiles of wo, gate/up and down; after
// the layers its tiles of the lm_head.  A CTA's tiles of a weight with
// n_tiles tiles are T = cta, cta + grid, ...
__host__ __device__ constexpr int ds_rec_bytes(int dt) { return dt == 4 ? 2304 : 3360; }
__host__ __device__ constexpr int ds_rps(int dt) { return dt == 4 ? 16 : 10; }  // records per stage

struct AttItem {
    int kvh, split, len, first, mine, jf;  // mine = chunks; jf = chunk (relative) holding the newest token
};

// ------------------------------------------------------------ producer
// A cursor over the CTA's stages in consumption order; next() describes the
// stage at the cursor (its copies) and advances.  The producer walks two
// cursors over the same sequence: one issues the shared-memory copies (and
// waits for ring slots), the other runs up to DS_L2_AHEAD bytes ahead of it
// issuing L2 prefetches, so HBM keeps streaming while the ring is full and
// the consumers wait on a grid barrier or a latency chain.
constexpr uint32_t DS_L2_AHEAD = 384 * 1024;
struct StageDesc {
    const uint8_t *src[5];
    uint32_t dst[5], bytes[5];
    int n;
    uint32_t total;
};
struct Cursor {
    int l = 0, ph = 0, T = -1, b0 = 0, j = 0;
    bool done = false;
};
__device__ __forceinline__ bool ds_gemv_phase(const DsArgs &A, int l, int ph, const uint8_t *&W, int &dt, int &n_rows,
                                              int &k) {
    if (l == A.n_layers) {
        if (ph != 0) return false;
        W = A.out, dt = A.dt_out, n_rows = A.vocab, k = A.H;
        return true;
    }
    const DsLayer &Ly = A.layers[l];
    switch (ph) {
    case 0: W = Ly.qkv, dt = Ly.dt_qkv, n_rows = A.qkv_n, k = A.H; return true;
    case 2: W = Ly.o, dt = Ly.dt_o, n_rows = A.H, k = A.n_heads * DS_HD; return true;
    case 3: W = Ly.gu, dt = Ly.dt_gu, n_rows = 2 * A.F, k = A.H; return true;
    case 4: W = Ly.down, dt = Ly.dt_down, n_rows = A.H, k = A.F; return true;
    default: return false;
    }
}
// Fills d with the stage at c and advances c; false at the end of the step.
__device__ bool ds_next(const DsArgs &A, const AttItem &it, const int *bt, Cursor &c, StageDesc &d) {
    while (!c.done) {
        if (c.l > A.n_layers || (c.l == A.n_layers && c.ph > 0)) {
            c.done = true;
            return false;
        }
        if (c.ph == 1) {  // attention chunks of this layer
            if (c.j < it.mine) {
                const uint32_t pbytes = DS_CHUNK * DS_HD * 2;
                const int page = bt[c.j];
                d.n = 0;
                d.total = 0;
                if (page >= 0) {
                    const __half *kpool = A.kv + (size_t)c.l * 2 * A.kv_layer, *vpool = kpool + A.kv_layer;
                    const size_t off = ((size_t)page * A.n_kv + it.kvh) * (size_t)DS_CHUNK * DS_HD;
                    for (int q = 0; q < 4; q++) {
                        d.src[q] = reinterpret_cast<const uint8_t *>(kpool + off) + q * (pbytes / 4);
                        d.dst[q] = q * DS_KQS;
                        d.bytes[q] = pbytes / 4;
                    }
                    d.src[4] = reinterpret_cast<const uint8_t *>(vpool + off);
                    d.dst[4] = DS_KREG;
                    d.bytes[4] = pbytes;
                    d.n = 5;
                    d.total = 2 * pbytes;
                }
                c.j++;
                return true;
            }
            c.ph = 2;
            c.T = -1;
            continue;
        }
        const uint8_t *W;
        int dt, n_rows, k;
        if (!ds_gemv_phase(A, c.l, c.ph, W, dt, n_rows, k)) {
            c.done = true;
            return false;
        }
        const int nb = k / QK, rec = ds_rec_bytes(dt), rps = ds_rps(dt), nt = (n_rows + 15) / 16;
        if (c.T < 0) {
            c.T = blockIdx.x;
            c.b0 = 0;
        }
        if (c.T < nt) {
            const int n = min(rps, nb - c.b0);
            d.src[0] = W + ((size_t)c.T * nb + c.b0) * rec;
            d.dst[0] = 0;
            d.bytes[0] = (uint32_t)(n * rec);
            d.n = 1;
            d.total = d.bytes[0];
            c.b0 += rps;
            if (c.b0 >= nb) {
                c.b0 = 0;
                c.T += gridDim.x;
            }
            return true;
        }
        // next phase
        c.T = -1;
        if (c.l == A.n_layers) {
            c.done = true;
            return false;
        }
        if (c.ph == 0) {
            c.ph = 1;
            c.j = 0;
        } else if (c.ph == 4) {
            c.l++;
            c.ph = 0;
        } else {
            c.ph++;
        }
    }
    return false;
}

__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// The producer lane: every stage of the step, in order.
__device__ void ds_produce(const DsArgs &A, const AttItem &it, const int *bt, uint8_t *ring, uint64_t *full,
                           uint64_t *empty) {
    const int nstage = A.nstage;
    Cursor cs, cp;
    StageDesc d, dp;
    long long s = 0;
    unsigned long long issued = 0, ahead = 0;  // bytes through the smem / L2 cursors
    unsigned long long blocked = 0;            // ns spent waiting for ring slots (timeline only)
    bool ok = true;
    while (ok && ds_next(A, it, bt, cs, d)) {
        // keep the L2 cursor DS_L2_AHEAD bytes ahead of this stage
        while (ahead < issued + d.total + DS_L2_AHEAD && ds_next(A, it, bt, cp, dp)) {
            for (int i = 0; i < dp.n; i++) prefetch_l2(dp.src[i], dp.bytes[i]);
            ahead += dp.total;
        }
        const int slot = (int)(s % nstage);
        if (s >= nstage) {
            const uint64_t t0 = A.trace ? globaltimer_ns() : 0;
            ok = ds_wait(&empty[slot], (uint32_t)((s / nstage - 1) & 1), A);
            if (A.trace) blocked += globaltimer_ns() - t0;
        }
        if (!ok) break;
        mbar_expect_tx(&full[slot], d.total);  // (0 bytes: completes the phase, the stage holds no data)
        uint8_t *dst = ring + (size_t)slot * DS_STAGE;
        for (int i = 0; i < d.n; i++) bulk_g2s(dst + d.dst[i], d.src[i], d.bytes[i], &full[slot]);
        issued += d.total;
        s++;
    }
    if (!ok) atomicExch(&A.sync[1], 1u);
    if (A.trace) {
        unsigned long long *row = A.trace + ((size_t)blockIdx.x * (A.n_layers + 1) + A.n_layers) * DS_TRACE_SLOTS;
        row[2] = blocked;
        row[3] = (unsigned long long)s;
        row[5] = issued;
    }
    // the copies still in flight land before the CTA exits
    for (long long k = max(0LL, s - nstage); k < s; k++) mbar_wait_bounded(&full[k % nstage], (uint32_t)((k / nstage) & 1));
}

// ------------------------------------------------------------ consumers
template <int G>
struct AttRegs {
    static constexpr int GH = G >= 2 ? G / 2 : 1;
    float m_run[G];
    double o[G][4], Lw[G];
};

// One 16-token unit of a staged 64-token chunk (the unit loop body of
// k_attn_decode: f32 scores in eight 16-dim FMA slices summed in slice
// order, then the unit's f32 softmax partial folded into the warp's binary64
// state, attn_unit.cuh; lane = 4 dims).
template <int G>
__device__ __forceinline__ void ds_att_unit(const uint8_t *kst, const __half *Vs, int qu, int nt, const float *q_s,
                                            float *ssw, float *pbw, float scale, int lane, AttRegs<G> &R) {
    constexpr unsigned FULL = 0xffffffffu;
    const int ti = lane & 7, qq4 = lane >> 3;
    float acc[2][2][G];
#pragma unroll
    for (int sl = 0; sl < 2; sl++)
#pragma unroll
        for (int t = 0; t < 2; t++)
#pragma unroll
            for (int g = 0; g < G; g++) acc[sl][t][g] = 0.f;
    {
        const int tc = DS_UNIT * qu + 2 * ti;
        const uint8_t *kp = kst + qq4 * DS_KQS + tc * 2;
        const float *qw = q_s + ds_qidx(32 * qq4, 0, G);
#pragma unroll
        for (int e = 0; e < 16; e++) {
#pragma unroll
            for (int sl = 0; sl < 2; sl++) {
                const int r = 16 * sl + e;
                const float2 k2 = __half22float2(*reinterpret_cast<const __half2 *>(kp + r * DS_KROW));
                float qv[G];
#pragma unroll
                for (int g = 0; g < G; g++) qv[g] = qw[r * G + g];
#pragma unroll
                for (int g = 0; g < G; g++) {
                    acc[sl][0][g] = __fmaf_rn(qv[g], k2.x, acc[sl][0][g]);
                    acc[sl][1][g] = __fmaf_rn(qv[g], k2.y, acc[sl][1][g]);
                }
            }
        }
    }
    float T[2][G];
#pragma unroll
    for (int t = 0; t < 2; t++)
#pragma unroll
        for (int g = 0; g < G; g++) T[t][g] = __fadd_rn(acc[0][t][g], acc[1][t][g]);
#pragma unroll
    for (int q = 1; q < 4; q++)
#pragma unroll
        for (int t = 0; t < 2; t++)
#pragma unroll
            for (int g = 0; g < G; g++) {
                const float x = __shfl_sync(FULL, T[t][g], ti + 8 * (q - 1));
                if (qq4 == q) T[t][g] = __fadd_rn(__fadd_rn(x, acc[0][t][g]), acc[1][t][g]);
            }
    float mx[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        const float s0 = 2 * ti < nt ? __fmul_rn(T[0][g], scale) : -INFINITY;
        const float s1 = 2 * ti + 1 < nt ? __fmul_rn(T[1][g], scale) : -INFINITY;
        if (qq4 == 3) {
            ssw[(2 * ti) * G + g] = s0;
            ssw[(2 * ti + 1) * G + g] = s1;
        }
        mx[g] = fmaxf(s0, s1);
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) mx[g] = fmaxf(mx[g], __shfl_xor_sync(FULL, mx[g], off));
        mx[g] = __shfl_sync(FULL, mx[g], 24);
    }
    __syncwarp();
    att_unit_fold<G>(ssw, pbw, Vs + (size_t)(DS_UNIT * qu) * DS_HD + 4 * lane, nt, mx, lane, R.m_run, R.Lw, R.o);
    __syncwarp();
}

// (the Q8_K store of attention.cu's merge: one warp per 256-value block)
__device__ __forceinline__ void ds_q8k_warp(const float (&v)[8], int lane, const Q8Act &a, int64_t row, int64_t blk) {
    q8k_store_warp(v, lane, a, row, blk);
}

template <int G>
struct Ds {
    const DsArgs &A;
    uint8_t *smem;
    DsLayout L;
    uint64_t *full, *empty;
    int *tcnt;
    int *s_ok;
    long long s = 0;  // stages consumed
    int tiles = 0;    // GEMV tiles finished by this CTA (reduction slot)
    int warp, lane, tid;
    bool ok = true;

    __device__ Ds(const DsArgs &a, uint8_t *sm, const DsLayout &l, uint64_t *f, uint64_t *e, int *tc, int *sok)
        : A(a), smem(sm), L(l), full(f), empty(e), tcnt(tc), s_ok(sok) {
        tid = threadIdx.x;
        warp = tid >> 5;
        lane = tid & 31;
    }
    unsigned long long wait_ns = 0;  // time this warp spent waiting for stages (timeline only)
    __device__ __forceinline__ const uint8_t *wait_stage() {
        const int slot = (int)(s % A.nstage);
        const uint64_t t0 = A.trace ? globaltimer_ns() : 0;
        if (ok && !ds_wait(&full[slot], (uint32_t)((s / A.nstage) & 1), A)) {
            ok = false;
            if (lane == 0) raise_abort(A, ERRBIT_WAIT_TIMEOUT);
        }
        if (A.trace) wait_ns += globaltimer_ns() - t0;
        return smem + L.ring + (size_t)slot * DS_STAGE;
    }
    __device__ __forceinline__ void release_stage() {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s % A.nstage]);
        s++;
    }
    // y[row] for the CTA's tiles of W[n_rows, k] against the Q8_K row in act.
    __device__ void gemv(const uint8_t *W, int dt, int n_rows, int k, const Q8Act &act, float *y) {
        const int nb = k / QK, rec = ds_rec_bytes(dt), rps = ds_rps(dt);
        const int nt = (n_rows + 15) / 16;
        double *red = reinterpret_cast<double *>(smem + L.red);
        const int nslot = A.nstage + 1;
        for (int T = blockIdx.x; T < nt; T += gridDim.x) {
            double acc[1] = {0.0};
            const int64_t row0 = (int64_t)T * 16;
            for (int b0 = 0; b0 < nb; b0 += rps) {
                const int n = min(rps, nb - b0);
                const uint8_t *st = wait_stage();
                if (ok) {
                    for (int i = warp; i < n; i += DS_NC) {
                        if (dt == 4)
                            q4k_block_dp4a<1, false>(st + (size_t)i * rec, act, b0 + i, nb, lane, row0, n_rows, acc,
                                                     nullptr, nullptr);
                        else
                            q6k_block_dp4a<1, false>(st + (size_t)i * rec, act, b0 + i, nb, lane, row0, n_rows, acc,
                                                     nullptr);
                    }
                }
                release_stage();
            }
            // the tile's partials: the last warp to arrive sums them in warp order
            const int slot = tiles % nslot;
            tiles++;
            double *rs = red + (size_t)slot * DS_NC * 16;
            if (lane < 16) rs[warp * 16 + lane] = acc[0];
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                __threadfence_block();
                last = atomicAdd(&tcnt[slot], 1) == DS_NC - 1;
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence_block();
                if (lane < 16 && ok) {
                    const volatile double *vr = rs;
                    double sum = 0.0;
#pragma unroll
                    for (int w = 0; w < DS_NC; w++) sum = __dadd_rn(sum, vr[w * 16 + lane]);
                    if (row0 + lane < n_rows) y[row0 + lane] = __double2float_rn(sum);
                }
                __syncwarp();
                if (lane == 0) tcnt[slot] = 0;
            }
        }
    }
    // Residual add + RMSNorm + Q8_K of the whole row, redundantly in every CTA,
    // in two parts so that everything independent of the preceding phase is
    // in flight before its grid barrier: norm_load issues the loads of the
    // residual x (written two or more barriers earlier) and of this lane's
    // gains; norm_finish (after the barrier) adds the projection output,
    // sums the squares in binary64, writes the CTA's slice of x to xout and
    // quantizes x / rms * g into the shared-memory act.  embed: x is the
    // dequantized embedding row of the step's token instead.
    struct NormIn {
        float4 x[DS_NMAXP];
        const float *g;
    };
    __device__ __forceinline__ void norm_load(const float *xin, const float *g, bool embed, NormIn &ni) {
        const int H = A.H;
#pragma unroll
        for (int p = 0; p < DS_NMAXP; p++) {
            const int i = 4 * (tid + p * DS_CT);
            ni.x[p] = (!embed && i < H) ? __ldcg(reinterpret_cast<const float4 *>(xin + i)) : make_float4(0, 0, 0, 0);
        }
        ni.g = g;
    }
    __device__ void norm_finish(const NormIn &ni, const float *add, float *xout, bool embed, const Q8Act &act) {
        const int H = A.H;
        // this lane's gains (read-only weights), in flight with the loads below
        float4 gl[2 * DS_NMAXB];
#pragma unroll
        for (int k = 0; k < DS_NMAXB; k++) {
            const int blk = warp + k * DS_NC;
            const bool v = blk < H / QK;
            const float4 *gp = reinterpret_cast<const float4 *>(ni.g + blk * QK + 8 * lane);
            gl[2 * k] = v ? __ldg(gp) : make_float4(0, 0, 0, 0);
            gl[2 * k + 1] = v ? __ldg(gp + 1) : make_float4(0, 0, 0, 0);
        }
        float *xr = reinterpret_cast<float *>(smem + L.uni);
        double *sh = reinterpret_cast<double *>(smem + L.red);  // red is free between GEMV phases
        double ss = 0.0;
        if (embed) {
            int t = A.tok[0];
            if (t < 0 || t >= A.vocab) {
                if (tid == 0 && blockIdx.x == 0) atomicOr(A.err, ERRBIT_BAD_TOKEN);
                t = 0;
            }
            const int nbe = H / QK;
            for (int i = tid; i < H; i += DS_CT) {
                const uint8_t *blk = A.emb + q4k_offset(t, i / QK, nbe);
                const uint32_t *hw = reinterpret_cast<const uint32_t *>(blk);
                const Q4Scales sc = q4k_unpack_scales(hw[1], hw[2], hw[3]);
                const float d = h2f((uint16_t)(hw[0] & 0xFFFF)), dmin = h2f((uint16_t)(hw[0] >> 16));
                const int r = i % QK, gq = r >> 6, rr = r & 63, hi = rr >> 5, l = rr & 31;
                const int j = 2 * gq + hi;
                const int scv = byte_of(j < 4 ? sc.sc_lo : sc.sc_hi, j & 3);
                const int mnv = byte_of(j < 4 ? sc.mn_lo : sc.mn_hi, j & 3);
                const int tt = l >> 3, e = l & 7;
                const int nib = (blk[16 + 32 * tt + 8 * gq + e] >> (4 * hi)) & 0xF;
                const float v = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)scv), (float)nib), __fmul_rn(dmin, (float)mnv));
                xr[i] = v;
                ss = __fma_rn((double)v, (double)v, ss);
            }
        } else {
            float4 a[DS_NMAXP];
#pragma unroll
            for (int p = 0; p < DS_NMAXP; p++) {
                const int i = 4 * (tid + p * DS_CT);
                a[p] = i < H ? __ldcg(reinterpret_cast<const float4 *>(add + i)) : make_float4(0, 0, 0, 0);
            }
#pragma unroll
            for (int p = 0; p < DS_NMAXP; p++) {
                const int i = 4 * (tid + p * DS_CT);
                if (i < H) {
                    const float4 x = ni.x[p];
                    const float4 v = make_float4(__fadd_rn(a[p].x, x.x), __fadd_rn(a[p].y, x.y), __fadd_rn(a[p].z, x.z),
                                                 __fadd_rn(a[p].w, x.w));
                    *reinterpret_cast<float4 *>(xr + i) = v;
                    ss = __fma_rn((double)v.x, (double)v.x, ss);
                    ss = __fma_rn((double)v.y, (double)v.y, ss);
                    ss = __fma_rn((double)v.z, (double)v.z, ss);
                    ss = __fma_rn((double)v.w, (double)v.w, ss);
                }
            }
        }
        ss = cons_sum64(ss, sh);  // (its barriers also publish xr)
        const float m = rms_of(ss, H, A.eps);
        // the CTA's slice of the residual for the next residual add
        const int per = ((H + gridDim.x - 1) / gridDim.x + 3) & ~3;
        for (int i = blockIdx.x * per + tid; i < min(H, (int)(blockIdx.x + 1) * per); i += DS_CT) xout[i] = xr[i];
#pragma unroll
        for (int k = 0; k < DS_NMAXB; k++) {
            const int blk = warp + k * DS_NC;
            if (blk < H / QK) {
                const float4 x0 = *reinterpret_cast<const float4 *>(xr + blk * QK + 8 * lane);
                const float4 x1 = *reinterpret_cast<const float4 *>(xr + blk * QK + 8 * lane + 4);
                const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                const float gs[8] = {gl[2 * k].x,     gl[2 * k].y,     gl[2 * k].z,     gl[2 * k].w,
                                     gl[2 * k + 1].x, gl[2 * k + 1].y, gl[2 * k + 1].z, gl[2 * k + 1].w};
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; e++) v[e] = __fmul_rn(__fdiv_rn(xs[e], m), gs[e]);
                q8k_store_warp(v, lane, act, 0, blk);
            }
        }
        cons_sync();  // act complete; sh / xr free
    }
    // Copies a global Q8_K row (device SoA form) into the shared-memory act:
    // all loads of a round (up to 8 x 16 bytes per thread) before its stores.
    __device__ void stage_act(const Q8Act &src, const Q8Act &dst, int64_t k) {
        // qs (k bytes), bs16 (k / 8 bytes) and bs32 (k / 16 bytes) in 16-byte
        // pieces; the k / 256 scales d one float per thread
        const int n0 = (int)(k / 16), n2 = (int)(k / 8 / 16), n3 = (int)(k / 16 / 16);
        const int ntot = n0 + n2 + n3, nd = (int)(k / QK);
        auto ptrs = [&](int i, const uint4 *&sp, uint4 *&dp) {
            if (i < n0) {
                sp = reinterpret_cast<const uint4 *>(src.qs) + i, dp = reinterpret_cast<uint4 *>(dst.qs) + i;
            } else if ((i -= n0) < n2) {
                sp = reinterpret_cast<const uint4 *>(src.bs16) + i, dp = reinterpret_cast<uint4 *>(dst.bs16) + i;
            } else {
                i -= n2;
                sp = reinterpret_cast<const uint4 *>(src.bs32) + i, dp = reinterpret_cast<uint4 *>(dst.bs32) + i;
            }
        };
        for (int base = 0; base < ntot; base += 8 * DS_CT) {
            uint4 r[8];
            float dv = 0.f;
            const bool dl = base == 0 && tid < nd;
            if (dl) dv = __ldcg(src.d + tid);
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int i = base + tid + u * DS_CT;
                if (i < ntot) {
                    const uint4 *sp;
                    uint4 *dp;
                    ptrs(i, sp, dp);
                    r[u] = __ldcg(sp);
                }
            }
            if (dl) dst.d[tid] = dv;
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int i = base + tid + u * DS_CT;
                if (i < ntot) {
                    const uint4 *sp;
                    uint4 *dp;
                    ptrs(i, sp, dp);
                    *dp = r[u];
                }
            }
        }
        cons_sync();
    }
    // SwiGLU + Q8_K of block blockIdx.x (one CTA per 256-value block).
    __device__ void swiglu() {
        const int F = A.F;
        float *shv = reinterpret_cast<float *>(smem + L.uni);
        int *shi = reinterpret_cast<int *>(smem + L.uni + 64);
        for (int blk = blockIdx.x; blk < F / QK; blk += gridDim.x) {
            const float gv = __ldcg(A.y_gu + blk * QK + tid), uv = __ldcg(A.y_gu + F + blk * QK + tid);
            q8k_store_block_cons(__fmul_rn(silu64(gv), uv), A.act_f, 0, blk, shv, shi);
        }
    }
    // The gains / RoPE factors of this warp's first prologue head: weights and
    // the position only, loaded before the grid barrier that precedes the
    // attention phase.
    __device__ __forceinline__ QkHead att_pre(int l, const AttItem &it) {
        QkHead qh{};
        if (it.kvh < 0 || it.mine < 0 || it.len <= 0) return qh;
        const bool owner = it.jf >= 0 && it.jf < it.mine;
        const int nwork = G + (owner ? 2 : 0);
        const int hh = warp, p = it.len - 1;
        if (hh < nwork && hh <= G) {
            const DsLayer &Ly = A.layers[l];
            qh = qk_head_load(lane, A.qk_norm ? (hh < G ? Ly.q_norm : Ly.k_norm) : nullptr,
                              A.rope_cos + (int64_t)p * (DS_HD / 2), A.rope_sin + (int64_t)p * (DS_HD / 2), A.rope_mode);
        }
        return qh;
    }
    __device__ void attention(int l, const AttItem &it, const int *bt, const QkHead &pre);
};

template <int G>
__device__ void Ds<G>::attention(int l, const AttItem &it, const int *bt, const QkHead &pre) {
    const DsAttLayout AL = ds_att_layout(G);
    uint8_t *u = smem + L.uni;
    float *q_s = reinterpret_cast<float *>(u + AL.q);
    __half *s_newkv = reinterpret_cast<__half *>(u + AL.newkv);
    const DsLayer &Ly = A.layers[l];
    __half *kpool = A.kv + (size_t)l * 2 * A.kv_layer, *vpool = kpool + A.kv_layer;
    const bool active = it.mine >= 0 && it.kvh >= 0;
    AttRegs<G> R;
#pragma unroll
    for (int g = 0; g < G; g++) {
        R.m_run[g] = -INFINITY;
#pragma unroll
        for (int e = 0; e < 4; e++) R.o[g][e] = 0.0;
    }
#pragma unroll
    for (int g = 0; g < G; g++) R.Lw[g] = 0.0;
    if (active && it.len > 0) {
        // prologue: q heads (every split), k / v of the new token (owner split)
        const bool owner = it.jf >= 0 && it.jf < it.mine;
        const int nwork = G + (owner ? 2 : 0);
        const int p = it.len - 1;
        for (int hh = warp; hh < nwork; hh += DS_NC) {
            const bool is_q = hh < G, is_k = hh == G;
            const QkHead qh = hh == warp ? pre
                              : (is_q || is_k)
                                  ? qk_head_load(lane, A.qk_norm ? (is_q ? Ly.q_norm : Ly.k_norm) : nullptr,
                                                 A.rope_cos + (int64_t)p * (DS_HD / 2),
                                                 A.rope_sin + (int64_t)p * (DS_HD / 2), A.rope_mode)
                                  : QkHead{};
            const int64_t off = is_q ? (int64_t)(it.kvh * G + hh) * DS_HD
                                     : ((int64_t)A.n_heads + (is_k ? it.kvh : A.n_kv + it.kvh)) * DS_HD;
            const float4 x = __ldcg(reinterpret_cast<const float4 *>(A.y_qkv + off + 4 * lane));
            float v[4] = {x.x, x.y, x.z, x.w};
            if (is_q || is_k) qk_head_apply(v, lane, qh, A.eps, A.rope_mode);
            if (is_q) {
#pragma unroll
                for (int e = 0; e < 4; e++) q_s[ds_qidx(4 * lane + e, hh, G)] = v[e];
                if (it.split == 0)
                    *reinterpret_cast<float4 *>(A.q_out + (int64_t)(it.kvh * G + hh) * DS_HD + 4 * lane) =
                        make_float4(v[0], v[1], v[2], v[3]);
            } else {
                const int page = bt[it.jf], slot = p % DS_CHUNK;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int d = 4 * lane + e;
                    const __half h = __float2half_rn(v[e]);
                    s_newkv[(is_k ? 0 : DS_HD) + d] = h;
                    if (page >= 0) {
                        if (is_k) kpool[(((size_t)page * A.n_kv + it.kvh) * DS_HD + d) * DS_CHUNK + slot] = h;
                        else vpool[(((size_t)page * A.n_kv + it.kvh) * DS_CHUNK + slot) * DS_HD + d] = h;
                    }
                }
            }
        }
    }
    cons_sync();  // q and the new k / v staged
    // ---- chunks: warps 0..3 take units 0..3 of even chunks, warps 4..7 of odd ones
    float *ssw = reinterpret_cast<float *>(u + AL.ss) + warp * DS_UNIT * G;
    float *pbw = reinterpret_cast<float *>(u + AL.pb) + warp * DS_UNIT * G;
    for (int j = 0; j < (active ? it.mine : 0); j++) {
        const uint8_t *kst = wait_stage();
        if (ok && (j & 1) == (warp >> 2)) {
            const int qu = warp & 3;
            const int tok0 = (it.first + j) * DS_CHUNK + DS_UNIT * qu;
            const int nt = min(DS_UNIT, it.len - tok0);
            if (nt > 0) {
                uint8_t *kw = const_cast<uint8_t *>(kst);
                const __half *Vs = reinterpret_cast<const __half *>(kst + DS_KREG);
                if (it.len - 1 < tok0 + DS_UNIT) {  // this unit holds the newest token: patch its staged k / v
                    const int tc = (it.len - 1) % DS_CHUNK;
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int d = 4 * lane + e;
                        *reinterpret_cast<__half *>(kw + (d >> 5) * DS_KQS + (d & 31) * DS_KROW + tc * 2) = s_newkv[d];
                        const_cast<__half *>(Vs)[(size_t)tc * DS_HD + d] = s_newkv[DS_HD + d];
                    }
                    __syncwarp();
                }
                ds_att_unit<G>(kst, Vs, qu, nt, q_s, ssw, pbw, A.scale, lane, R);
            }
        }
        release_stage();
    }
    // ---- CTA merge of the warps' (max, sum, o): every warp scales its partial
    // by exp64(m_w - M); then a fixed tree 8 -> 4 -> 2 -> 1 in shared memory
    double *mw = reinterpret_cast<double *>(u + AL.mw), *lw = reinterpret_cast<double *>(u + AL.lw);
    double *tree = reinterpret_cast<double *>(u + AL.tree);
    double *mmax = reinterpret_cast<double *>(u + AL.mmax);
#pragma unroll
    for (int g = 0; g < G; g++)
        if (lane == 0) lw[warp * G + g] = R.Lw[g];
#pragma unroll
    for (int g = 0; g < G; g++)
        if (lane == g) mw[warp * G + g] = (double)R.m_run[g];
    cons_sync();
    double wt[G];
    double lsc[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        double M = -INFINITY;
#pragma unroll
        for (int w = 0; w < DS_NC; w++) M = fmax(M, mw[w * G + g]);
        const double m = mw[warp * G + g];
        wt[g] = m == -INFINITY ? 0.0 : exp64(__dsub_rn(m, M));
        lsc[g] = __dmul_rn(wt[g], lw[warp * G + g]);
        if (warp == 0 && lane == 0) mmax[g] = M;
#pragma unroll
        for (int e = 0; e < 4; e++) R.o[g][e] = __dmul_rn(R.o[g][e], wt[g]);
    }
    // tree rounds: upper half of the active warps stores, lower half adds
    constexpr int TS = DS_HD + 1;  // per (slot, head): 128 dims + the sum
#pragma unroll
    for (int half = DS_NC / 2; half >= 1; half >>= 1) {
        if (warp >= half && warp < 2 * half) {
            double *t = tree + (size_t)(warp - half) * G * TS;
#pragma unroll
            for (int g = 0; g < G; g++) {
#pragma unroll
                for (int e = 0; e < 4; e++) t[g * TS + 4 * lane + e] = R.o[g][e];
                if (lane == 0) t[g * TS + DS_HD] = lsc[g];
            }
        }
        cons_sync();
        if (warp < half) {
            const double *t = tree + (size_t)warp * G * TS;
#pragma unroll
            for (int g = 0; g < G; g++) {
#pragma unroll
                for (int e = 0; e < 4; e++) R.o[g][e] = __dadd_rn(R.o[g][e], t[g * TS + 4 * lane + e]);
                lsc[g] = __dadd_rn(lsc[g], t[g * TS + DS_HD]);
            }
        }
        cons_sync();
    }
    // ---- split partial -> global; the last split of this kv head merges
    const int ns = A.ns;
    const int64_t hb0 = (int64_t)(active ? it.kvh : 0) * G * ns;
    __shared__ int s_last;
    if (active) {
        if (warp == 0) {
#pragma unroll
            for (int g = 0; g < G; g++) {
#pragma unroll
                for (int e = 0; e < 4; e++)
                    A.part_o[(hb0 + (int64_t)g * ns + it.split) * DS_HD + 4 * lane + e] = R.o[g][e];
                if (lane == 0) {
                    A.part_ml[2 * (hb0 + (int64_t)g * ns + it.split)] = mmax[g];
                    A.part_ml[2 * (hb0 + (int64_t)g * ns + it.split) + 1] = lsc[g];
                }
            }
            __threadfence();
        }
        cons_sync();
        if (tid == 0) {
            const int prev = atomicAdd(&A.att_cnt[it.kvh], 1);
            s_last = prev == ns - 1;
            if (s_last) {
                A.att_cnt[it.kvh] = 0;  // ready for the next layer
                __threadfence();
            }
        }
        cons_sync();
        if (s_last) {
            double *wts = reinterpret_cast<double *>(u + AL.wts), *wl = reinterpret_cast<double *>(u + AL.wl);
            float *fin = reinterpret_cast<float *>(u + AL.fin);
            if (warp < G) {  // warp g: split weights of head g (lane = split)
                const int g = warp;
                double Mr = -INFINITY, Lr = 0.0;
                if (lane < ns) {
                    Mr = __ldcg(&A.part_ml[2 * (hb0 + (int64_t)g * ns + lane)]);
                    Lr = __ldcg(&A.part_ml[2 * (hb0 + (int64_t)g * ns + lane) + 1]);
                }
                double M = Mr;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) M = fmax(M, __shfl_xor_sync(0xffffffffu, M, off));
                if (lane < ns) {
                    const double w = Mr == -INFINITY ? 0.0 : exp64(__dsub_rn(Mr, M));
                    wts[g * DS_SPLITS_MAX + lane] = w;
                    wl[g * DS_SPLITS_MAX + lane] = __dmul_rn(w, Lr);
                }
            }
            cons_sync();
            for (int i = tid; i < G * DS_HD; i += DS_CT) {
                const int g = i / DS_HD, d = i % DS_HD;
                double Lsum = 0.0, O = 0.0;
                for (int r0 = 0; r0 < ns; r0 += 16) {
                    double Or[16];
#pragma unroll
                    for (int k = 0; k < 16; k++)
                        Or[k] = r0 + k < ns ? __ldcg(&A.part_o[(hb0 + (int64_t)g * ns + r0 + k) * DS_HD + d]) : 0.0;
#pragma unroll
                    for (int k = 0; k < 16; k++)
                        if (r0 + k < ns) {
                            Lsum = __dadd_rn(Lsum, wl[g * DS_SPLITS_MAX + r0 + k]);
                            O = __dadd_rn(O, __dmul_rn(wts[g * DS_SPLITS_MAX + r0 + k], Or[k]));
                        }
                }
                const float val = Lsum > 0.0 ? __double2float_rn(__ddiv_rn(O, Lsum)) : 0.f;
                A.attn[(int64_t)(it.kvh * G + g) * DS_HD + d] = val;
                fin[i] = val;
            }
            cons_sync();
            for (int blk = warp; blk < G / 2; blk += DS_NC) {
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; e++) v[e] = fin[blk * 256 + 8 * lane + e];
                q8k_store_warp(v, lane, A.act_a, 0, (int64_t)it.kvh * G / 2 + blk);
            }
        }
    }
}

// Attention item of this CTA: (kv head, split) = (cta / ns, cta % ns) for
// cta < n_kv * ns; its chunks and the page of each (thread 0, into smem).
__device__ void ds_att_item(const DsArgs &A, AttItem &it, int *bt) {
    const int items = A.n_kv * A.ns;
    it.kvh = -1;
    it.split = 0;
    it.len = 0;
    it.first = 0;
    it.mine = -1;
    it.jf = -1;
    if ((int)blockIdx.x >= items) return;
    it.kvh = blockIdx.x / A.ns;
    it.split = blockIdx.x % A.ns;
    int len = A.pos[0] + 1;
    const int cap = min(A.pages_per_seq * DS_CHUNK, A.rope_rows);
    if (len < 1 || len > cap) {
        if (it.split == 0 && it.kvh == 0) atomicOr(A.err, ERRBIT_BAD_POS);
        len = 0;
    }
    const int nch = (len + DS_CHUNK - 1) / DS_CHUNK;
    const int cpr = (nch + A.ns - 1) / A.ns;
    const int first = min(it.split * cpr, nch);
    it.len = len;
    it.first = first;
    it.mine = min(min(cpr, nch - first), DS_BT_CAP);
    it.jf = len > 0 ? (len - 1) / DS_CHUNK - first : -1;
    for (int j = 0; j < it.mine; j++) {
        const int lp = first + j;
        int page = lp < A.pages_per_seq ? A.block_table[lp] : -1;
        if (page < 0 || page >= A.num_pages) {
            atomicOr(A.err, ERRBIT_BAD_PAGE);
            page = -1;
        }
        bt[j] = page;
    }
}

template <int G>
__global__ void __launch_bounds__(DS_THREADS, 1) k_decode_step(DsArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[DS_MAXSTAGE], empty[DS_MAXSTAGE];
    __shared__ int tcnt[DS_MAXSTAGE + 1];
    __shared__ int bt[DS_BT_CAP];
    __shared__ AttItem s_it;
    __shared__ int s_ok;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kmax = max(max(A.H, A.F), A.n_heads * DS_HD);
    const DsLayout L = ds_layout(A.nstage, kmax, A.H, G);
    if (tid == 0) {
        for (int i = 0; i < A.nstage; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], DS_NC);
        }
        mbar_fence_init();
        ds_att_item(A, s_it, bt);
    }
    if (tid <= A.nstage) tcnt[tid] = 0;
    __syncthreads();
    const AttItem it = s_it;
    const int H = A.H, F = A.F, qd = A.n_heads * DS_HD;

    if (warp == DS_NC) {
        // ---------------- producer: one lane issues every stage in consumption order
        if (lane == 0) ds_produce(A, it, bt, smem + L.ring, full, empty);
        return;
    }
    // ---------------- consumers
    Ds<G> C(A, smem, L, full, empty, tcnt, &s_ok);
    const Q8Act act = ds_act_view(smem + L.act, kmax);
    const Q8Act act_h = ds_act_view(smem + L.act, H);
    const Q8Act act_q = ds_act_view(smem + L.act, qd);
    const Q8Act act_f = ds_act_view(smem + L.act, F);
    (void)act;
    unsigned bar_k = 0;
    float *xa = A.xa, *xb = A.xb;
    // phase timeline (optional): stamp k of layer l after each phase
    auto stamp = [&](int l, int k) {
        if (A.trace && tid == 0)
            A.trace[((size_t)blockIdx.x * (A.n_layers + 1) + l) * DS_TRACE_SLOTS + k] = globaltimer_ns();
    };
    stamp(0, 15);
    typename Ds<G>::NormIn ni;
    C.norm_load(nullptr, A.layers[0].attn_norm, true, ni);
    C.norm_finish(ni, nullptr, xb, true, act_h);
    {
        float *t = xa;
        xa = xb;
        xb = t;
    }
    bool done = false;
    for (int l = 0; l < A.n_layers; l++) {
        const DsLayer &Ly = A.layers[l];
        stamp(l, 0);
        C.gemv(Ly.qkv, Ly.dt_qkv, A.qkv_n, H, act_h, A.y_qkv);
        stamp(l, 1);
        const QkHead qh = C.att_pre(l, it);
        if (!C.ok || !grid_barrier(A, ++bar_k, &s_ok)) break;
        stamp(l, 2);
        C.attention(l, it, bt, qh);
        stamp(l, 3);
        if (!C.ok || !grid_barrier(A, ++bar_k, &s_ok)) break;
        stamp(l, 4);
        C.stage_act(A.act_a, act_q, qd);
        C.gemv(Ly.o, Ly.dt_o, H, qd, act_q, A.y_o);
        stamp(l, 5);
        C.norm_load(xa, Ly.ffn_norm, false, ni);
        if (!C.ok || !grid_barrier(A, ++bar_k, &s_ok)) break;
        stamp(l, 6);
        // x += y_o; act = Q8_K(RMSNorm(x) * ffn_norm)
        C.norm_finish(ni, A.y_o, xb, false, act_h);
        {
            float *t = xa;
            xa = xb;
            xb = t;
        }
        stamp(l, 7);
        C.gemv(Ly.gu, Ly.dt_gu, 2 * F, H, act_h, A.y_gu);
        stamp(l, 8);
        if (!C.ok || !grid_barrier(A, ++bar_k, &s_ok)) break;
        stamp(l, 9);
        C.swiglu();
        stamp(l, 10);
        if (!C.ok || !grid_barrier(A, ++bar_k, &s_ok)) break;
        stamp(l, 11);
        C.stage_act(A.act_f, act_f, F);
        C.gemv(Ly.down, Ly.dt_down, H, F, act_f, A.y_d);
        stamp(l, 12);
        const bool last = l + 1 == A.n_layers;
        C.norm_load(xa, last ? A.out_norm : A.layers[l + 1].attn_norm, false, ni);
        if (!C.ok || !grid_barrier(A, ++bar_k, &s_ok)) break;
        stamp(l, 13);
        if (A.trace && tid == 0) A.trace[((size_t)blockIdx.x * (A.n_layers + 1) + l) * DS_TRACE_SLOTS + 14] = C.wait_ns;
        // x += y_down; act = Q8_K(RMSNorm(x) * g) with the next layer's
        // attn_norm, or the final norm before the lm_head
        C.norm_finish(ni, A.y_d, xb, false, act_h);
        if (!last) {
            float *t = xa;
            xa = xb;
            xb = t;
        } else {
            done = true;
        }
    }
    if (done && C.ok && !aborted(A)) {
        stamp(A.n_layers, 0);
        C.gemv(A.out, A.dt_out, A.vocab, H, act_h, A.logits);
        stamp(A.n_layers, 1);
    }
    (void)lane;
}

// ------------------------------------------------------------ host side
template <int G>
static bool ds_plan_g(const fb_ctx *ctx, int H, int F, int qd, int n_kv, int pages_per_seq, DsPlan &p) {
    const int kmax = std::max(std::max(H, F), qd);
    for (int ns = DS_MAXSTAGE; ns >= 3; ns--) {
        const size_t sm = ds_layout(ns, kmax, H, G).total;
        if (sm <= 227 * 1024 - 4096) {
            p.nstage = ns;
            p.smem = sm;
            break;
        }
    }
    if (!p.nstage) return false;
    p.ns = std::min(DS_SPLITS_MAX, ctx->num_sms / n_kv);
    if (p.ns < 1) return false;
    if ((pages_per_seq + p.ns - 1) / p.ns > DS_BT_CAP) return false;
    return true;
}

bool decode_step_plan(const fb_ctx *ctx, int H, int F, int n_heads, int n_kv, int pages_per_seq, int page,
                      DsPlan *out) {
    if (page != DS_CHUNK || n_heads % n_kv != 0) return false;
    const int G = n_heads / n_kv;
    const int qd = n_heads * DS_HD;
    if (H % QK || F % QK || qd % QK || H % 4) return false;
    // residual row registers (norm_load) and one scale per thread (stage_act)
    if (H > DS_NMAXP * 4 * DS_CT || H / QK > DS_NMAXB * DS_NC || F / QK > DS_CT || qd / QK > DS_CT) return false;
    DsPlan p;
    bool ok = false;
    switch (G) {
    case 2: ok = ds_plan_g<2>(ctx, H, F, qd, n_kv, pages_per_seq, p); break;
    case 4: ok = ds_plan_g<4>(ctx, H, F, qd, n_kv, pages_per_seq, p); break;
    case 8: ok = ds_plan_g<8>(ctx, H, F, qd, n_kv, pages_per_seq, p); break;
    default: return false;
    }
    if (ok && out) *out = p;
    return ok;
}

template <int G>
static void launch_g(fb_ctx *ctx, const DsArgs &A, size_t smem) {
    auto kern = k_decode_step<G>;
    static std::mutex mu;
    static std::map<int, size_t> done;
    {
        std::lock_guard<std::mutex> lock(mu);
        auto itd = done.find(ctx->device);
        if (itd == done.end() || itd->second < smem) {
            FB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            done[ctx->device] = smem;
        }
    }
    int occ = 0;
    FB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, DS_THREADS, smem));
    FB_REQUIRE(occ >= 1, "decode step: the persistent kernel does not fit on an SM");
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.gridDim = dim3(ctx->num_sms);
    cfg.blockDim = dim3(DS_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    FB_CUDA(cudaLaunchKernelEx(&cfg, kern, A));
}

void launch_decode_step(fb_ctx *ctx, const DsArgs &A, size_t smem) {
    // barrier arrivals, abort flag and the split-merge counters start at zero
    FB_CUDA(cudaMemsetAsync(A.sync, 0, 64 * sizeof(unsigned), ctx->stream));
    FB_CUDA(cudaMemsetAsync(A.att_cnt, 0, (size_t)A.n_kv * sizeof(int), ctx->stream));
    switch (A.n_heads / A.n_kv) {
    case 2: launch_g<2>(ctx, A, smem); break;
    case 4: launch_g<4>(ctx, A, smem); break;
    case 8: launch_g<8>(ctx, A, smem); break;
    default: fail(FB_ERR_INVALID, "decode step: GQA group must be 2, 4 or 8");
    }
}

}  // namespace fb
