// GQA flash-decode attention over a paged fp16 KV cache.
//
// Replaces the attention inside candle-transformers 0.8.4 quantized_llama
// (q.k^T / sqrt(hd) -> softmax_last_dim -> .v over an f32 KV cache that grows
// by concatenation; called from crates/ferrite-wasm-host/src/adapter.rs:
// 61-70) and the reference's own stub kernel
// crates/ferrite-core/kernels/flash_attention.cu:166-225 (f32, hd <= 64,
// never launched).
//
// KV layout (per layer): K pages are dim-major, [page][kv head][hd][page
// tokens], V pages token-major, [page][kv head][page tokens][hd], fp16.
//
// B200 design (HBM-bound: 2 * ctx * n_kv * hd * 2 bytes per layer and token):
//  * one CTA per (split, kv head, sequence); the sequence's 64-token chunks
//    are split evenly over the splits at run time (from the sequence length
//    on the device), so the grid does not depend on the context length;
//  * each CTA streams its chunks through a ring of `depth` shared-memory
//    stages with cp.async.bulk (TMA, no multicast) on per-stage mbarriers; the
//    four 32-dim quarters of a K page land 32 bytes apart (bank shift);
//  * warps work independently, without CTA barriers: a chunk is four units
//    of 16 tokens and warp w takes units w, w + NW, ... (NW divides the 4 *
//    depth units of one pass over the ring, so a warp meets every stage it
//    waits on once per pass and never waits a phase ahead).  Per unit the
//    warp computes the f32 scores (lane = 2 tokens x one 32-dim quarter, the
//    quarters' slice sums chained in slice order through shuffles), the
//    unit's softmax partial in f32 (exponentials spread over all lanes, P.V
//    with lane = 4 dims) and folds it into its binary64 running state.  The
//    last of a chunk's four units refills its stage;
//  * the CTA merges its warps' (max, sum, o) partials in shared memory, then
//    the splits merge either through distributed shared memory in a 16-CTA
//    cluster (CTA r owns dims [8r, 8r+8) of every head; push, no atomics), or
//    through global partials and a last-CTA merge (model path, and the
//    allocation-free entry point); the result is written as f32 and, in the
//    model path, as the Q8_K rows of the output projection.
// Dots and the 16-token unit partials are f32 in the CPU oracle's fixed
// order; everything above the units runs in binary64 with one rounding to
// f32 at the end, so the result equals the CPU oracle's bit for bit whatever
// the split and warp layout.  All mbarrier waits are bounded: on timeout the kernel raises
// ERRBIT_WAIT_TIMEOUT in the context's error word.
#include <math.h>

#include <algorithm>
#include <cooperative_groups.h>
#include <map>
#include <mutex>

#include "fb_internal.h"
#include "kq_common.cuh"
#include "attn_unit.cuh"

namespace cg = cooperative_groups;

namespace fb {

constexpr int ATT_HD = 128;
constexpr int ATT_CHUNK = 64;  // tokens per pipeline stage (one or two pages)
constexpr int ATT_UNIT = 16;   // tokens per warp work unit (four per chunk)
// warps per CTA: 16 for GQA groups up to 4, 8 for groups of 8 (their binary64
// P.V accumulators double) and for the cluster variant (two-stage ring)
__host__ __device__ constexpr int att_warps(int G, bool cluster) { return G <= 4 && !cluster ? 16 : 8; }
__host__ __device__ constexpr int att_depth(bool cluster) { return cluster ? 2 : 4; }
constexpr int ATT_DPR = ATT_HD / ATT_SPLITS;  // output dims merged per cluster rank
constexpr int ATT_MAX_DEPTH = 4;
constexpr int ATT_QPAD = 32;  // bytes between the four 32-dim quarters of a staged K page
constexpr uint32_t ATT_STAGE_K = 2 * (32 * ATT_HD * 2 + 4 * ATT_QPAD);  // K region of a stage (two 32-token pages)
constexpr uint32_t ATT_STAGE = ATT_STAGE_K + ATT_CHUNK * ATT_HD * 2;     // + V region
static_assert(ATT_CHUNK * ATT_HD * 2 + 4 * ATT_QPAD <= ATT_STAGE_K, "one 64-token K page must fit the K region");
static_assert(4 * att_depth(false) % att_warps(1, false) == 0 && 4 * att_depth(false) % att_warps(8, false) == 0 &&
                  4 * att_depth(true) % att_warps(1, true) == 0,
              "a pass over the ring must hand every warp whole units");

__device__ __forceinline__ int seq_len_of(const AttnArgs &A, int b) {
    return A.seq_lens ? A.seq_lens[b] : A.pos[b] + 1;
}

// q in shared memory: [hd][G] f32 with G floats of padding after each 32-dim
// quarter, so the four quarter groups of a warp read different banks
__host__ __device__ constexpr int att_qidx(int d, int g, int G) { return (d + (d >> 5)) * G + g; }

__device__ __forceinline__ void q8k_store_warp_ext(const float (&v)[8], int lane, const Q8Act &a, int64_t row,
                                                   int64_t blk);

// Dynamic shared memory of one CTA (byte offsets).
struct AttnLayout {
    size_t q, ss, pb, misc, inbox, q8in, bt, total;
};
__host__ __device__ inline AttnLayout attn_layout(int G, int NW, int depth, int bt_cap) {
    AttnLayout L;
    size_t off = (size_t)depth * ATT_STAGE;  // the ring; [NW][G][hd] f64 warp partials at the end
    off = (off + 127) & ~(size_t)127;
    L.q = off;  // q (att_qidx layout); merged outputs [G][hd] f32 at the end
    off += (size_t)(ATT_HD + 4) * G * 4;
    off = (off + 15) & ~(size_t)15;
    L.ss = off;  // per warp: scores [unit token][G] f32
    off += (size_t)NW * ATT_UNIT * G * 4;
    off = (off + 15) & ~(size_t)15;
    L.pb = off;  // per warp: p [unit token][G] f32 (room for f64); CTA partial o [G][hd] f64 at the end
    off += (size_t)NW * ATT_UNIT * G * 8;
    L.misc = off;  // M[G] L[G] tmp[G] mw[NW][G] lw[NW][G] wt[NW][G] wts[G][S] wl[G][S] f64
    off += (size_t)(3 * G + 3 * NW * G + 2 * G * ATT_SPLITS_MAX) * 8;
    L.inbox = off;  // cluster merge: [src rank][G][ATT_DPR + 2] f64 pushed by the peers
    off += (size_t)ATT_SPLITS * G * (ATT_DPR + 2) * 8;
    L.q8in = off;  // cluster merge: [2][hd] f32 outputs of one Q8_K block
    off += (size_t)2 * ATT_HD * 4;
    L.bt = off;  // block-table entries of the CTA's pages
    off += (size_t)bt_cap * 4;
    L.total = (off + 127) & ~(size_t)127;
    return L;
}

__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// G consecutive f32 from shared memory (16-byte aligned for G >= 4).
template <int G>
__device__ __forceinline__ void lds_f32(float (&v)[G], const float *p) {
    if constexpr (G % 4 == 0) {
#pragma unroll
        for (int i = 0; i < G; i += 4) {
            const float4 x = *reinterpret_cast<const float4 *>(p + i);
            v[i] = x.x;
            v[i + 1] = x.y;
            v[i + 2] = x.z;
            v[i + 3] = x.w;
        }
    } else if constexpr (G == 2) {
        const float2 x = *reinterpret_cast<const float2 *>(p);
        v[0] = x.x;
        v[1] = x.y;
    } else {
        v[0] = p[0];
    }
}

// grid (splits, n_kv, batch): CLUSTER: ATT_SPLITS splits, cluster dims
// (ATT_SPLITS, 1, 1); otherwise gridDim.x (<= ATT_SPLITS_MAX) splits.
//
// Numerics (identical to the CPU oracle, or_attn_dot / or_exp64):
//   s_t = f32 dot of q and k_t in eight 16-dim fused-multiply-add slices,
//         summed in slice order, times scale
//   per 16-token unit u (positions 16u .. 16u + 15; f32, fixed order):
//             m_u = max s_t, p_t = f32(exp64(s_t - m_u)), l_u = pairwise
//             sum of the 16 slots (absent tokens 0), o_u = FMA chain of
//             p_t v_t in token order
//   per warp (binary64): the units' (m_u, l_u, o_u) folded into a running
//             (m, l, o), the side with the smaller max weighted by exp64 of
//             the difference
//   merges (warps of a CTA, then splits): M = max m, w = exp64(m - M),
//             out = f32(sum w*o / sum w*l)
// The unit partials do not depend on how the units are spread over warps and
// CTAs, and the binary64 stages above them make the result independent of it
// too (up to binary64 rounding, far below the final f32 rounding).
template <int G, bool CLUSTER>
__global__ void __launch_bounds__(32 * att_warps(G, CLUSTER), 1)
    k_attn_decode(AttnArgs A, float *__restrict__ out_f32, Q8Act aq, int use_q8, int *__restrict__ counters,
                  int bt_cap) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[ATT_MAX_DEPTH];
    __shared__ int used[ATT_MAX_DEPTH];  // units consumed per stage (the fourth of a chunk refills it)
    __shared__ int s_len, s_first, s_mine, s_last, s_last2;
    __shared__ __half s_newkv[2 * ATT_HD];  // fused prologue: the new token's k and v (fp16)
    constexpr int S = ATT_SPLITS;
    const int ns = CLUSTER ? S : (int)gridDim.x;  // splits of this (kv head, sequence)
    constexpr int NW = att_warps(G, CLUSTER), NT = 32 * NW;
    constexpr int GH = G >= 2 ? G / 2 : 1;  // heads exponentiated per lane
    constexpr int IB = ATT_DPR + 2;         // inbox doubles per (source rank, head)
    constexpr unsigned FULL = 0xffffffffu;
    // peers may push into this CTA's shared memory once every CTA of the
    // cluster has started: arrive now, wait just before the first push
    if constexpr (CLUSTER) cluster_arrive_relaxed();
    const int rank = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    // ring stages (a compile-time constant: the stage and phase of chunk j
    // are bit operations, not divisions, in the unit loop)
    constexpr int depth = att_depth(CLUSTER);
    const int P = A.page_size, PPC = ATT_CHUNK / P;  // pages per chunk
    const int lgP = P == 64 ? 6 : 5;                 // page sizes 32 and 64 (checked on the host)
    const AttnLayout Ly = attn_layout(G, NW, depth, bt_cap);
    uint8_t *ring = smem;
    float *q_s = reinterpret_cast<float *>(smem + Ly.q);
    double *M_s = reinterpret_cast<double *>(smem + Ly.misc);
    double *L_s = M_s + G, *tmpM = L_s + G, *mw = tmpM + G, *lw = mw + NW * G, *wt = lw + NW * G;
    double *wts = wt + NW * G, *wl = wts + G * ATT_SPLITS_MAX;
    double *inbox = reinterpret_cast<double *>(smem + Ly.inbox);
    float *q8in = reinterpret_cast<float *>(smem + Ly.q8in);
    int *bt_s = reinterpret_cast<int *>(smem + Ly.bt);
    double *O_s = reinterpret_cast<double *>(smem + Ly.pb);  // [G][hd] CTA partial at the end
    double *red = reinterpret_cast<double *>(ring);          // [NW][G][hd] warp partials at the end
    float *fin = q_s;                                        // merged outputs at the end

    if (tid == 0) {
        for (int i = 0; i < depth; i++) {
            mbar_init(&full[i], 1);
            used[i] = 0;
        }
        mbar_fence_init();
        // sequence lengths are inputs of the whole step (written before it began)
        int len = seq_len_of(A, b);
        const int cap = A.qkv ? min(A.max_pages * P, A.rope_rows) : A.max_pages * P;
        if (len < 1 || len > cap) {
            atomicOr(A.err, ERRBIT_BAD_POS);
            len = 0;  // no work: the output of this sequence is zero
        }
        const int nch = (len + ATT_CHUNK - 1) / ATT_CHUNK;
        const int cpr = (nch + ns - 1) / ns;  // chunks per rank
        const int first = min(rank * cpr, nch);
        s_len = len;
        s_first = first;
        s_mine = min(cpr, nch - first);
    }
    __syncthreads();
    const int len = s_len, first = s_first, mine = s_mine;
    // block-table entries of this CTA's pages (-1: past the sequence end)
    for (int i = tid; i < mine * PPC; i += NT) {
        const int lp = first * PPC + i;
        int page = -1;
        if (lp * P < len) {
            page = lp < A.max_pages ? A.block_table[(int64_t)b * A.max_pages + lp] : -1;
            if (page < 0 || page >= A.num_pages) {
                atomicOr(A.err, ERRBIT_BAD_PAGE);
                page = -1;
            }
        }
        bt_s[i] = page;
    }
    // the chunk holding the newest position: without the fused prologue its
    // newest token is written by the preceding kernel, so it is copied after
    // griddepcontrol.wait; every other copy streams in before the wait
    const int jf = len > 0 ? (len - 1) / ATT_CHUNK - first : -1;
    const bool owner = jf >= 0 && jf < mine;
    const int pre = min(mine, depth);
    // fused prologue: warp hh < G transforms q head hh, warps G and G + 1 (the
    // newest chunk's owner) the new k and v; their gains and RoPE factors
    // depend only on weights and the position: their loads are issued here,
    // in flight together with the block-table reads above
    const int nwork = A.qkv && len > 0 ? G + (owner ? 2 : 0) : 0;
    QkHead qh{};
    if (warp < nwork && warp <= G)
        qh = qk_head_load(lane, A.q_norm ? (warp < G ? A.q_norm : A.k_norm) : nullptr,
                          A.rope_cos + (int64_t)(len - 1) * (ATT_HD / 2), A.rope_sin + (int64_t)(len - 1) * (ATT_HD / 2),
                          A.rope_mode);
    __syncthreads();
    const uint32_t pbytes = (uint32_t)P * ATT_HD * 2;         // one K (or V) page
    const uint32_t KPG = pbytes + 4 * ATT_QPAD;               // staged K page stride
    const uint32_t KQS = pbytes / 4 + ATT_QPAD;               // staged K quarter stride (32 dims)
    const uint32_t KROW = 2u * P;                             // bytes between consecutive dims
    auto k_at = [&](uint8_t *kst, int d, int tc) -> __half * {  // staged K element (dim d, chunk token tc)
        return reinterpret_cast<__half *>(kst + (tc >> lgP) * KPG + (d >> 5) * KQS + (d & 31) * KROW +
                                          (tc & (P - 1)) * 2);
    };
    // copy `piece` (0..3: the K quarters, 4: the V page) of page i of chunk j
    // into stage j % depth
    const uint64_t kvpol = l2_evict_first_policy();  // the cache is read once per step
    auto issue_piece = [&](int j, int i, int piece) {
        const int page = bt_s[j * PPC + i];
        if (page < 0) return;
        uint8_t *kd = ring + (size_t)(j % depth) * ATT_STAGE;
        const size_t off = ((size_t)page * A.n_kv + kvh) * (size_t)P * ATT_HD;
        if (piece < 4)
            bulk_g2s_stream(kd + i * KPG + piece * KQS,
                            reinterpret_cast<const uint8_t *>(reinterpret_cast<const __half *>(A.kpool) + off) +
                                piece * (pbytes / 4),
                            pbytes / 4, &full[j % depth], kvpol);
        else
            bulk_g2s_stream(kd + ATT_STAGE_K + i * pbytes, reinterpret_cast<const __half *>(A.vpool) + off, pbytes,
                            &full[j % depth], kvpol);
    };
    auto arm = [&](int j) {  // the bytes chunk j brings (zero: the phase completes without data)
        uint32_t bytes = 0;
        for (int i = 0; i < PPC; i++)
            if (bt_s[j * PPC + i] >= 0) bytes += 2 * pbytes;
        mbar_expect_tx(&full[j % depth], bytes);
    };
    auto issue = [&](int j) {  // chunk j of this CTA into stage j % depth
        arm(j);
        for (int i = 0; i < PPC; i++)
            for (int piece = 0; piece < 5; piece++) issue_piece(j, i, piece);
    };
    // the first chunks stream in before the wait, one copy per lane of warp 0
    // (lane j < pre arms stage j; the copies may complete before the arm)
    if (warp == 0) {
        for (int c = lane; c < pre * PPC * 5; c += 32) {
            const int j = c / (PPC * 5);
            if (j != jf || A.qkv) issue_piece(j, (c / 5) % PPC, c % 5);
        }
        if (lane < pre && (lane != jf || A.qkv)) arm(lane);
    }
    pdl_wait();
    if (tid == 0 && !A.qkv && jf >= 0 && jf < pre) issue(jf);
    if (A.qkv) {
        // q of the G heads (every CTA), k and v of the new token (owner only)
        const int p = len - 1;
        const float *yrow = A.qkv + (int64_t)b * A.qkv_ld;
        for (int hh = warp; hh < nwork; hh += NW) {
            if (hh != warp && hh <= G)  // a second head on this warp (GQA group 8): load its factors now
                qh = qk_head_load(lane, A.q_norm ? (hh < G ? A.q_norm : A.k_norm) : nullptr,
                                  A.rope_cos + (int64_t)p * (ATT_HD / 2), A.rope_sin + (int64_t)p * (ATT_HD / 2),
                                  A.rope_mode);
            const bool is_q = hh < G, is_k = hh == G;
            const int64_t off = is_q ? (int64_t)(kvh * G + hh) * ATT_HD
                                     : ((int64_t)A.n_heads + (is_k ? kvh : A.n_kv + kvh)) * ATT_HD;
            const float4 x = *reinterpret_cast<const float4 *>(yrow + off + 4 * lane);
            float v[4] = {x.x, x.y, x.z, x.w};
            if (is_q || is_k) qk_head_apply(v, lane, qh, A.eps, A.rope_mode);
            if (is_q) {
#pragma unroll
                for (int e = 0; e < 4; e++) q_s[att_qidx(4 * lane + e, hh, G)] = v[e];
                if (rank == 0 && A.q_out)
                    *reinterpret_cast<float4 *>(A.q_out + ((int64_t)b * A.n_heads + kvh * G + hh) * ATT_HD +
                                                4 * lane) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
                // into the KV pool (for later steps) and, in the main loop, into the staged chunk
                const int tc = p % ATT_CHUNK, page = bt_s[jf * PPC + tc / P], slot = p % P;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int d = 4 * lane + e;
                    const __half h = __float2half_rn(v[e]);
                    s_newkv[(is_k ? 0 : ATT_HD) + d] = h;
                    if (page >= 0) {
                        if (is_k)
                            reinterpret_cast<__half *>(const_cast<void *>(A.kpool))
                                [(((size_t)page * A.n_kv + kvh) * ATT_HD + d) * P + slot] = h;
                        else
                            reinterpret_cast<__half *>(const_cast<void *>(A.vpool))
                                [(((size_t)page * A.n_kv + kvh) * P + slot) * ATT_HD + d] = h;
                    }
                }
            }
        }
    } else {
        const float *qg = A.q + ((int64_t)b * A.n_heads + (int64_t)kvh * G) * ATT_HD;
        for (int i = tid; i < G * ATT_HD; i += NT) q_s[att_qidx(i % ATT_HD, i / ATT_HD, G)] = qg[i];
    }
    __syncthreads();  // q and the new token's k / v are staged

    // ---- main loop: this warp's units
    float *ssw = reinterpret_cast<float *>(smem + Ly.ss) + warp * ATT_UNIT * G;
    float *pbw = reinterpret_cast<float *>(smem + Ly.pb) + warp * ATT_UNIT * G;
    const int ti = lane & 7, qq4 = lane >> 3;  // score phase: token pair, 32-dim quarter
    float m_run[G];
    double o[G][4], Lw[G];  // the warp's binary64 state (Lw, m_run warp-uniform; o: this lane's dims)
#pragma unroll
    for (int g = 0; g < G; g++) {
        m_run[g] = -INFINITY;
        Lw[g] = 0.0;
#pragma unroll
        for (int e = 0; e < 4; e++) o[g][e] = 0.0;
    }
    bool ok = true;
    for (int u = warp; u < 4 * mine; u += NW) {
        const int j = u >> 2, qu = u & 3, st = j % depth;
        uint8_t *kst = ring + (size_t)st * ATT_STAGE;
        __half *Vs = reinterpret_cast<__half *>(kst + ATT_STAGE_K);
        const int tok0 = (first + j) * ATT_CHUNK + ATT_UNIT * qu;  // position of the unit's first token
        const int nt = min(ATT_UNIT, len - tok0);                  // tokens of the unit (<= 0: none)
        ok = mbar_wait_bounded(&full[st], (uint32_t)(j / depth) & 1u) && ok;
        if (nt > 0) {
            if (A.qkv && len - 1 < tok0 + ATT_UNIT) {
                // this unit holds the newest token, whose staged copy predates
                // this step: patch in the k / v the prologue produced
                const int tc = (len - 1) % ATT_CHUNK;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int d = 4 * lane + e;
                    *k_at(kst, d, tc) = s_newkv[d];
                    Vs[(size_t)tc * ATT_HD + d] = s_newkv[ATT_HD + d];
                }
                __syncwarp();
            }
            // ---- scores: lane (ti, qq4) dots tokens 2ti, 2ti + 1 of the unit
            // over dims [32 qq4, 32 qq4 + 32) as two 16-dim slices
            float acc[2][2][G];
#pragma unroll
            for (int sl = 0; sl < 2; sl++)
#pragma unroll
                for (int t = 0; t < 2; t++)
#pragma unroll
                    for (int g = 0; g < G; g++) acc[sl][t][g] = 0.f;
            {
                const int tc = ATT_UNIT * qu + 2 * ti;
                const uint8_t *kp = reinterpret_cast<const uint8_t *>(k_at(kst, 32 * qq4, tc));
                const float *qw = q_s + att_qidx(32 * qq4, 0, G);
#pragma unroll
                for (int e = 0; e < 16; e++) {
#pragma unroll
                    for (int sl = 0; sl < 2; sl++) {
                        const int r = 16 * sl + e;
                        const float2 k2 = __half22float2(*reinterpret_cast<const __half2 *>(kp + r * KROW));
                        float qv[G];
                        lds_f32<G>(qv, qw + r * G);
#pragma unroll
                        for (int g = 0; g < G; g++) {
                            acc[sl][0][g] = __fmaf_rn(qv[g], k2.x, acc[sl][0][g]);
                            acc[sl][1][g] = __fmaf_rn(qv[g], k2.y, acc[sl][1][g]);
                        }
                    }
                }
            }
            // slice sums in slice order: quarter 0 adds s0 + s1, quarter q
            // continues with s_2q, s_2q+1 from quarter q - 1's running sum
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
            // quarter 3 holds the full dots: scale, mask, unit max per head
            float mx[G];
#pragma unroll
            for (int g = 0; g < G; g++) {
                const float s0 = 2 * ti < nt ? __fmul_rn(T[0][g], A.scale) : -INFINITY;
                const float s1 = 2 * ti + 1 < nt ? __fmul_rn(T[1][g], A.scale) : -INFINITY;
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
            // ---- the unit's softmax partial in f32, folded into the warp's
            // binary64 state (attn_unit.cuh)
            att_unit_fold<G>(ssw, pbw, Vs + (size_t)(ATT_UNIT * qu) * ATT_HD + 4 * lane, nt, mx, lane, m_run, Lw, o);
        }
        // this warp is done with the unit's slice of stage st; the fourth unit
        // of the chunk refills the stage with chunk j + depth
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            if ((atomicAdd(&used[st], 1) & 3) == 3 && j + depth < mine) {
                fence_proxy_async_smem();
                issue(j + depth);
            }
        }
    }
    // the next kernel (the output projection) may start streaming its weights:
    // after the chunk loop its prefetch no longer competes with the K/V
    // stream, and the merges still leave it time (earlier, right after the
    // grid-dependency wait, measured 1% slower per decode step)
    pdl_launch();
    // every warp is done with the ring; on a timed-out wait let the copies in
    // flight land before the ring is reused
    if (__syncthreads_or(!ok)) {
        if (tid == 0) {
            atomicOr(A.err, ERRBIT_WAIT_TIMEOUT);
            for (int st = 0; st < min(depth, mine); st++) {
                const int jl = st + ((mine - 1 - st) / depth) * depth;
                mbar_wait_bounded(&full[st], (uint32_t)(jl / depth) & 1u);
            }
        }
        __syncthreads();
    }
    // ---- CTA partial: the warps' (max, sum, o) merged in fixed warp order
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int e = 0; e < 4; e++) red[(warp * G + g) * ATT_HD + 4 * lane + e] = o[g][e];
#pragma unroll
    for (int g = 0; g < G; g++)
        if (lane == 0) lw[warp * G + g] = Lw[g];
#pragma unroll
    for (int g = 0; g < G; g++)
        if (lane == g) mw[warp * G + g] = (double)m_run[g];
    __syncthreads();
    if (tid < NW * G) {
        const int g = tid % G;
        double M = -INFINITY;
        for (int w = 0; w < NW; w++) M = fmax(M, mw[w * G + g]);
        const double m = mw[tid];
        wt[tid] = m == -INFINITY ? 0.0 : exp64(__dsub_rn(m, M));
        if (tid < G) tmpM[g] = M;
    }
    __syncthreads();
    for (int i = tid; i < G * ATT_HD; i += NT) {
        const int g = i / ATT_HD, d = i % ATT_HD;
        double sum = 0.0;
#pragma unroll 8
        for (int w = 0; w < NW; w++) sum = __fma_rn(wt[w * G + g], red[(w * G + g) * ATT_HD + d], sum);
        O_s[i] = sum;
    }
    if (tid < G) {
        double l = 0.0;
        for (int w = 0; w < NW; w++) l = __fma_rn(wt[w * G + tid], lw[w * G + tid], l);
        L_s[tid] = l;
        M_s[tid] = tmpM[tid];
    }
    constexpr unsigned wmask = G * S >= 32 ? 0xffffffffu : (1u << (G * S)) - 1u;
    if constexpr (CLUSTER) {
        cg::cluster_group cl = cg::this_cluster();
        __syncthreads();
        cluster_wait();  // every CTA of the cluster has started
        // push: rank r receives dims [r*DPR, (r+1)*DPR) of each head plus (max, sum)
        for (int i = tid; i < S * G * IB; i += NT) {
            const int r = i / (G * IB), g = (i / IB) % G, k = i % IB;
            const double v = k < ATT_DPR ? O_s[g * ATT_HD + r * ATT_DPR + k] : (k == ATT_DPR ? M_s[g] : L_s[g]);
            *cl.map_shared_rank(&inbox[(rank * G + g) * IB + k], r) = v;
        }
        cluster_sync_all();  // every push has landed
        if (tid < G * S) {
            const int g = tid / S, r = tid % S;
            const double Mr = inbox[(r * G + g) * IB + ATT_DPR];
            const double Lr = inbox[(r * G + g) * IB + ATT_DPR + 1];
            double M = Mr;
#pragma unroll
            for (int off = S / 2; off > 0; off >>= 1) M = fmax(M, __shfl_xor_sync(wmask, M, off));
            const double w = Mr == -INFINITY ? 0.0 : exp64(__dsub_rn(Mr, M));
            wts[tid] = w;
            wl[tid] = __dmul_rn(w, Lr);
        }
        __syncthreads();
        if (tid < G * ATT_DPR) {
            const int g = tid / ATT_DPR, dd = tid % ATT_DPR, d = rank * ATT_DPR + dd;
            double L = 0.0, O = 0.0;
#pragma unroll
            for (int r = 0; r < S; r++) {
                L = __dadd_rn(L, wl[g * S + r]);
                O = __dadd_rn(O, __dmul_rn(wts[g * S + r], inbox[(r * G + g) * IB + dd]));
            }
            const float val = L > 0.0 ? __double2float_rn(__ddiv_rn(O, L)) : 0.f;
            if (out_f32) out_f32[((int64_t)b * A.n_heads + (int64_t)kvh * G + g) * ATT_HD + d] = val;
            // Q8_K block g/2 (heads g & ~1, g | 1) is quantized by rank g/2
            if (use_q8) *cl.map_shared_rank(&q8in[(g & 1) * ATT_HD + d], g >> 1) = val;
        }
        if (use_q8) {
            cluster_sync_all();  // the block's 256 values have landed
            if (rank < G / 2 && warp == 0) {
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; e++) v[e] = q8in[8 * lane + e];
                q8k_store_warp_ext(v, lane, aq, b, (int64_t)kvh * G / 2 + rank);
            }
        }
    } else {
        // partial slots per head: the ns splits, then -- more than
        // ATT_MERGE1_MAX splits (a multiple of ATT_GROUP) -- one merged slot per
        // group of ATT_GROUP splits (two-level merge: the last CTA of a group
        // merges its group, the last group merger merges the groups)
        const int ng = ns > ATT_MERGE1_MAX ? ns / ATT_GROUP : 0;
        const int sst = ns + ng;
        const int64_t hb0 = ((int64_t)b * A.n_heads + (int64_t)kvh * G) * sst;
        __syncthreads();
        for (int i = tid; i < G * ATT_HD; i += NT) {
            const int g = i / ATT_HD, d = i % ATT_HD;
            A.part_o[(hb0 + (int64_t)g * sst + rank) * ATT_HD + d] = O_s[i];
        }
        if (tid < G) {
            A.part_ml[2 * (hb0 + (int64_t)tid * sst + rank)] = M_s[tid];
            A.part_ml[2 * (hb0 + (int64_t)tid * sst + rank) + 1] = L_s[tid];
        }
        __threadfence();
        __syncthreads();
        int *cnt = counters + ((int64_t)b * A.n_kv + kvh) * (ng ? ATT_CNT_PER : 1);
        // merges slots [s0, s0 + n) of every head: dst < 0 -> the output
        // (f32 and Q8_K), else a merged partial (max, sum, o) into slot dst
        auto merge = [&](int s0, int n, int dst) {
            if (warp < G) {  // warp g: weights of head g (lane = slots r, r + 32)
                const int g = warp;
                double Mr[ATT_SPLITS_MAX / 32], Lr[ATT_SPLITS_MAX / 32];
                double M = -INFINITY;
#pragma unroll
                for (int k = 0; k < ATT_SPLITS_MAX / 32; k++) {
                    const int r = lane + 32 * k;
                    Mr[k] = r < n ? __ldcg(&A.part_ml[2 * (hb0 + (int64_t)g * sst + s0 + r)]) : -INFINITY;
                    Lr[k] = r < n ? __ldcg(&A.part_ml[2 * (hb0 + (int64_t)g * sst + s0 + r) + 1]) : 0.0;
                    M = fmax(M, Mr[k]);
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) M = fmax(M, __shfl_xor_sync(0xffffffffu, M, off));
#pragma unroll
                for (int k = 0; k < ATT_SPLITS_MAX / 32; k++) {
                    const int r = lane + 32 * k;
                    if (r < n) {
                        const double w = Mr[k] == -INFINITY ? 0.0 : exp64(__dsub_rn(Mr[k], M));
                        wts[g * ATT_SPLITS_MAX + r] = w;
                        wl[g * ATT_SPLITS_MAX + r] = __dmul_rn(w, Lr[k]);
                    }
                }
                if (lane == 0) tmpM[g] = M;
            }
            __syncthreads();
            for (int i = tid; i < G * ATT_HD; i += NT) {
                const int g = i / ATT_HD, d = i % ATT_HD;
                double L = 0.0, O = 0.0;
                for (int r0 = 0; r0 < n; r0 += 16) {  // 16 partial loads in flight, summed in slot order
                    double Or[16];
#pragma unroll
                    for (int k = 0; k < 16; k++)
                        Or[k] = r0 + k < n ? __ldcg(&A.part_o[(hb0 + (int64_t)g * sst + s0 + r0 + k) * ATT_HD + d])
                                           : 0.0;
#pragma unroll
                    for (int k = 0; k < 16; k++)
                        if (r0 + k < n) {
                            L = __dadd_rn(L, wl[g * ATT_SPLITS_MAX + r0 + k]);
                            O = __dadd_rn(O, __dmul_rn(wts[g * ATT_SPLITS_MAX + r0 + k], Or[k]));
                        }
                }
                if (dst >= 0) {
                    A.part_o[(hb0 + (int64_t)g * sst + dst) * ATT_HD + d] = O;
                    if (d == 0) {
                        A.part_ml[2 * (hb0 + (int64_t)g * sst + dst)] = tmpM[g];
                        A.part_ml[2 * (hb0 + (int64_t)g * sst + dst) + 1] = L;
                    }
                } else {
                    const float val = L > 0.0 ? __double2float_rn(__ddiv_rn(O, L)) : 0.f;
                    if (out_f32) out_f32[((int64_t)b * A.n_heads + (int64_t)kvh * G + g) * ATT_HD + d] = val;
                    fin[i] = val;
                }
            }
            if (dst < 0 && use_q8) {
                __syncthreads();
                for (int blk = warp; blk < G / 2; blk += NW) {
                    float v[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) v[e] = fin[blk * 256 + 8 * lane + e];
                    q8k_store_warp_ext(v, lane, aq, b, (int64_t)kvh * G / 2 + blk);
                }
            }
        };
        if (ng == 0) {
            if (tid == 0) {
                const int prev = atomicAdd(&cnt[0], 1);
                s_last = prev == ns - 1;
                if (s_last) {
                    cnt[0] = 0;        // ready for the next call
                    __threadfence();  // the partials' reads below follow the counter
                }
            }
            __syncthreads();
            if (s_last) merge(0, ns, -1);
        } else {
            const int grp = rank / ATT_GROUP;
            if (tid == 0) {
                const int prev = atomicAdd(&cnt[1 + grp], 1);
                s_last = prev == ATT_GROUP - 1;
                if (s_last) cnt[1 + grp] = 0;
            }
            __syncthreads();
            if (s_last) {
                __threadfence();
                merge(grp * ATT_GROUP, ATT_GROUP, ns + grp);
                __threadfence();
                __syncthreads();
                if (tid == 0) {
                    const int prev = atomicAdd(&cnt[0], 1);
                    s_last2 = prev == ng - 1;
                    if (s_last2) cnt[0] = 0;
                }
                __syncthreads();
                if (s_last2) {
                    __threadfence();
                    merge(ns, ng, -1);
                }
            }
        }
    }
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


constexpr int ATT_BT_MAX = 8192;  // block-table entries one CTA stages in shared memory

static int attn_bt_cap(int max_pages, int page_size) {
    const int nch = (int)(((int64_t)max_pages * page_size + ATT_CHUNK - 1) / ATT_CHUNK);
    return (nch + ATT_SPLITS - 1) / ATT_SPLITS * (ATT_CHUNK / page_size);
}

// Whether a cluster of ATT_SPLITS CTAs with this shared-memory footprint can
// be resident on the device (cached per device and size).
template <int G>
static bool attn_cluster_fits(int device, size_t smem) {
    static std::mutex mu;
    static std::map<std::pair<int, size_t>, bool> cache;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_pair(device, smem);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    auto kern = k_attn_decode<G, true>;
    bool fits = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) == cudaSuccess &&
                cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
    if (fits) {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = ATT_SPLITS;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(ATT_SPLITS, 1, 1);
        cfg.blockDim = dim3(32 * att_warps(G, true));
        cfg.dynamicSmemBytes = smem;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        fits = cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n >= 1;
    }
    cudaGetLastError();  // a refused query leaves no sticky error
    cache[key] = fits;
    return fits;
}

template <int G>
static bool attn_plan(fb_ctx *ctx, const AttnArgs &A, int batch, bool want_cluster, int *depth, int *bt_cap,
                      size_t *smem) {
    *bt_cap = attn_bt_cap(A.max_pages, A.page_size);
    // clusters: two stages keep a CTA under half of an SM's shared memory, so
    // a 16-CTA cluster fits a GPC even where other work holds some SMs.
    // Without clusters: four stages (over half of the shared memory, so one
    // CTA per SM: the scheduler spreads the grid over all SMs).
    (void)batch;
    bool cluster = false;
    if (want_cluster) {
        *depth = att_depth(true);
        *smem = attn_layout(G, att_warps(G, true), *depth, *bt_cap).total;
        cluster = attn_cluster_fits<G>(ctx->device, *smem);
    }
    if (!cluster) {
        *depth = att_depth(false);
        *smem = attn_layout(G, att_warps(G, false), *depth, *bt_cap).total;
    }
    return cluster;
}

bool attn_uses_cluster(fb_ctx *ctx, const AttnArgs &A, int batch) {
    int depth, cap;
    size_t smem;
    switch (A.n_heads / A.n_kv) {
        case 1: return attn_plan<1>(ctx, A, batch, true, &depth, &cap, &smem);
        case 2: return attn_plan<2>(ctx, A, batch, true, &depth, &cap, &smem);
        case 4: return attn_plan<4>(ctx, A, batch, true, &depth, &cap, &smem);
        case 8: return attn_plan<8>(ctx, A, batch, true, &depth, &cap, &smem);
        default: return false;
    }
}

template <int G>
static void launch_attn_g(fb_ctx *ctx, const AttnArgs &A, int batch, int max_seq_len, float *out_f32,
                          const Q8Act *aq, int *counters, bool pdl, bool want_cluster) {
    int depth, bt_cap;
    size_t smem;
    const bool cluster = attn_plan<G>(ctx, A, batch, want_cluster, &depth, &bt_cap, &smem);
    // cluster-free merge: as many splits as fill one wave (one CTA per SM;
    // one split per (kv head, sequence) once those alone fill it), each with a
    // chunk of the longest sequence; above ATT_MERGE1_MAX a multiple of
    // ATT_GROUP (two-level merge).  The CTA's block-table entries (shared
    // memory) bound the chunks per split from below.
    int ns = ATT_SPLITS;
    if (!cluster) {
        const int PPC = ATT_CHUNK / A.page_size;
        const int64_t nch = (max_seq_len + ATT_CHUNK - 1) / ATT_CHUNK;
        const int64_t nch_cap = ((int64_t)A.max_pages * A.page_size + ATT_CHUNK - 1) / ATT_CHUNK;
        // at most ATT_MERGE1_MAX splits (one-level merge) unless the block
        // table needs more: with one or two kv heads per GPU (tensor
        // parallel) more splits only lengthen the merge of a small K/V
        int64_t want = std::min<int64_t>({(int64_t)ctx->num_sms / ((int64_t)A.n_kv * batch), (int64_t)A.nsplit_max,
                                          (int64_t)ATT_MERGE1_MAX, nch});
        const int64_t lo = std::max<int64_t>(1, (nch_cap * PPC + ATT_BT_MAX - 1) / ATT_BT_MAX);
        want = std::max(want, lo);
        if (want > ATT_MERGE1_MAX) {
            want -= want % ATT_GROUP;
            if (want < lo) want += ATT_GROUP;
        }
        FB_REQUIRE(want <= ATT_SPLITS_MAX && want <= A.nsplit_max, "attn: block table too long for the split scratch");
        ns = (int)want;
        bt_cap = (int)((nch_cap + ns - 1) / ns) * PPC;
        smem = attn_layout(G, att_warps(G, false), depth, bt_cap).total;
    }
    FB_REQUIRE(cluster || (counters && A.part_o && A.part_ml), "attn: the cluster-free merge needs scratch");
    Q8Act q = aq ? *aq : Q8Act{nullptr, nullptr, nullptr, nullptr, 0};
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    // older KV chunks are read before griddepcontrol.wait: only valid when the
    // preceding kernel is one of this library's (the model's decode step)
    attr[0].val.programmaticStreamSerializationAllowed = (ctx->pdl && pdl) ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = ATT_SPLITS;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.gridDim = dim3(cluster ? ATT_SPLITS : ns, A.n_kv, batch);
    cfg.blockDim = dim3(32 * att_warps(G, cluster));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = cluster ? 2 : 1;
    if (cluster) {
        auto kern = k_attn_decode<G, true>;
        FB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        FB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        FB_CUDA(cudaLaunchKernelEx(&cfg, kern, A, out_f32, q, aq ? 1 : 0, counters, bt_cap));
    } else {
        auto kern = k_attn_decode<G, false>;
        FB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        FB_CUDA(cudaLaunchKernelEx(&cfg, kern, A, out_f32, q, aq ? 1 : 0, counters, bt_cap));
    }
}

// Paged decode attention.  out_f32 and/or (aq != null, needs an even GQA
// group) receive the result.  With want_cluster the 16 splits of each (kv
// head, sequence) merge through distributed shared memory when the device can
// hold such a cluster; otherwise A.part_o / A.part_ml (ATT_SPLITS splits) and
// `counters` (batch * n_kv int32, zero on entry and again on exit) are used.
void launch_attn_decode(fb_ctx *ctx, const AttnArgs &A, int batch, int max_seq_len, float *out_f32, const Q8Act *aq,
                        int *counters, bool pdl, bool want_cluster) {
    const int G = A.n_heads / A.n_kv;
    FB_REQUIRE(A.n_heads % A.n_kv == 0, "attn: n_heads must be a multiple of n_kv_heads");
    FB_REQUIRE(A.page_size == 32 || A.page_size == 64, "attn: page_size must be 32 or 64");
    FB_REQUIRE(!aq || G % 2 == 0, "attn: fused Q8_K output needs an even GQA group");
    FB_REQUIRE(max_seq_len >= 1 && max_seq_len <= A.max_pages * A.page_size, "attn: max_seq_len exceeds the block table");
    switch (G) {
        case 1: launch_attn_g<1>(ctx, A, batch, max_seq_len, out_f32, aq, counters, pdl, want_cluster); break;
        case 2: launch_attn_g<2>(ctx, A, batch, max_seq_len, out_f32, aq, counters, pdl, want_cluster); break;
        case 4: launch_attn_g<4>(ctx, A, batch, max_seq_len, out_f32, aq, counters, pdl, want_cluster); break;
        case 8: launch_attn_g<8>(ctx, A, batch, max_seq_len, out_f32, aq, counters, pdl, want_cluster); break;
        default: fail(FB_ERR_INVALID, "attn: GQA group size must be 1, 2, 4 or 8");
    }
}

// ---------------------------------------------------------------------------
// Allocation-free decode attention (fb_attn_decode_noalloc).
//
// fb_attn_decode merges its 16 splits through distributed shared memory when
// the GPU can hold a 16-CTA cluster, and otherwise takes global split scratch
// from the context's workspace, which is grown with cudaMalloc and a stream
// synchronisation on first use.  Some callers cannot allow that: code running
// under a caching or pooled device allocator that forbids direct
// cudaMalloc/cudaFree (ferrite-os routes device allocations through its own
// TLSF pool), and latency-critical loops that must never take the implicit
// device synchronisation cudaMalloc/cudaFree may cause.  For them this entry
// point always runs the cluster-free merge and keeps its scratch in a fixed,
// file-scope device array instead.
//
// The array is a `static __device__` object: every GPU that loads the library
// holds it until the process exits.  Host code cannot use the array's name as
// a device address (it is a host-side stand-in), so its device address is
// looked up per device with cudaGetSymbolAddress, with that device current,
// the first time the entry point runs on it; that first call should therefore
// come before any stream capture.  All calls on a device share the one array:
// calls that overlap on the GPU (two streams, or two contexts of one device)
// race on it.  The partial sums need no clearing (every slot a call reads is
// written by the same call first); the merge counters at its start must be
// zero, so each call clears them (cudaMemsetAsync, no allocation).
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
                                      int num_pages, int max_seq_len, float scale) {
    using namespace fb;
    return guarded([&] {
        FB_REQUIRE(ctx && q_dev && k_pages_dev && v_pages_dev && block_table_dev && seq_lens_dev && out_dev,
                   "null argument");
        FB_REQUIRE(head_dim == 128, "head_dim must be 128");
        FB_REQUIRE(page_size == 32 || page_size == 64, "page_size must be 32 or 64");
        FB_REQUIRE(batch >= 1 && n_heads >= 1 && n_kv_heads >= 1 && max_pages >= 1 && max_seq_len >= 1,
                   "bad shape");
        FB_REQUIRE(max_seq_len <= max_pages * page_size, "max_seq_len exceeds the block table");
        FB_REQUIRE(num_pages >= 1, "num_pages must be positive");
        const int nsplit = ATT_SPLITS;
        const size_t cnt_bytes = ((size_t)batch * n_kv_heads * sizeof(int) + 255) & ~(size_t)255;
        const size_t need = (size_t)batch * n_heads * nsplit * (head_dim + 2) * sizeof(double) + cnt_bytes;
        if (need > kAttnNoAllocScratchBytes)
            fail(FB_ERR_INVALID, "attn_decode_noalloc: batch * n_heads * " + std::to_string(nsplit) + " splits * " +
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
        A.num_pages = num_pages;  // block-table ids outside the pool set ERRBIT_BAD_PAGE and are skipped
        A.nsplit_max = nsplit;
        A.scale = scale;
        A.err = ctx->err_word;
        launch_attn_decode(ctx, A, batch, max_seq_len, out_dev, nullptr, counters, false, false);
    });
}
