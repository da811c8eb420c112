// Quantized Llama / Qwen3 decode runtime behind fb_model_* — the B200
// counterpart of ferrite-core's InferenceModel implemented for candle at
// crates/ferrite-wasm-host/src/adapter.rs:60-93 (forward / prefill /
// clear_cache), with greedy sampling kept on the device like
// Sampler::argmax (crates/ferrite-core/src/sampling.rs:108-112).
//
// One decode step for a batch of b sequences is a fixed chain of kernels:
//   [embed + RMSNorm + Q8_K]
//   per layer: QKV GEMV -> QK-norm + RoPE + KV write -> flash-decode split
//              -> combine + Q8_K -> O GEMV -> residual + RMSNorm + Q8_K
//              -> gate/up GEMV -> SwiGLU + Q8_K -> down GEMV
//              -> residual + RMSNorm (next layer or final) + Q8_K
//   lm_head GEMV -> argmax
// launched with programmatic dependent launch and captured once per batch
// size into a CUDA graph.  All buffers are allocated up front; the step reads
// token ids and positions from device buffers, so replays need no host work.
//
// Tensor parallel (fb_model_create_tp): the rank keeps its shard of the
// heads, the FFN and the vocab; attn_output and ffn_down push binary64
// partial sums to every rank's inbox and the residual + RMSNorm kernel that
// follows adds them (one exchange per row-parallel projection, no separate
// collective launch); the greedy argmax merges the ranks' (max, index).
#include <cuda_fp16.h>
#include <math.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <memory>
#include <string>

#include "decode_step.h"
#include "fb_internal.h"

using namespace fb;

namespace {

constexpr int kPage = 64;

enum TensorKind {
    T_TOKEN_EMBD = 1, T_OUTPUT_NORM = 2, T_OUTPUT = 3,
    T_ATTN_NORM = 10, T_ATTN_Q, T_ATTN_K, T_ATTN_V, T_ATTN_OUTPUT, T_ATTN_Q_NORM, T_ATTN_K_NORM,
    T_FFN_NORM, T_FFN_GATE, T_FFN_UP, T_FFN_DOWN
};

int kind_of(const char *name) {
    static const std::map<std::string, int> m = {
        {"token_embd", T_TOKEN_EMBD},   {"output_norm", T_OUTPUT_NORM}, {"output", T_OUTPUT},
        {"attn_norm", T_ATTN_NORM},     {"attn_q", T_ATTN_Q},           {"attn_k", T_ATTN_K},
        {"attn_v", T_ATTN_V},           {"attn_output", T_ATTN_OUTPUT}, {"attn_q_norm", T_ATTN_Q_NORM},
        {"attn_k_norm", T_ATTN_K_NORM}, {"ffn_norm", T_FFN_NORM},       {"ffn_gate", T_FFN_GATE},
        {"ffn_up", T_FFN_UP},           {"ffn_down", T_FFN_DOWN}};
    auto it = m.find(name ? name : "");
    return it == m.end() ? 0 : it->second;
}

struct QT {
    fb_qtensor *t = nullptr;
    QT() = default;
    QT(const QT &) = delete;
    QT &operator=(const QT &) = delete;
    ~QT() { fb_qtensor_destroy(t); }
    void reset(fb_qtensor *n = nullptr) {
        fb_qtensor_destroy(t);
        t = n;
    }
};

struct Layer {
    QT wq, wk, wv, wo, wgate, wup, wdown;  // as set
    QT wqkv, wgu;                          // fused by finalize
    DevBuf attn_norm, ffn_norm, q_norm, k_norm;
};

// Per-tensor seed of the random-init model: seed + 0x1000 * (layer + 1) + kind
// (layer = -1 for the global tensors).
uint64_t tensor_seed(uint64_t seed, int layer, int kind) {
    return seed + 0x1000ull * (uint64_t)(layer + 1) + (uint64_t)kind;
}

}  // namespace

struct fb_model {
    fb_ctx *ctx = nullptr;
    fb_model_config c{};   // full model
    fb_model_config lc{};  // this rank's shard: n_heads, n_kv_heads, ffn, vocab divided by the world size
    fb_comm *comm = nullptr;  // tensor parallel when set
    int W = 1, rank = 0, v_off = 0;
    DevBuf epoch, ss_part, ss_tag;  // tensor-parallel step counter and norm exchange slots
    std::vector<std::unique_ptr<Layer>> layers;
    QT tok_embd, output;
    DevBuf out_norm;
    bool finalized = false;
    // KV cache and tables
    int pages_per_seq = 0, num_pages = 0, nsplit_max = 0;
    DevBuf kv;  // [L][K|V][num_pages][n_kv][page][hd] fp16
    DevBuf block_table, rope_cos, rope_sin;
    // step buffers
    DevBuf x, x2, y_qkv, q, attn, y_o, y_gu, y_d, logits, part_o, part_ml, att_cnt, argmax_ws;
    float *x_last = nullptr;  // residual buffer holding the last step's final value
    DevBuf act_h, act_a, act_f;
    DevBuf tok, pos, next;
    int32_t *pinned = nullptr;  // host staging [3 * max_batch]
    cudaStream_t work = nullptr;        // private stream the step graph runs on
    cudaEvent_t ev_in = nullptr, ev_out = nullptr;
    std::map<int, cudaGraphExec_t> graphs;
    int len0 = 0;  // tokens held by sequence slot 0 (forward / prefill API)
    int launches_per_step = 0;
    // persistent decode step (batch 1, single GPU): per-layer tensor table,
    // barrier counters and launch plan; ds_on selects it over the kernel chain
    // (off by default: measured slower than the chain on B200, 3.4-4.1 vs
    // 2.07 ms per Qwen3-8B step -- one 9-warp CTA per SM cannot hide the
    // consumers' latency and each layer pays six grid barriers)
    DevBuf ds_layers, ds_sync;
    DsPlan ds_plan;
    bool ds_ok = false, ds_on = false;
    // batched prefill buffers (allocated on first use, rows = pf_cap)
    DevBuf pf_tok, pf_x, pf_xn, pf_yd, pf_yqkv, pf_q, pf_attn, pf_ygu, pf_act;
    DevBuf pf_xh, pf_rs;  // fp16 GEMM operand rows written by the norm / SwiGLU kernels, their row scales
    int pf_cap = 0;

    size_t kv_half_layer() const { return (size_t)num_pages * lc.n_kv_heads * kPage * c.head_dim; }
    __half *kpool(int l) const { return kv.as<__half>() + (size_t)l * 2 * kv_half_layer(); }
    __half *vpool(int l) const { return kpool(l) + kv_half_layer(); }

    ~fb_model() {
        for (auto &g : graphs) cudaGraphExecDestroy(g.second);
        if (pinned) cudaFreeHost(pinned);
        if (work) cudaStreamDestroy(work);
        if (ev_in) cudaEventDestroy(ev_in);
        if (ev_out) cudaEventDestroy(ev_out);
    }
};

static void upload_f32(fb_ctx *ctx, DevBuf &buf, const void *host, size_t n) {
    buf.alloc(n * 4);
    FB_CUDA(cudaMemcpyAsync(buf.ptr, host, n * 4, cudaMemcpyHostToDevice, ctx->stream));
}

// Optional per-class timing of an eager step (fb_model_profile): one event
// after every kernel class, elapsed times read after the step completes.
struct StepProbe {
    std::vector<cudaEvent_t> ev;
    std::vector<int> kinds;
    float ms[FB_PROF_KINDS] = {0};
    int launches[FB_PROF_KINDS] = {0};
    cudaStream_t s = nullptr;
    ~StepProbe() {
        for (cudaEvent_t e : ev) cudaEventDestroy(e);
    }
    cudaEvent_t next_event() {
        cudaEvent_t e;
        FB_CUDA(cudaEventCreate(&e));
        ev.push_back(e);
        return e;
    }
    void start() {
        FB_CUDA(cudaEventRecord(next_event(), s));
        kinds.push_back(-1);
    }
    void mark(int kind, int nlaunch) {
        FB_CUDA(cudaEventRecord(next_event(), s));
        kinds.push_back(kind);
        launches[kind] += nlaunch;
    }
    void collect() {
        FB_CUDA(cudaStreamSynchronize(s));
        for (size_t i = 1; i < ev.size(); i++) {
            if (kinds[i] < 0) continue;
            float t = 0.f;
            FB_CUDA(cudaEventElapsedTime(&t, ev[i - 1], ev[i]));
            ms[kinds[i]] += t;
        }
    }
};

// Tensor-parallel exchange arguments (comm regions of all ranks as mapped in
// this process).
static PeerOut peer_out(const fb_model *m, size_t inbox_off) {
    const fb_comm *cm = m->comm;
    PeerOut po{};
    for (int p = 0; p < cm->world; p++)
        po.dst[p] = cm->at<uint64_t>(p, inbox_off) + 2 * (size_t)cm->rank * cm->max_batch * cm->hidden;
    po.ld = cm->hidden;
    po.world = cm->world;
    po.epoch = m->epoch.as<uint32_t>();
    po.nx = 2 * m->c.n_layers;
    return po;
}
static TpNorm tp_norm(const fb_model *m, size_t inbox_off) {
    const fb_comm *cm = m->comm;
    TpNorm t{};
    t.inbox = cm->at<uint64_t>(cm->rank, inbox_off);
    t.epoch = m->epoch.as<uint32_t>();
    t.ss_part = m->ss_part.as<double>();
    t.ss_tag = m->ss_tag.as<uint32_t>();
    t.limit_ns = cm->timeout_ns;
    t.world = cm->world;
    t.batch_cap = cm->max_batch;
    t.nx = 2 * m->c.n_layers;
    return t;
}
static TpArgmax tp_argmax(const fb_model *m) {
    const fb_comm *cm = m->comm;
    TpArgmax t{};
    for (int p = 0; p < cm->world; p++) {
        t.peer_slot[p] = cm->at<uint64_t>(p, cm->L.am_inbox) + (size_t)cm->rank * cm->max_batch;
        t.peer_flag[p] = cm->at<uint32_t>(p, cm->L.am_flags) + (size_t)cm->rank * cm->max_batch;
    }
    t.my_inbox = cm->at<uint64_t>(cm->rank, cm->L.am_inbox);
    t.my_flags = cm->at<uint32_t>(cm->rank, cm->L.am_flags);
    t.epoch = m->epoch.as<uint32_t>();
    t.limit_ns = cm->timeout_ns;
    t.world = cm->world;
    t.batch_cap = cm->max_batch;
    t.vocab_off = m->v_off;
    return t;
}

// The batch-1 step as one persistent kernel (decode_step.cu) + argmax.
static bool persistent_step(fb_model *m, int b, StepProbe *probe, unsigned long long *trace = nullptr) {
    if (!(m->ds_ok && m->ds_on && b == 1 && !probe && !m->comm)) return false;
    fb_ctx *ctx = m->ctx;
    const fb_model_config &c = m->c, &lc = m->lc;
    const int qd = lc.n_heads * c.head_dim;
    DsArgs A{};
    A.layers = m->ds_layers.as<DsLayer>();
    A.n_layers = c.n_layers;
    A.H = c.hidden;
    A.F = lc.ffn;
    A.n_heads = lc.n_heads;
    A.n_kv = lc.n_kv_heads;
    A.vocab = lc.vocab;
    A.qkv_n = (lc.n_heads + 2 * lc.n_kv_heads) * c.head_dim;
    A.emb = m->tok_embd.t->main();
    A.out = m->output.t->main();
    A.dt_out = m->output.t->dtype == FB_Q4_K ? 4 : 6;
    A.out_norm = m->out_norm.as<float>();
    A.eps = c.eps;
    A.scale = (float)(1.0 / sqrt((double)c.head_dim));
    A.tok = m->tok.as<int32_t>();
    A.pos = m->pos.as<int32_t>();
    A.kv = m->kv.as<__half>();
    A.kv_layer = m->kv_half_layer();
    A.block_table = m->block_table.as<int32_t>();
    A.pages_per_seq = m->pages_per_seq;
    A.num_pages = m->num_pages;
    A.rope_cos = m->rope_cos.as<float>();
    A.rope_sin = m->rope_sin.as<float>();
    A.rope_rows = c.max_ctx;
    A.rope_mode = c.rope_mode;
    A.qk_norm = c.qk_norm;
    A.xa = m->x.as<float>();
    A.xb = m->x2.as<float>();
    A.y_qkv = m->y_qkv.as<float>();
    A.q_out = m->q.as<float>();
    A.attn = m->attn.as<float>();
    A.y_o = m->y_o.as<float>();
    A.y_gu = m->y_gu.as<float>();
    A.y_d = m->y_d.as<float>();
    A.logits = m->logits.as<float>();
    A.act_a = q8act_view(m->act_a.ptr, c.max_batch, qd);
    A.act_f = q8act_view(m->act_f.ptr, c.max_batch, lc.ffn);
    A.part_o = m->part_o.as<double>();
    A.part_ml = m->part_ml.as<double>();
    A.att_cnt = m->att_cnt.as<int>();
    A.sync = m->ds_sync.as<unsigned>();
    A.err = ctx->err_word;
    A.ns = m->ds_plan.ns;
    A.nstage = m->ds_plan.nstage;
    A.trace = trace;
    launch_decode_step(ctx, A, m->ds_plan.smem);
    launch_argmax(ctx, m->logits.as<float>(), b, lc.vocab, m->next.as<int32_t>(), m->argmax_ws.ptr);
    m->x_last = m->x2.as<float>();
    m->launches_per_step = 2;
    return true;
}

static void step(fb_model *m, int b, StepProbe *probe = nullptr) {
    if (persistent_step(m, b, probe)) return;
    fb_ctx *ctx = m->ctx;
    int nl = 0;
    auto mark = [&](int kind, int n) {
        nl += n;
        if (probe) probe->mark(kind, n);
    };
    if (probe) probe->start();
    const fb_model_config &c = m->c, &lc = m->lc;
    const int H = c.hidden, qd = lc.n_heads * c.head_dim, F = lc.ffn;
    const bool tp = m->comm != nullptr;
    PeerOut po_o{}, po_d{};
    TpNorm tn_o{}, tn_d{};
    TpArgmax tam{};
    if (tp) {
        po_o = peer_out(m, m->comm->L.inbox_o);
        po_d = peer_out(m, m->comm->L.inbox_d);
        tn_o = tp_norm(m, m->comm->L.inbox_o);
        tn_d = tp_norm(m, m->comm->L.inbox_d);
        tam = tp_argmax(m);
    }
    const Q8Act ah = q8act_view(m->act_h.ptr, b, H);
    const Q8Act aa = q8act_view(m->act_a.ptr, b, qd);
    const Q8Act af = q8act_view(m->act_f.ptr, b, F);
    // residual stream ping-pongs between two buffers (the norm kernels read
    // one row while writing the updated row)
    float *xa = m->x.as<float>(), *xb = m->x2.as<float>();
    if (tp)
        launch_embed_rmsnorm_q8k(ctx, xa, m->layers[0]->attn_norm.as<float>(), b, H, c.eps, ah, m->tok_embd.t,
                                 m->tok.as<int32_t>(), c.vocab, m->epoch.as<uint32_t>());
    else
        launch_residual_rmsnorm_q8k(ctx, nullptr, nullptr, xa, m->layers[0]->attn_norm.as<float>(), b, H, c.eps, ah,
                                    m->tok_embd.t, m->tok.as<int32_t>(), c.vocab);
    mark(FB_PROF_EMBED_NORM, 1);
    AttnArgs A{};
    A.q = m->q.as<float>();
    A.block_table = m->block_table.as<int32_t>();
    A.seq_lens = nullptr;
    A.pos = m->pos.as<int32_t>();
    A.part_o = m->part_o.as<double>();
    A.part_ml = m->part_ml.as<double>();
    A.n_heads = lc.n_heads;
    A.n_kv = lc.n_kv_heads;
    A.page_size = kPage;
    A.max_pages = m->pages_per_seq;
    A.num_pages = m->num_pages;
    A.nsplit_max = m->nsplit_max;
    A.scale = (float)(1.0 / sqrt((double)c.head_dim));
    A.err = ctx->err_word;
    // QK-norm, RoPE and the KV-cache write run in the attention prologue
    A.qkv = m->y_qkv.as<float>();
    A.qkv_ld = (int64_t)(lc.n_heads + 2 * lc.n_kv_heads) * c.head_dim;
    A.eps = c.eps;
    A.rope_cos = m->rope_cos.as<float>();
    A.rope_sin = m->rope_sin.as<float>();
    A.rope_rows = c.max_ctx;
    A.rope_mode = c.rope_mode;
    A.q_out = m->q.as<float>();
    for (int l = 0; l < c.n_layers; l++) {
        Layer &L = *m->layers[l];
        launch_gemv(ctx, L.wqkv.t, ah, b, m->y_qkv.as<float>(), L.wqkv.t->n);
        mark(FB_PROF_QKV, 1);
        A.kpool = m->kpool(l);
        A.vpool = m->vpool(l);
        A.q_norm = c.qk_norm ? L.q_norm.as<float>() : nullptr;
        A.k_norm = c.qk_norm ? L.k_norm.as<float>() : nullptr;
        const bool q8_fused = (lc.n_heads / lc.n_kv_heads) % 2 == 0;
        // cluster-free merge: inside the step the 16-CTA clusters would be
        // packed two per SM next to the still-running projection
        launch_attn_decode(ctx, A, b, c.max_ctx, m->attn.as<float>(), q8_fused ? &aa : nullptr,
                           m->att_cnt.as<int>(), true, false);
        if (!q8_fused) launch_quantize_q8k(ctx, m->attn.as<float>(), b, qd, aa);
        mark(FB_PROF_ATTN, q8_fused ? 1 : 2);
        po_o.xi = 2 * l;
        po_d.xi = 2 * l + 1;
        if (tp) launch_gemv_peer(ctx, L.wo.t, aa, b, po_o);
        else launch_gemv(ctx, L.wo.t, aa, b, m->y_o.as<float>(), H);
        mark(FB_PROF_O, 1);
        if (tp)
            launch_tp_residual_rmsnorm_q8k(ctx, xa, xb, L.ffn_norm.as<float>(), b, H, c.eps, ah, tn_o, 2 * l);
        else
            launch_residual_rmsnorm_q8k(ctx, xa, m->y_o.as<float>(), xb, L.ffn_norm.as<float>(), b, H, c.eps, ah,
                                        nullptr, nullptr, c.vocab);
        std::swap(xa, xb);
        mark(FB_PROF_NORM, 1);
        launch_gemv(ctx, L.wgu.t, ah, b, m->y_gu.as<float>(), 2 * F);
        mark(FB_PROF_GATE_UP, 1);
        launch_swiglu_q8k(ctx, m->y_gu.as<float>(), F, b, af);
        mark(FB_PROF_SWIGLU, 1);
        if (tp) launch_gemv_peer(ctx, L.wdown.t, af, b, po_d);
        else launch_gemv(ctx, L.wdown.t, af, b, m->y_d.as<float>(), H);
        mark(FB_PROF_DOWN, 1);
        const float *gn = (l + 1 < c.n_layers) ? m->layers[l + 1]->attn_norm.as<float>() : m->out_norm.as<float>();
        if (tp)
            launch_tp_residual_rmsnorm_q8k(ctx, xa, xb, gn, b, H, c.eps, ah, tn_d, 2 * l + 1);
        else
            launch_residual_rmsnorm_q8k(ctx, xa, m->y_d.as<float>(), xb, gn, b, H, c.eps, ah, nullptr, nullptr,
                                        c.vocab);
        std::swap(xa, xb);
        mark(FB_PROF_NORM, 1);
    }
    m->x_last = xa;
    launch_gemv(ctx, m->output.t, ah, b, m->logits.as<float>(), lc.vocab);
    mark(FB_PROF_LM_HEAD, 1);
    if (tp) launch_argmax_tp(ctx, m->logits.as<float>(), b, lc.vocab, m->next.as<int32_t>(), m->argmax_ws.ptr, tam);
    else launch_argmax(ctx, m->logits.as<float>(), b, lc.vocab, m->next.as<int32_t>(), m->argmax_ws.ptr);
    mark(FB_PROF_ARGMAX, 1);
    m->launches_per_step = nl;
}

// Runs one step; the first call for a batch size runs eagerly and then
// captures the chain into a CUDA graph for later replays.
// The step's kernels are issued on the model's private stream (a captured
// graph cannot live on the legacy default stream), ordered after everything
// queued on the context stream and joined back to it.
struct StreamSwap {
    fb_model *m;
    cudaStream_t user;
    explicit StreamSwap(fb_model *mm) : m(mm), user(mm->ctx->stream) {
        FB_CUDA(cudaEventRecord(m->ev_in, user));
        FB_CUDA(cudaStreamWaitEvent(m->work, m->ev_in, 0));
        m->ctx->stream = m->work;
    }
    ~StreamSwap() {
        m->ctx->stream = user;
        cudaEventRecord(m->ev_out, m->work);
        cudaStreamWaitEvent(user, m->ev_out, 0);
    }
};

static void run_step(fb_model *m, int b) {
    fb_ctx *ctx = m->ctx;
    StreamSwap swap(m);
    auto it = m->graphs.find(b);
    if (it != m->graphs.end()) {
        FB_CUDA(cudaGraphLaunch(it->second, ctx->stream));
        return;
    }
    step(m, b);
    cudaGraph_t g = nullptr;
    FB_CUDA(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
    try {
        step(m, b);
    } catch (...) {
        cudaStreamEndCapture(ctx->stream, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    FB_CUDA(cudaStreamEndCapture(ctx->stream, &g));
    cudaGraphExec_t ge = nullptr;
    const cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    FB_CUDA(e);
    m->graphs[b] = ge;
}

static void require_ready(const fb_model *m) {
    if (!m->finalized) fail(FB_ERR_STATE, "model not finalized (call fb_model_finalize after setting tensors)");
}

static void check_no_device_error(fb_model *m) {
    uint32_t flags = 0;
    FB_CUDA(cudaMemcpyAsync(&flags, m->ctx->err_word, 4, cudaMemcpyDeviceToHost, m->ctx->stream));
    FB_CUDA(cudaStreamSynchronize(m->ctx->stream));
    if (flags) {
        FB_CUDA(cudaMemsetAsync(m->ctx->err_word, 0, 4, m->ctx->stream));
        fail(FB_ERR_DEVICE, "device error word set: 0x" + std::to_string(flags));
    }
}

// Which part of a full tensor a tensor-parallel rank keeps.
enum Shard { SH_ALL, SH_ROWS, SH_COLS };

// Shard of `kind` for this rank: (row0, rows, col0, cols) of the [n, k] tensor.
static void shard_range(const fb_model *m, int kind, int64_t n, int64_t k, int64_t &r0, int64_t &nr, int64_t &c0,
                        int64_t &nc) {
    const fb_model_config &c = m->c, &lc = m->lc;
    const int hd = c.head_dim;
    r0 = 0, nr = n, c0 = 0, nc = k;
    if (m->W == 1) return;
    switch (kind) {
    case T_ATTN_Q: nr = (int64_t)lc.n_heads * hd; r0 = m->rank * nr; break;
    case T_ATTN_K:
    case T_ATTN_V: nr = (int64_t)lc.n_kv_heads * hd; r0 = m->rank * nr; break;
    case T_FFN_GATE:
    case T_FFN_UP: nr = lc.ffn; r0 = m->rank * nr; break;
    case T_OUTPUT: nr = lc.vocab; r0 = m->v_off; break;
    case T_ATTN_OUTPUT: nc = (int64_t)lc.n_heads * hd; c0 = m->rank * nc; break;
    case T_FFN_DOWN: nc = lc.ffn; c0 = m->rank * nc; break;
    default: break;  // token_embd and the norms stay whole
    }
}

// Device QTensor of this rank's shard of a full GGUF tensor (host or device).
static fb_qtensor *make_shard(fb_model *m, int kind, int dtype, int64_t n, int64_t k, const void *src, int on_dev) {
    int64_t r0, nr, c0, nc;
    shard_range(m, kind, n, k, r0, nr, c0, nc);
    fb_qtensor *t = nullptr;
    int rc;
    if (r0 == 0 && nr == n && c0 == 0 && nc == k)
        rc = on_dev ? fb_qtensor_upload_dev(m->ctx, dtype, n, k, src, &t) : fb_qtensor_upload(m->ctx, dtype, n, k, src, &t);
    else
        rc = fb_qtensor_upload_slice(m->ctx, dtype, n, k, src, on_dev, r0, nr, c0, nc, &t);
    if (rc != FB_OK) fail(rc, fb_last_error());
    return t;
}

static void create_model(fb_ctx *ctx, const fb_model_config *cfg, fb_comm *comm, fb_model **out) {
    FB_REQUIRE(ctx && cfg && out, "null argument");
    *out = nullptr;
    const fb_model_config &c = *cfg;
    FB_REQUIRE(c.n_layers > 0 && c.hidden > 0 && c.n_heads > 0 && c.n_kv_heads > 0 && c.ffn > 0 && c.vocab > 0,
               "model dims must be positive");
    FB_REQUIRE(c.head_dim == 128, "head_dim must be 128");
    FB_REQUIRE(c.hidden % 256 == 0 && c.ffn % 256 == 0 && (c.n_heads * c.head_dim) % 256 == 0,
               "hidden, ffn and n_heads*head_dim must be multiples of 256");
    FB_REQUIRE(c.n_heads % c.n_kv_heads == 0, "n_heads must be a multiple of n_kv_heads");
    const int G = c.n_heads / c.n_kv_heads;
    FB_REQUIRE(G == 1 || G == 2 || G == 4 || G == 8, "GQA group must be 1, 2, 4 or 8");
    FB_REQUIRE(c.max_ctx >= 1 && c.max_batch >= 1 && c.max_batch <= 32, "need max_ctx >= 1, 1 <= max_batch <= 32");
    FB_REQUIRE(c.rope_mode == 0 || c.rope_mode == 1, "rope_mode must be 0 or 1");
    auto m = std::make_unique<fb_model>();
    m->ctx = ctx;
    m->c = c;
    m->lc = c;
    if (comm) {
        const int W = comm->world;
        FB_REQUIRE(comm->opened, "comm not opened (fb_comm_open)");
        FB_REQUIRE(comm->ctx->device == ctx->device, "comm belongs to another device");
        FB_REQUIRE(comm->hidden == c.hidden && c.max_batch <= comm->max_batch,
                   "comm was created for another hidden size or a smaller batch");
        FB_REQUIRE(c.n_kv_heads % W == 0, "n_kv_heads must be divisible by the world size");
        FB_REQUIRE(c.ffn % (256 * W) == 0, "ffn / world must be a multiple of 256");
        FB_REQUIRE((c.n_heads / W * c.head_dim) % 256 == 0, "n_heads * head_dim / world must be a multiple of 256");
        FB_REQUIRE(c.vocab % W == 0, "vocab must be divisible by the world size");
        m->comm = comm;
        m->W = W;
        m->rank = comm->rank;
        m->lc.n_heads = c.n_heads / W;
        m->lc.n_kv_heads = c.n_kv_heads / W;
        m->lc.ffn = c.ffn / W;
        m->lc.vocab = c.vocab / W;
        m->v_off = comm->rank * m->lc.vocab;
        m->epoch.alloc(256);
        FB_CUDA(cudaMemsetAsync(m->epoch.ptr, 0, 256, ctx->stream));
        // the step counter restarts: clear the sequence numbers peers left in
        // this rank's flags (ranks create their models before the host barrier
        // that precedes the first step, so no peer is publishing yet)
        FB_CUDA(cudaMemsetAsync(comm->region.as<uint8_t>() + comm->L.flags, 0, comm->L.inbox_o - comm->L.flags,
                                ctx->stream));
        const size_t nslot = (size_t)comm->max_batch * (c.hidden / 256);
        m->ss_part.alloc(nslot * 8);
        m->ss_tag.alloc(nslot * 4);
        FB_CUDA(cudaMemsetAsync(m->ss_tag.ptr, 0, nslot * 4, ctx->stream));
    }
    const fb_model_config &lc = m->lc;
    for (int l = 0; l < c.n_layers; l++) m->layers.push_back(std::make_unique<Layer>());
    m->pages_per_seq = (c.max_ctx + kPage - 1) / kPage;
    m->num_pages = m->pages_per_seq * c.max_batch;
    m->nsplit_max = ATT_SPLITS_MAX;  // cluster-free attention merge scratch (splits per kv head and sequence)
    m->kv.alloc(m->kv_half_layer() * 2 * c.n_layers * sizeof(__half));
    FB_CUDA(cudaMemsetAsync(m->kv.ptr, 0, m->kv.bytes, ctx->stream));
    std::vector<int32_t> bt((size_t)c.max_batch * m->pages_per_seq);
    for (size_t i = 0; i < bt.size(); i++) bt[i] = (int32_t)i;  // slot s owns pages [s*pps, (s+1)*pps)
    m->block_table.alloc(bt.size() * 4);
    FB_CUDA(cudaMemcpyAsync(m->block_table.ptr, bt.data(), bt.size() * 4, cudaMemcpyHostToDevice, ctx->stream));
    std::vector<float> ct, st;
    rope_tables(c.max_ctx, c.head_dim, c.rope_theta, ct, st);
    upload_f32(ctx, m->rope_cos, ct.data(), ct.size());
    upload_f32(ctx, m->rope_sin, st.data(), st.size());
    const int B = c.max_batch, H = c.hidden, qd = lc.n_heads * c.head_dim;
    const int kd = lc.n_kv_heads * c.head_dim;
    m->x.alloc((size_t)B * H * 4);
    m->x2.alloc((size_t)B * H * 4);
    m->y_qkv.alloc((size_t)B * (qd + 2 * kd) * 4);
    m->q.alloc((size_t)B * qd * 4);
    m->attn.alloc((size_t)B * qd * 4);
    m->y_o.alloc((size_t)B * H * 4);
    m->y_gu.alloc((size_t)B * 2 * lc.ffn * 4);
    m->y_d.alloc((size_t)B * H * 4);
    m->logits.alloc((size_t)B * lc.vocab * 4);
    m->argmax_ws.alloc(argmax_ws_bytes(B));
    FB_CUDA(cudaMemsetAsync(m->argmax_ws.ptr, 0, m->argmax_ws.bytes, ctx->stream));
    m->part_o.alloc((size_t)B * lc.n_heads * ATT_SLOTS_MAX * c.head_dim * 8);
    m->part_ml.alloc((size_t)B * lc.n_heads * ATT_SLOTS_MAX * 2 * 8);
    m->att_cnt.alloc((size_t)B * lc.n_kv_heads * ATT_CNT_PER * 4);
    FB_CUDA(cudaMemsetAsync(m->att_cnt.ptr, 0, m->att_cnt.bytes, ctx->stream));
    m->act_h.alloc(q8act_bytes(B, H));
    m->act_a.alloc(q8act_bytes(B, qd));
    m->act_f.alloc(q8act_bytes(B, lc.ffn));
    m->tok.alloc((size_t)B * 4);
    m->pos.alloc((size_t)B * 4);
    m->next.alloc((size_t)B * 4);
    FB_CUDA(cudaMemsetAsync(m->tok.ptr, 0, (size_t)B * 4, ctx->stream));
    FB_CUDA(cudaMemsetAsync(m->pos.ptr, 0, (size_t)B * 4, ctx->stream));
    FB_CUDA(cudaMallocHost(&m->pinned, (size_t)3 * B * 4));
    FB_CUDA(cudaStreamCreateWithFlags(&m->work, cudaStreamNonBlocking));
    FB_CUDA(cudaEventCreateWithFlags(&m->ev_in, cudaEventDisableTiming));
    FB_CUDA(cudaEventCreateWithFlags(&m->ev_out, cudaEventDisableTiming));
    FB_CUDA(cudaStreamSynchronize(ctx->stream));
    *out = m.release();
}

extern "C" {

int fb_model_create(fb_ctx *ctx, const fb_model_config *cfg, fb_model **out) {
    return guarded([&] { create_model(ctx, cfg, nullptr, out); });
}

int fb_model_create_tp(fb_ctx *ctx, const fb_model_config *cfg, fb_comm *comm, fb_model **out) {
    return guarded([&] {
        FB_REQUIRE(comm, "null comm");
        create_model(ctx, cfg, comm, out);
    });
}

int fb_model_tp_info(const fb_model *m, int *rank, int *world, int *vocab_offset, int *vocab_count) {
    return guarded([&] {
        FB_REQUIRE(m, "null model");
        if (rank) *rank = m->rank;
        if (world) *world = m->W;
        if (vocab_offset) *vocab_offset = m->v_off;
        if (vocab_count) *vocab_count = m->lc.vocab;
    });
}

int fb_model_destroy(fb_model *m) {
    return guarded([&] {
        if (!m) return;
        cudaStreamSynchronize(m->ctx->stream);
        delete m;
    });
}

int fb_model_set_tensor(fb_model *m, const char *name, int layer, int dtype, int64_t rows, int64_t cols,
                        const void *data_host) {
    return guarded([&] {
        FB_REQUIRE(m && name && data_host, "null argument");
        FB_REQUIRE(!m->finalized, "model already finalized");
        const fb_model_config &c = m->c;
        const int kind = kind_of(name);
        FB_REQUIRE(kind != 0, std::string("unknown tensor name: ") + name);
        const bool global = kind < T_ATTN_NORM;
        if (global) FB_REQUIRE(layer < 0, "global tensors take layer = -1");
        else FB_REQUIRE(layer >= 0 && layer < c.n_layers, "layer index out of range");
        const int qd = c.n_heads * c.head_dim, kd = c.n_kv_heads * c.head_dim;
        auto vec = [&](DevBuf &buf, int64_t n) {
            FB_REQUIRE(dtype == FB_F32 && rows * cols == n, std::string(name) + ": expected f32 vector");
            upload_f32(m->ctx, buf, data_host, (size_t)n);
        };
        auto mat = [&](QT &slot, int64_t r, int64_t k, bool allow_q6, bool allow_q4) {
            FB_REQUIRE(rows == r && cols == k, std::string(name) + ": shape mismatch");
            FB_REQUIRE((dtype == FB_Q6_K && allow_q6) || (dtype == FB_Q4_K && allow_q4),
                       std::string(name) + ": unsupported dtype");
            slot.reset(make_shard(m, kind, dtype, r, k, data_host, 0));
        };
        switch (kind) {
        case T_TOKEN_EMBD: mat(m->tok_embd, c.vocab, c.hidden, false, true); break;
        case T_OUTPUT_NORM: vec(m->out_norm, c.hidden); break;
        case T_OUTPUT: mat(m->output, c.vocab, c.hidden, true, true); break;
        default: {
            Layer &L = *m->layers[layer];
            switch (kind) {
            case T_ATTN_NORM: vec(L.attn_norm, c.hidden); break;
            case T_ATTN_Q: mat(L.wq, qd, c.hidden, true, true); break;
            case T_ATTN_K: mat(L.wk, kd, c.hidden, true, true); break;
            case T_ATTN_V: mat(L.wv, kd, c.hidden, true, true); break;
            case T_ATTN_OUTPUT: mat(L.wo, c.hidden, qd, true, true); break;
            case T_ATTN_Q_NORM: vec(L.q_norm, c.head_dim); break;
            case T_ATTN_K_NORM: vec(L.k_norm, c.head_dim); break;
            case T_FFN_NORM: vec(L.ffn_norm, c.hidden); break;
            case T_FFN_GATE: mat(L.wgate, c.ffn, c.hidden, true, true); break;
            case T_FFN_UP: mat(L.wup, c.ffn, c.hidden, true, true); break;
            case T_FFN_DOWN: mat(L.wdown, c.hidden, c.ffn, true, true); break;
            }
        }
        }
    });
}

int fb_model_synth(fb_model *m, uint64_t seed) {
    return guarded([&] {
        FB_REQUIRE(m, "null model");
        FB_REQUIRE(!m->finalized, "model already finalized");
        fb_ctx *ctx = m->ctx;
        const fb_model_config &c = m->c;
        const int qd = c.n_heads * c.head_dim, kd = c.n_kv_heads * c.head_dim;
        const float sigma = 0.02f;
        DevBuf staging;  // full GGUF tensor when sharding
        auto mat_kind = [&](QT &slot, int kind, int dtype, int64_t r, int64_t k, uint64_t s) {
            int64_t r0, nr, c0, nc;
            shard_range(m, kind, r, k, r0, nr, c0, nc);
            if (nr == r && nc == k) {
                fb_qtensor *t = nullptr;
                const int rc = fb_qtensor_synth(ctx, dtype, r, k, s, sigma, &t);
                if (rc != FB_OK) fail(rc, fb_last_error());
                slot.reset(t);
                return;
            }
            const size_t bytes = (size_t)(r * (k / 256)) * (dtype == FB_Q4_K ? 144 : 210);
            if (staging.bytes < bytes) staging.alloc(bytes);
            launch_synth(ctx, dtype, r * (k / 256), s, sigma, staging.ptr);
            slot.reset(make_shard(m, kind, dtype, r, k, staging.ptr, 1));
        };
        auto vec = [&](DevBuf &buf, int64_t n, uint64_t s) {
            buf.alloc((size_t)n * 4);
            launch_synth_f32(ctx, buf.as<float>(), n, s, 1.0f, 0.02f);
        };
        auto mat = [&](QT &slot, int kind, int dtype, int64_t r, int64_t k, int layer) {
            mat_kind(slot, kind, dtype, r, k, tensor_seed(seed, layer, kind));
        };
        mat(m->tok_embd, T_TOKEN_EMBD, FB_Q4_K, c.vocab, c.hidden, -1);
        vec(m->out_norm, c.hidden, tensor_seed(seed, -1, T_OUTPUT_NORM));
        mat(m->output, T_OUTPUT, FB_Q6_K, c.vocab, c.hidden, -1);
        for (int l = 0; l < c.n_layers; l++) {
            Layer &L = *m->layers[l];
            vec(L.attn_norm, c.hidden, tensor_seed(seed, l, T_ATTN_NORM));
            mat(L.wq, T_ATTN_Q, FB_Q4_K, qd, c.hidden, l);
            mat(L.wk, T_ATTN_K, FB_Q4_K, kd, c.hidden, l);
            mat(L.wv, T_ATTN_V, FB_Q4_K, kd, c.hidden, l);
            mat(L.wo, T_ATTN_OUTPUT, FB_Q4_K, c.hidden, qd, l);
            vec(L.q_norm, c.head_dim, tensor_seed(seed, l, T_ATTN_Q_NORM));
            vec(L.k_norm, c.head_dim, tensor_seed(seed, l, T_ATTN_K_NORM));
            vec(L.ffn_norm, c.hidden, tensor_seed(seed, l, T_FFN_NORM));
            mat(L.wgate, T_FFN_GATE, FB_Q4_K, c.ffn, c.hidden, l);
            mat(L.wup, T_FFN_UP, FB_Q4_K, c.ffn, c.hidden, l);
            mat(L.wdown, T_FFN_DOWN, FB_Q6_K, c.hidden, c.ffn, l);
        }
        FB_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int fb_model_finalize(fb_model *m) {
    return guarded([&] {
        FB_REQUIRE(m, "null model");
        if (m->finalized) return;
        fb_ctx *ctx = m->ctx;
        const fb_model_config &c = m->c;
        FB_REQUIRE(m->tok_embd.t && m->output.t && m->out_norm.ptr, "token_embd, output and output_norm are required");
        for (int l = 0; l < c.n_layers; l++) {
            Layer &L = *m->layers[l];
            FB_REQUIRE(L.wq.t && L.wk.t && L.wv.t && L.wo.t && L.wgate.t && L.wup.t && L.wdown.t && L.attn_norm.ptr &&
                           L.ffn_norm.ptr,
                       "layer " + std::to_string(l) + " is missing tensors");
            if (c.qk_norm) FB_REQUIRE(L.q_norm.ptr && L.k_norm.ptr, "qk_norm needs attn_q_norm / attn_k_norm");
            FB_REQUIRE(L.wq.t->dtype == L.wk.t->dtype && L.wq.t->dtype == L.wv.t->dtype,
                       "attn_q/k/v must share a dtype");
            FB_REQUIRE(L.wgate.t->dtype == L.wup.t->dtype, "ffn_gate/up must share a dtype");
            const fb_qtensor *qkv[3] = {L.wq.t, L.wk.t, L.wv.t};
            fb_qtensor *f = nullptr;
            int rc = fb_qtensor_concat_rows(ctx, qkv, 3, &f);
            if (rc != FB_OK) fail(rc, fb_last_error());
            L.wqkv.reset(f);
            const fb_qtensor *gu[2] = {L.wgate.t, L.wup.t};
            rc = fb_qtensor_concat_rows(ctx, gu, 2, &f);
            if (rc != FB_OK) fail(rc, fb_last_error());
            L.wgu.reset(f);
            L.wq.reset();
            L.wk.reset();
            L.wv.reset();
            L.wgate.reset();
            L.wup.reset();
        }
        // the persistent batch-1 step, where the shape allows it
        const fb_model_config &lc = m->lc;
        bool dt_ok = m->tok_embd.t->dtype == FB_Q4_K;
        for (int l = 0; l < c.n_layers && dt_ok; l++) {
            const Layer &L = *m->layers[l];
            for (const fb_qtensor *t : {L.wqkv.t, L.wo.t, L.wgu.t, L.wdown.t, m->output.t})
                dt_ok = dt_ok && (t->dtype == FB_Q4_K || t->dtype == FB_Q6_K);
        }
        m->ds_ok = !m->comm && dt_ok &&
                   decode_step_plan(ctx, c.hidden, lc.ffn, lc.n_heads, lc.n_kv_heads, m->pages_per_seq, kPage,
                                    &m->ds_plan);
        if (m->ds_ok) {
            std::vector<DsLayer> tab((size_t)c.n_layers);
            auto dt = [](const fb_qtensor *t) { return t->dtype == FB_Q4_K ? 4 : 6; };
            for (int l = 0; l < c.n_layers; l++) {
                const Layer &L = *m->layers[l];
                DsLayer &d = tab[(size_t)l];
                d.qkv = L.wqkv.t->main();
                d.o = L.wo.t->main();
                d.gu = L.wgu.t->main();
                d.down = L.wdown.t->main();
                d.dt_qkv = dt(L.wqkv.t);
                d.dt_o = dt(L.wo.t);
                d.dt_gu = dt(L.wgu.t);
                d.dt_down = dt(L.wdown.t);
                d.attn_norm = L.attn_norm.as<float>();
                d.ffn_norm = L.ffn_norm.as<float>();
                d.q_norm = c.qk_norm ? L.q_norm.as<float>() : nullptr;
                d.k_norm = c.qk_norm ? L.k_norm.as<float>() : nullptr;
            }
            m->ds_layers.alloc(tab.size() * sizeof(DsLayer));
            FB_CUDA(cudaMemcpyAsync(m->ds_layers.ptr, tab.data(), tab.size() * sizeof(DsLayer), cudaMemcpyHostToDevice,
                                    ctx->stream));
            m->ds_sync.alloc(256);
            FB_CUDA(cudaMemsetAsync(m->ds_sync.ptr, 0, 256, ctx->stream));
            FB_CUDA(cudaStreamSynchronize(ctx->stream));
        }
        m->finalized = true;
    });
}

int fb_model_set_persistent(fb_model *m, int enable, int *supported) {
    return guarded([&] {
        FB_REQUIRE(m, "null model");
        require_ready(m);
        if (supported) *supported = m->ds_ok ? 1 : 0;
        const bool on = enable != 0;
        if (on != m->ds_on) {
            FB_CUDA(cudaStreamSynchronize(m->ctx->stream));
            for (auto &g : m->graphs) cudaGraphExecDestroy(g.second);
            m->graphs.clear();
            m->ds_on = on;
        }
    });
}

int fb_model_decode_dev(fb_model *m, const int32_t *tokens_dev, const int32_t *pos_dev, int batch, int32_t *next_dev,
                        float *logits_dev) {
    return guarded([&] {
        FB_REQUIRE(m && tokens_dev && pos_dev, "null argument");
        require_ready(m);
        FB_REQUIRE(batch >= 1 && batch <= m->c.max_batch, "batch out of range");
        cudaStream_t s = m->ctx->stream;
        FB_CUDA(cudaMemcpyAsync(m->tok.ptr, tokens_dev, (size_t)batch * 4, cudaMemcpyDeviceToDevice, s));
        FB_CUDA(cudaMemcpyAsync(m->pos.ptr, pos_dev, (size_t)batch * 4, cudaMemcpyDeviceToDevice, s));
        run_step(m, batch);
        if (next_dev) FB_CUDA(cudaMemcpyAsync(next_dev, m->next.ptr, (size_t)batch * 4, cudaMemcpyDeviceToDevice, s));
        if (logits_dev)
            FB_CUDA(cudaMemcpyAsync(logits_dev, m->logits.ptr, (size_t)batch * m->lc.vocab * 4,
                                    cudaMemcpyDeviceToDevice, s));
    });
}

int fb_model_decode_greedy(fb_model *m, const int32_t *tokens_host, const int32_t *pos_host, int batch,
                           int32_t *next_host) {
    return guarded([&] {
        FB_REQUIRE(m && tokens_host && pos_host && next_host, "null argument");
        require_ready(m);
        FB_REQUIRE(batch >= 1 && batch <= m->c.max_batch, "batch out of range");
        for (int i = 0; i < batch; i++) {
            FB_REQUIRE(tokens_host[i] >= 0 && tokens_host[i] < m->c.vocab, "token id out of range");
            FB_REQUIRE(pos_host[i] >= 0 && pos_host[i] < m->c.max_ctx, "position out of range");
        }
        cudaStream_t s = m->ctx->stream;
        int32_t *pt = m->pinned, *pp = m->pinned + m->c.max_batch, *pn = m->pinned + 2 * m->c.max_batch;
        memcpy(pt, tokens_host, (size_t)batch * 4);
        memcpy(pp, pos_host, (size_t)batch * 4);
        FB_CUDA(cudaMemcpyAsync(m->tok.ptr, pt, (size_t)batch * 4, cudaMemcpyHostToDevice, s));
        FB_CUDA(cudaMemcpyAsync(m->pos.ptr, pp, (size_t)batch * 4, cudaMemcpyHostToDevice, s));
        run_step(m, batch);
        FB_CUDA(cudaMemcpyAsync(pn, m->next.ptr, (size_t)batch * 4, cudaMemcpyDeviceToHost, s));
        FB_CUDA(cudaStreamSynchronize(s));
        memcpy(next_host, pn, (size_t)batch * 4);
        if (pos_host[0] + 1 > m->len0) m->len0 = pos_host[0] + 1;
        check_no_device_error(m);
    });
}

}  // extern "C"

// Batched prefill of slot 0 (prompt tokens at positions pos0 .. pos0 + T - 1):
// the projections run as tensor-core GEMMs over all T rows (the float form
// candle's CUDA QMatMul uses for more than 8 rows), the attention as one
// causal prefill kernel per layer, and the last row's lm_head in float as
// well (dequantized weights, binary64 accumulation): an integer lm_head
// would re-quantize the last hidden row to 8 bits and turn the prompt
// pass's 16-bit-operand differences into ~20x larger logit differences.
static constexpr int kPrefillRows = 2048;   // rows per chunk
static constexpr int kPrefillMinRows = 17;  // shorter prompts go token by token

static void ensure_prefill(fb_model *m, int T) {
    if (m->pf_cap >= T) return;
    const fb_model_config &c = m->c, &lc = m->lc;
    const size_t H = c.hidden, qd = (size_t)lc.n_heads * c.head_dim, kd = (size_t)lc.n_kv_heads * c.head_dim;
    m->pf_tok.alloc((size_t)T * 4);
    m->pf_x.alloc((size_t)T * H * 4);
    m->pf_xn.alloc((size_t)T * H * 4);
    m->pf_yd.alloc((size_t)T * H * 4);
    m->pf_yqkv.alloc((size_t)T * (qd + 2 * kd) * 4);
    m->pf_q.alloc((size_t)T * qd * 4);
    m->pf_attn.alloc((size_t)T * qd * 4);
    m->pf_ygu.alloc((size_t)T * 2 * lc.ffn * 4);
    m->pf_act.alloc((size_t)T * lc.ffn * 4);
    m->pf_xh.alloc((size_t)T * std::max<size_t>(H, lc.ffn) * 2);
    m->pf_rs.alloc((size_t)T * 4);
    m->pf_cap = T;
}

// all_logits != null: the logits of every row [T][vocab] (prefill GEMM over
// the final-normed rows) instead of the last row's float lm_head + argmax.
static void prefill_chunk(fb_model *m, int T, int pos0, float *all_logits = nullptr) {
    fb_ctx *ctx = m->ctx;
    const fb_model_config &c = m->c, &lc = m->lc;
    const int H = c.hidden, qd = lc.n_heads * c.head_dim, kd = lc.n_kv_heads * c.head_dim, F = lc.ffn;
    float *x = m->pf_x.as<float>(), *xn = m->pf_xn.as<float>(), *yd = m->pf_yd.as<float>();
    const int32_t *bt = m->block_table.as<int32_t>();  // slot 0's row
    const float scale = (float)(1.0 / sqrt((double)c.head_dim));
    __half *xh = m->pf_xh.as<__half>();
    float *rs = m->pf_rs.as<float>();
    // residual add + RMSNorm rows feeding a projection
    auto norm_then_gemm = [&](const float *add, const float *gain, const fb_qtensor *w, float *out) {
        if (prefill_gemm_supported(w, T)) {
            launch_add_rmsnorm_rows(ctx, x, add, gain, nullptr, T, H, c.eps, xh, rs);
            prefill_gemm_x16(ctx, w, xh, rs, out, T);
        } else {
            launch_add_rmsnorm_rows(ctx, x, add, gain, xn, T, H, c.eps);
            qmatmul_prefill(ctx, w, xn, out, T);
        }
    };
    launch_embed_rows(ctx, m->tok_embd.t, m->pf_tok.as<int32_t>(), T, c.vocab, H, x);
    for (int l = 0; l < c.n_layers; l++) {
        Layer &L = *m->layers[l];
        // x += down projection of the previous layer; xn = attn_norm(x), as
        // the fp16 GEMM operand when the projection takes the tensor-core path
        norm_then_gemm(l ? yd : nullptr, L.attn_norm.as<float>(), L.wqkv.t, m->pf_yqkv.as<float>());
        launch_prefill_qkv_rope(ctx, m->pf_yqkv.as<float>(), qd + 2 * kd, T, pos0, lc.n_heads, lc.n_kv_heads,
                                c.qk_norm ? L.q_norm.as<float>() : nullptr,
                                c.qk_norm ? L.k_norm.as<float>() : nullptr, c.eps, m->rope_cos.as<float>(),
                                m->rope_sin.as<float>(), c.rope_mode, m->pf_q.as<float>(), m->kpool(l), m->vpool(l),
                                bt, kPage, m->num_pages);
        launch_attn_prefill(ctx, m->pf_q.as<float>(), m->kpool(l), m->vpool(l), bt, m->pages_per_seq, m->num_pages,
                            pos0, T, lc.n_heads, lc.n_kv_heads, scale, m->pf_attn.as<float>());
        qmatmul_prefill(ctx, L.wo.t, m->pf_attn.as<float>(), yd, T);
        norm_then_gemm(yd, L.ffn_norm.as<float>(), L.wgu.t, m->pf_ygu.as<float>());
        if (prefill_gemm_supported(L.wdown.t, T)) {
            launch_swiglu_rows_x16(ctx, m->pf_ygu.as<float>(), F, T, xh, rs);
            prefill_gemm_x16(ctx, L.wdown.t, xh, rs, yd, T);
        } else {
            launch_swiglu_rows(ctx, m->pf_ygu.as<float>(), F, T, m->pf_act.as<float>());
            qmatmul_prefill(ctx, L.wdown.t, m->pf_act.as<float>(), yd, T);
        }
    }
    if (all_logits) {
        launch_add_rmsnorm_rows(ctx, x, yd, m->out_norm.as<float>(), xn, T, H, c.eps);
        qmatmul_prefill(ctx, m->output.t, xn, all_logits, T);
        return;
    }
    // last row: x + down, final RMSNorm, float lm_head, argmax
    float *xl = x + (size_t)(T - 1) * H, *xnl = xn + (size_t)(T - 1) * H;
    launch_add_rmsnorm_rows(ctx, xl, yd + (size_t)(T - 1) * H, m->out_norm.as<float>(), xnl, 1, H, c.eps);
    FB_CUDA(cudaMemcpyAsync(m->x.ptr, xl, (size_t)H * 4, cudaMemcpyDeviceToDevice, ctx->stream));
    m->x_last = m->x.as<float>();
    launch_gemv_float(ctx, m->output.t, xnl, m->logits.as<float>());
    launch_argmax(ctx, m->logits.as<float>(), 1, lc.vocab, m->next.as<int32_t>(), m->argmax_ws.ptr);
}

// Rows of the next chunk when `rem` rows are left: at most `cap`, and never
// leaving a tail shorter than the tensor-core GEMM's 17 rows.
static int chunk_rows(int rem, int cap) {
    if (rem <= cap) return rem;
    return rem - cap < kPrefillMinRows ? rem / 2 : cap;
}

static void prefill_batched(fb_model *m, const int32_t *tokens_host, int n, int pos) {
    cudaStream_t s = m->ctx->stream;
    for (int done = 0; done < n;) {
        const int T = chunk_rows(n - done, kPrefillRows);
        ensure_prefill(m, std::min(kPrefillRows, n));
        FB_CUDA(cudaMemcpyAsync(m->pf_tok.ptr, tokens_host + done, (size_t)T * 4, cudaMemcpyHostToDevice, s));
        prefill_chunk(m, T, pos + done);
        FB_CUDA(cudaStreamSynchronize(s));  // host tokens are pageable: keep them alive until copied
        done += T;
    }
}

extern "C" {

int fb_model_forward_all(fb_model *m, const int32_t *tokens_host, int n, int pos, float *logits_host) {
    return guarded([&] {
        FB_REQUIRE(m && tokens_host && logits_host, "null argument");
        require_ready(m);
        FB_REQUIRE(n >= 1 && pos >= 0 && pos + n <= m->c.max_ctx, "tokens do not fit the KV capacity");
        FB_REQUIRE(pos <= m->len0, "pos beyond the cached sequence");
        for (int i = 0; i < n; i++)
            FB_REQUIRE(tokens_host[i] >= 0 && tokens_host[i] < m->c.vocab, "token id out of range");
        cudaStream_t s = m->ctx->stream;
        const size_t V = (size_t)m->lc.vocab;
        if (n >= kPrefillMinRows && !m->comm && m->output.t->n % 128 == 0) {
            constexpr int kRows = 256;  // rows per chunk: logits [256][vocab] on the device
            DevBuf lg;
            lg.alloc((size_t)std::min(kRows, n) * V * 4);
            ensure_prefill(m, std::min(kRows, n));
            for (int done = 0; done < n;) {
                const int T = chunk_rows(n - done, kRows);
                if (T > m->pf_cap) ensure_prefill(m, T);
                if ((size_t)T * V * 4 > lg.bytes) lg.alloc((size_t)T * V * 4);
                FB_CUDA(cudaMemcpyAsync(m->pf_tok.ptr, tokens_host + done, (size_t)T * 4, cudaMemcpyHostToDevice, s));
                prefill_chunk(m, T, pos + done, lg.as<float>());
                FB_CUDA(cudaMemcpyAsync(logits_host + (size_t)done * V, lg.ptr, (size_t)T * V * 4,
                                        cudaMemcpyDeviceToHost, s));
                FB_CUDA(cudaStreamSynchronize(s));
                done += T;
            }
        } else {
            for (int i = 0; i < n; i++) {
                m->pinned[0] = tokens_host[i];
                m->pinned[1] = pos + i;
                FB_CUDA(cudaMemcpyAsync(m->tok.ptr, &m->pinned[0], 4, cudaMemcpyHostToDevice, s));
                FB_CUDA(cudaMemcpyAsync(m->pos.ptr, &m->pinned[1], 4, cudaMemcpyHostToDevice, s));
                run_step(m, 1);
                FB_CUDA(cudaMemcpyAsync(logits_host + (size_t)i * V, m->logits.ptr, V * 4, cudaMemcpyDeviceToHost, s));
                FB_CUDA(cudaStreamSynchronize(s));
            }
        }
        m->len0 = pos + n;
        check_no_device_error(m);
    });
}

int fb_model_forward(fb_model *m, const int32_t *tokens_host, int n, int pos, float *logits_host) {
    return guarded([&] {
        FB_REQUIRE(m && tokens_host, "null argument");
        require_ready(m);
        FB_REQUIRE(n >= 1 && pos >= 0 && pos + n <= m->c.max_ctx, "tokens do not fit the KV capacity");
        FB_REQUIRE(pos <= m->len0, "pos beyond the cached sequence");
        for (int i = 0; i < n; i++)
            FB_REQUIRE(tokens_host[i] >= 0 && tokens_host[i] < m->c.vocab, "token id out of range");
        cudaStream_t s = m->ctx->stream;
        if (n >= kPrefillMinRows && !m->comm) {
            prefill_batched(m, tokens_host, n, pos);
            m->len0 = pos + n;
            if (logits_host)
                FB_CUDA(cudaMemcpyAsync(logits_host, m->logits.ptr, (size_t)m->lc.vocab * 4, cudaMemcpyDeviceToHost,
                                        s));
            FB_CUDA(cudaStreamSynchronize(s));
            check_no_device_error(m);
            return;
        }
        // token by token through the decode step (causal by construction)
        for (int i = 0; i < n; i++) {
            m->pinned[0] = tokens_host[i];
            m->pinned[1] = pos + i;
            FB_CUDA(cudaMemcpyAsync(m->tok.ptr, &m->pinned[0], 4, cudaMemcpyHostToDevice, s));
            FB_CUDA(cudaMemcpyAsync(m->pos.ptr, &m->pinned[1], 4, cudaMemcpyHostToDevice, s));
            run_step(m, 1);
            FB_CUDA(cudaStreamSynchronize(s));  // pinned staging is reused next iteration
        }
        m->len0 = pos + n;
        if (logits_host)  // this rank's vocab slice under tensor parallelism
            FB_CUDA(cudaMemcpyAsync(logits_host, m->logits.ptr, (size_t)m->lc.vocab * 4, cudaMemcpyDeviceToHost, s));
        FB_CUDA(cudaStreamSynchronize(s));
        check_no_device_error(m);
    });
}

int fb_model_prefill(fb_model *m, const int32_t *tokens_host, int n, float *logits_host) {
    return fb_model_forward(m, tokens_host, n, 0, logits_host);
}

int fb_model_clear_cache(fb_model *m) {
    return guarded([&] {
        FB_REQUIRE(m, "null model");
        m->len0 = 0;
    });
}

int fb_model_synth_kv(fb_model *m, uint64_t seed, int ctx, float scale) {
    return guarded([&] {
        FB_REQUIRE(m, "null model");
        FB_REQUIRE(ctx >= 0 && ctx <= m->c.max_ctx, "ctx out of range");
        const fb_model_config &c = m->c;
        for (int l = 0; l < c.n_layers; l++)
            for (int which = 0; which < 2; which++)
                launch_synth_kv(m->ctx, which ? (void *)m->vpool(l) : (void *)m->kpool(l), l, which, ctx,
                                m->lc.n_kv_heads, c.head_dim, kPage, m->block_table.as<int32_t>(), m->pages_per_seq,
                                c.max_batch, seed, scale, m->rank * m->lc.n_kv_heads);
        FB_CUDA(cudaStreamSynchronize(m->ctx->stream));
        m->len0 = ctx;
    });
}

int fb_model_read_kv(fb_model *m, int layer, int which, int pos, float *out_host) {
    return guarded([&] {
        FB_REQUIRE(m && out_host, "null argument");
        const fb_model_config &c = m->lc;  // this rank's kv heads
        FB_REQUIRE(layer >= 0 && layer < c.n_layers && (which == 0 || which == 1) && pos >= 0 && pos < c.max_ctx,
                   "index out of range");
        const __half *pool = which ? m->vpool(layer) : m->kpool(layer);
        const int page = pos / kPage;  // slot 0 uses pages [0, pages_per_seq)
        std::vector<__half> tmp((size_t)c.head_dim);
        for (int h = 0; h < c.n_kv_heads; h++) {
            if (which == 0) {  // K pages are dim-major: gather one column
                const __half *src = pool + ((size_t)page * c.n_kv_heads + h) * c.head_dim * kPage + (pos % kPage);
                FB_CUDA(cudaMemcpy2DAsync(tmp.data(), 2, src, (size_t)kPage * 2, 2, (size_t)c.head_dim,
                                          cudaMemcpyDeviceToHost, m->ctx->stream));
            } else {
                const __half *src = pool + (((size_t)page * c.n_kv_heads + h) * kPage + (pos % kPage)) * c.head_dim;
                FB_CUDA(cudaMemcpyAsync(tmp.data(), src, (size_t)c.head_dim * 2, cudaMemcpyDeviceToHost,
                                        m->ctx->stream));
            }
            FB_CUDA(cudaStreamSynchronize(m->ctx->stream));
            for (int d = 0; d < c.head_dim; d++) out_host[h * c.head_dim + d] = __half2float(tmp[d]);
        }
    });
}

int fb_model_weight_bytes(const fb_model *m, int64_t *bytes) {
    return guarded([&] {
        FB_REQUIRE(m && bytes, "null argument");
        int64_t tot = 0;
        auto add = [&](const QT &q) {
            if (q.t) tot += (int64_t)q.t->buf.bytes;
        };
        add(m->tok_embd);
        add(m->output);
        for (const auto &Lp : m->layers) {
            const Layer &L = *Lp;
            add(L.wq), add(L.wk), add(L.wv), add(L.wo), add(L.wgate), add(L.wup), add(L.wdown);
            add(L.wqkv), add(L.wgu);
        }
        *bytes = tot;
    });
}

int fb_model_profile(fb_model *m, const int32_t *tokens_dev, const int32_t *pos_dev, int batch, int steps,
                     float *ms_out, int *launches_out) {
    return guarded([&] {
        FB_REQUIRE(m && tokens_dev && pos_dev && ms_out, "null argument");
        require_ready(m);
        FB_REQUIRE(batch >= 1 && batch <= m->c.max_batch && steps >= 1, "bad batch / steps");
        cudaStream_t s = m->ctx->stream;
        StepProbe probe;
        probe.s = s;
        const bool pdl = m->ctx->pdl;
        m->ctx->pdl = false;
        try {
            for (int i = 0; i < steps; i++) {
                FB_CUDA(cudaMemcpyAsync(m->tok.ptr, tokens_dev, (size_t)batch * 4, cudaMemcpyDeviceToDevice, s));
                FB_CUDA(cudaMemcpyAsync(m->pos.ptr, pos_dev, (size_t)batch * 4, cudaMemcpyDeviceToDevice, s));
                step(m, batch, &probe);
            }
            probe.collect();
        } catch (...) {
            m->ctx->pdl = pdl;
            throw;
        }
        m->ctx->pdl = pdl;
        for (int k = 0; k < FB_PROF_KINDS; k++) {
            ms_out[k] = probe.ms[k];
            if (launches_out) launches_out[k] = probe.launches[k] / steps;
        }
    });
}

int fb_model_step_timeline(fb_model *m, const int32_t *tokens_dev, const int32_t *pos_dev, uint64_t *stamps_host,
                           int64_t capacity, int *ctas_out, int *slots_out) {
    return guarded([&] {
        FB_REQUIRE(m && tokens_dev && pos_dev && stamps_host && ctas_out && slots_out, "null argument");
        require_ready(m);
        FB_REQUIRE(m->ds_ok && m->ds_on && !m->comm, "the persistent step is not in use for this model");
        const int ctas = m->ctx->num_sms, per = (m->c.n_layers + 1) * DS_TRACE_SLOTS;
        const int64_t n = (int64_t)ctas * per;
        FB_REQUIRE(capacity >= n, "stamps_host holds fewer than num_sms * (n_layers + 1) * 16 entries");
        cudaStream_t s = m->ctx->stream;
        DevBuf tr;
        tr.alloc((size_t)n * 8);
        FB_CUDA(cudaMemsetAsync(tr.ptr, 0, (size_t)n * 8, s));
        FB_CUDA(cudaMemcpyAsync(m->tok.ptr, tokens_dev, 4, cudaMemcpyDeviceToDevice, s));
        FB_CUDA(cudaMemcpyAsync(m->pos.ptr, pos_dev, 4, cudaMemcpyDeviceToDevice, s));
        persistent_step(m, 1, nullptr, tr.as<unsigned long long>());
        FB_CUDA(cudaMemcpyAsync(stamps_host, tr.ptr, (size_t)n * 8, cudaMemcpyDeviceToHost, s));
        FB_CUDA(cudaStreamSynchronize(s));
        *ctas_out = ctas;
        *slots_out = DS_TRACE_SLOTS;
    });
}

int fb_model_launches_per_step(const fb_model *m, int *launches) {
    return guarded([&] {
        FB_REQUIRE(m && launches, "null argument");
        require_ready(m);
        const int L = m->c.n_layers;
        const bool q8_fused = (m->lc.n_heads / m->lc.n_kv_heads) % 2 == 0;
        // matches step(): embed-norm; per layer qkv, attention (+ Q8_K quantize
        // for odd GQA groups), o, norm, gate_up, swiglu, down, norm; lm_head,
        // argmax -- or, batch 1 with the persistent step, its kernel and argmax
        *launches = m->launches_per_step > 0 ? m->launches_per_step : 1 + (q8_fused ? 8 : 9) * L + 2;
    });
}

int fb_model_read_activation(fb_model *m, const char *name, int row, float *out_host, int64_t count) {
    return guarded([&] {
        FB_REQUIRE(m && name && out_host, "null argument");
        const fb_model_config &c = m->lc;  // this rank's shard dims
        FB_REQUIRE(row >= 0 && row < c.max_batch, "row out of range");
        const int64_t qd = (int64_t)c.n_heads * c.head_dim, kd = (int64_t)c.n_kv_heads * c.head_dim;
        const std::string n(name);
        const DevBuf *buf = nullptr;
        int64_t len = 0;
        if (n == "x") {
            FB_REQUIRE(m->x_last, "no decode step has run yet");
            len = c.hidden;
            FB_CUDA(cudaMemcpyAsync(out_host, m->x_last + (size_t)row * len, (size_t)len * 4, cudaMemcpyDeviceToHost,
                                    m->ctx->stream));
            FB_CUDA(cudaStreamSynchronize(m->ctx->stream));
            return;
        } else if (n == "qkv") buf = &m->y_qkv, len = qd + 2 * kd;
        else if (n == "q") buf = &m->q, len = qd;
        else if (n == "attn") buf = &m->attn, len = qd;
        else if ((n == "o" || n == "down") && m->comm)
            fail(FB_ERR_STATE, "row-parallel projection outputs are exchanged as partial sums under tensor parallelism");
        else if (n == "o") buf = &m->y_o, len = c.hidden;
        else if (n == "gate_up") buf = &m->y_gu, len = 2LL * c.ffn;
        else if (n == "down") buf = &m->y_d, len = c.hidden;
        else if (n == "logits") buf = &m->logits, len = c.vocab;
        else fail(FB_ERR_INVALID, "unknown activation name: " + n);
        FB_REQUIRE(count == len, "count must equal the row length (" + std::to_string(len) + ")");
        FB_CUDA(cudaMemcpyAsync(out_host, buf->as<float>() + (size_t)row * len, (size_t)len * 4,
                                cudaMemcpyDeviceToHost, m->ctx->stream));
        FB_CUDA(cudaStreamSynchronize(m->ctx->stream));
    });
}

// ---------------------------------------------------------------------------
int fb_attn_prefill(fb_ctx *ctx, const float *q_dev, const void *k_pages_dev, const void *v_pages_dev,
                    const int32_t *block_table_dev, int max_pages, int num_pages, int pos0, int n_tokens,
                    int n_heads, int n_kv_heads, int head_dim, int page_size, float scale, float *out_dev) {
    return guarded([&] {
        FB_REQUIRE(ctx && q_dev && k_pages_dev && v_pages_dev && block_table_dev && out_dev, "null argument");
        FB_REQUIRE(head_dim == 128 && page_size == 64, "prefill attention: head_dim 128, page_size 64");
        FB_REQUIRE(n_tokens >= 1 && n_heads >= 1 && n_kv_heads >= 1 && num_pages >= 1, "bad shape");
        launch_attn_prefill(ctx, q_dev, k_pages_dev, v_pages_dev, block_table_dev, max_pages, num_pages, pos0,
                            n_tokens, n_heads, n_kv_heads, scale, out_dev);
    });
}

int fb_attn_decode(fb_ctx *ctx, const float *q_dev, const void *k_pages_dev, const void *v_pages_dev,
                   const int32_t *block_table_dev, const int32_t *seq_lens_dev, float *out_dev, int batch,
                   int n_heads, int n_kv_heads, int head_dim, int page_size, int max_pages, int num_pages,
                   int max_seq_len, float scale) {
    return guarded([&] {
        FB_REQUIRE(ctx && q_dev && k_pages_dev && v_pages_dev && block_table_dev && seq_lens_dev && out_dev,
                   "null argument");
        FB_REQUIRE(head_dim == 128, "head_dim must be 128");
        FB_REQUIRE(page_size == 32 || page_size == 64, "page_size must be 32 or 64");
        FB_REQUIRE(batch >= 1 && n_heads >= 1 && n_kv_heads >= 1 && max_pages >= 1 && max_seq_len >= 1,
                   "bad shape");
        FB_REQUIRE(num_pages >= 1, "num_pages must be positive");
        FB_REQUIRE(max_seq_len <= max_pages * page_size, "max_seq_len exceeds the block table");
        AttnArgs A{};
        A.q = q_dev;
        A.kpool = k_pages_dev;
        A.vpool = v_pages_dev;
        A.block_table = block_table_dev;
        A.seq_lens = seq_lens_dev;
        A.pos = nullptr;
        A.n_heads = n_heads;
        A.n_kv = n_kv_heads;
        A.page_size = page_size;
        A.max_pages = max_pages;
        A.num_pages = num_pages;  // block-table ids outside the pool set ERRBIT_BAD_PAGE and are skipped
        A.nsplit_max = ATT_SPLITS;
        A.scale = scale;
        A.err = ctx->err_word;
        int *counters = nullptr;
        if (n_heads % n_kv_heads == 0 && !attn_uses_cluster(ctx, A, batch)) {
            // cluster-free merge: split partials and merge counters in the workspace
            const size_t cnt_bytes = ((size_t)batch * n_kv_heads * 4 + 255) & ~(size_t)255;
            uint8_t *raw = static_cast<uint8_t *>(
                ctx->ensure_scratch(cnt_bytes + (size_t)batch * n_heads * ATT_SPLITS * (head_dim + 2) * 8));
            counters = reinterpret_cast<int *>(raw);
            FB_CUDA(cudaMemsetAsync(counters, 0, cnt_bytes, ctx->stream));
            A.part_o = reinterpret_cast<double *>(raw + cnt_bytes);
            A.part_ml = A.part_o + (size_t)batch * n_heads * ATT_SPLITS * head_dim;
        }
        launch_attn_decode(ctx, A, batch, max_seq_len, out_dev, nullptr, counters, false, true);
    });
}

}  // extern "C"

namespace fb {
// m > 16: the tensor-core GEMM when the shape allows (n a multiple of 128),
// else the Q8_K integer path in chunks of 16 rows.
void qmatmul_prefill(fb_ctx *ctx, const fb_qtensor *w, const float *x, float *y, int64_t m) {
    if (prefill_gemm_supported(w, m)) {
        prefill_gemm(ctx, w, x, y, m);
        return;
    }
    const int rc = fb_qmatmul_q8k(ctx, w, x, y, m);
    if (rc != FB_OK) fail(rc, fb_last_error());
}
}  // namespace fb
