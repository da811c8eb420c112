// Host / device interface of the persistent decode-step kernel
// (decode_step.cu).  Internal to the library.
#pragma once

#include <cuda_fp16.h>

#include "fb_internal.h"

namespace fb {

// One layer's tensors as the persistent kernel reads them (device copy of an
// array of these is built when the model is finalized).
struct DsLayer {
    const uint8_t *qkv, *o, *gu, *down;  // tile-major records
    int dt_qkv, dt_o, dt_gu, dt_down;    // 4 (Q4_K) or 6 (Q6_K)
    const float *attn_norm, *ffn_norm, *q_norm, *k_norm;
};

struct DsArgs {
    const DsLayer *layers;
    int n_layers, H, F, n_heads, n_kv, vocab, qkv_n;
    const uint8_t *emb;  // token_embd, Q4_K tile-major
    const uint8_t *out;  // lm_head
    int dt_out;
    const float *out_norm;
    float eps, scale;
    const int32_t *tok, *pos;
    __half *kv;        // [L][K|V][num_pages][n_kv][..]
    size_t kv_layer;   // halves of one layer's K pool (the V pool follows it)
    const int32_t *block_table;
    int pages_per_seq, num_pages;
    const float *rope_cos, *rope_sin;
    int rope_rows, rope_mode, qk_norm;
    float *xa, *xb;  // residual ping-pong; the step's final residual lands in xb
    float *y_qkv, *q_out, *attn, *y_o, *y_gu, *y_d, *logits;
    Q8Act act_a, act_f;  // global Q8_K rows: attention output, SwiGLU output
    double *part_o, *part_ml;
    int *att_cnt;
    unsigned *sync;  // [0] grid-barrier arrivals, [1] abort flag, [32] last barrier released (zero at launch)
    uint32_t *err;
    int ns;      // attention splits per kv head
    int nstage;  // ring stages
    // optional phase timeline: [cta][layer + 1][DS_TRACE_SLOTS] %globaltimer
    // stamps written by each CTA's consumer thread 0 (null: not recorded)
    unsigned long long *trace;
};
constexpr int DS_TRACE_SLOTS = 16;

struct DsPlan {
    int nstage = 0, ns = 0;
    size_t smem = 0;
};

// Whether the persistent step supports this single-GPU batch-1 model shape
// (GQA group 2, 4 or 8, 64-token pages, shared memory for at least three
// ring stages); fills the launch plan.
bool decode_step_plan(const fb_ctx *ctx, int H, int F, int n_heads, int n_kv, int pages_per_seq, int page,
                      DsPlan *out);
// Clears the barrier / merge counters and launches the cooperative kernel.
void launch_decode_step(fb_ctx *ctx, const DsArgs &A, size_t smem);

}  // namespace fb
