"""Decode benchmark: Qwen3-8B-architecture Q4_K_M decode tok/s on B200.

Workload (one "step" = one greedy decode token per sequence): random-init
Qwen3-8B architecture (36 layers, hidden 4096, 32 q / 8 kv heads, head_dim
128, QK-norm, RoPE theta 1e6, SwiGLU 12288, vocab 151936), Q4_K weights
except ffn_down and output (Q6_K), fp16 paged KV cache holding 4096 tokens
when decoding starts, batch 1 by default.

  value  device-resident throughput: token ids fed back on the device, one
         CUDA-graph replay per step, CUDA events over K timed steps.
  e2e    the same metric through the public host API fb_model_decode_greedy
         (token + position copied from pinned host memory, next token read
         back every step).
  roofline  the dominant kernel class (by measured time) from a live
         per-kernel CUDA-event profile of the same workload.
  cpu_baseline  the CPU oracle (C restatement of candle's CPU quantized path)
         decoding the same random-init model on the host cores (rank 0, N=1).
  prefill_2048, batch16  (N=1, batch 1 runs) a 2048-token prompt pass through
         fb_model_forward, and decode at batch 16 on its own model.

N > 1 (torchrun): the N ranks hold ONE tensor-parallel model (column-parallel
q/k/v, gate/up and lm_head shards, row-parallel attn_output and ffn_down
whose partial sums are exchanged over NVLink by the projection and norm
kernels; greedy argmax merged across ranks); value is the batch's tokens per
second, max-over-ranks device time (strong scaling).  --replicas instead runs
an independent replica per GPU (weak scaling, no data-path collective).
--impl reference: the CPU oracle alone (the reference's path restated; the
reference itself is Rust + candle and cannot be built here), rank 0 only,
on all host threads, timing exactly --steps greedy tokens.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, os.path.join(ROOT, "ferrite-llm_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

MODELS = {
    "qwen3-8b": dict(n_layers=36, hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128, ffn=12288, vocab=151936,
                     rope_theta=1e6, eps=1e-6, qk_norm=1, rope_mode=1),
    "llama3-70b": dict(n_layers=80, hidden=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn=28672, vocab=128256,
                       rope_theta=5e5, eps=1e-5, qk_norm=0, rope_mode=0),
}
METRIC = "Q4_K_M decode tok/s + GEMV HBM GB/s vs roofline (Qwen3-8B arch, 1-8 B200)"
SEED = 1234


def peaks() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def step_bytes(cfg: dict, batch: int, ctx: int, world: int = 1) -> dict:
    """Algorithmic bytes per decode step by kernel class (weights once per
    step, KV once per sequence, activations f32/Q8_K once), for one rank of
    a `world`-way tensor-parallel model (world 1: the whole model)."""
    H, F, V, L = cfg["hidden"], cfg["ffn"] // world, cfg["vocab"] // world, cfg["n_layers"]
    qd, kd = cfg["n_heads"] // world * cfg["head_dim"], cfg["n_kv_heads"] // world * cfg["head_dim"]
    q4, q6 = 144 / 256, 210 / 256

    def q8(k):  # Q8_K activation row: qs + d + bsums(16 and 32)
        return k + 4 * k / 256 + 2 * k / 16 + 2 * k / 32

    b = batch
    per = {
        "qkv": (qd + 2 * kd) * H * q4 + b * (q8(H) + 4 * (qd + 2 * kd)),
        "o": H * qd * q4 + b * (q8(qd) + 4 * H),
        "gate_up": 2 * F * H * q4 + b * (q8(H) + 8 * F),
        "down": H * F * q6 + b * (q8(F) + 4 * H),
        "attn": b * (2 * (ctx + 1) * kd * 2 + 4 * qd * 2),
    }
    tot = {k: v * L for k, v in per.items()}
    tot["lm_head"] = V * H * q6 + b * (q8(H) + 4 * V)
    tot["embed"] = b * H * q4
    # latency-bound classes (not part of the step's byte total above, which
    # counts each tensor once): residual + RMSNorm reads x and the projection
    # output and writes x and the Q8_K row; SwiGLU reads gate|up and writes
    # Q8_K; argmax reads the logits
    extra = {"norm": b * (3 * 4 * H + q8(H)) + 4 * H, "swiglu": b * (8 * F + q8(F)), "argmax": b * 4 * V,
             "embed_norm": b * (H * q4 + 4 * H + q8(H)) + 4 * H}
    return {"per_launch": per | {"lm_head": tot["lm_head"]} | extra, "per_step": tot, "total": sum(tot.values())}


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict | None:
        rows = []
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def cpu_oracle_decode(cfg: dict, ctx: int, batch: int, budget_s: float, max_tokens: int, warmup: int = 1):
    """Decode with the CPU oracle on all host threads (set explicitly: under
    torchrun OMP_NUM_THREADS defaults to 1); returns (tok/s, tokens
    measured, threads)."""
    from oracle import oracle as O

    nthreads = os.cpu_count() or 1
    ocfg = dict(cfg, max_ctx=ctx + warmup + max_tokens + 2, kv_f16=1)
    w = O.synth_model_weights(ocfg, SEED)
    m = O.Model(ocfg, w, nthreads=nthreads)
    m.synth_kv(SEED + 7, ctx)
    tok = int(O.synth_tokens(2, 1, cfg["vocab"])[0])
    pos = ctx
    for _ in range(warmup):
        tok = int(O.np.argmax(m.forward([tok], pos)))
        pos += 1
    n, t0 = 0, time.perf_counter()
    while n < max_tokens:
        tok = int(O.np.argmax(m.forward([tok], pos)))
        pos += 1
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    m.close()
    return n / dt, n, nthreads


def run_reference(args, cfg):
    ws, rank, _ = dist_setup()
    if rank != 0:
        return
    # every one of the --steps tokens is timed (about 0.7 s each on 32 host
    # threads); the budget only guards against a far slower host
    tps, n, cores = cpu_oracle_decode(cfg, args.ctx, 1, budget_s=600.0, max_tokens=args.steps, warmup=args.warmup)
    line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": "tok/s", "n_gpus": ws, "steps": n,
            "warmup": args.warmup, "ms_per_step": 1000.0 / tps, "higher_is_better": True,
            "scaling": "strong" if use_tp(args) else "weak",
            "vs_baseline": None, "dtype": "int8 (Q4_K/Q6_K x Q8_K, CPU scalar)", "data": "synthetic",
            "config": workload_config(args), "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0,
                                                     "d2h_bytes_per_step": 0},
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"{n} greedy decode tokens of the full model at ctx {args.ctx}, batch 1, "
                                       f"{cores} host threads "
                                       f"(CPU oracle = C restatement of candle 0.8.4's CPU quantized path; "
                                       f"the Rust reference cannot be built here)"}}
    print(json.dumps(line), flush=True)


PREFILL_SHAPES = {  # (class, dtype name, n = output rows, k) per layer
    "qwen3-8b": [("qkv", "Q4_K", 6144, 4096), ("o", "Q4_K", 4096, 4096), ("gate_up", "Q4_K", 24576, 4096),
                 ("down", "Q6_K", 4096, 12288)],
    "llama3-70b": [("qkv", "Q4_K", 10240, 8192), ("o", "Q4_K", 8192, 8192), ("gate_up", "Q4_K", 57344, 8192),
                   ("down", "Q6_K", 8192, 28672)],
}


def run_prefill_gemm(args):
    """Prefill QMatMul (tcgen05 dequant-GEMM) on one layer's projections at
    T = args.prefill_gemm activation rows; TFLOP/s per class against the
    measured bf16 tensor peak.  Inputs: f32 activations T x k (re-used; the
    weights of one class are 13-130 MB, the outputs T x n f32 up to 200 MB)."""
    import torch

    import ferrite_b200 as fb

    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream()
    ctx = fb.Context(0, stream.cuda_stream)
    T = args.prefill_gemm
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        peak, kind = float(pk["bf16_tflops"]), "measured (burst)"
    except Exception:
        peak, kind = 1590.0, "fallback"
    res, tot_fl, tot_ms = {}, 0.0, 0.0
    with ClockSampler(0) as clk:
        for name, dts, n, k in PREFILL_SHAPES[args.model]:
            w = fb.QTensor.synth(ctx, getattr(fb, dts), n, k, seed=n + k)
            x = torch.randn(T, k, device="cuda", generator=torch.Generator(device="cuda").manual_seed(k))
            y = torch.empty(T, n, device="cuda")
            mm = fb.QMatMul(w)
            for _ in range(args.warmup):
                mm.forward(x.data_ptr(), y.data_ptr(), T)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                mm.forward(x.data_ptr(), y.data_ptr(), T)
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            fl = 2.0 * T * n * k
            res[name] = {"n": n, "k": k, "dtype": dts, "ms": ms, "tflops": fl / ms / 1e9}
            tot_fl, tot_ms = tot_fl + fl, tot_ms + ms
            del w, x, y, mm
            torch.cuda.empty_cache()
    achieved = tot_fl / tot_ms / 1e9
    line = {"metric": "prefill QMatMul TFLOP/s (Q4_K/Q6_K dequant-GEMM, fp16 tcgen05, f32 accumulate)",
            "value": achieved, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": tot_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp16 x fp16 -> f32", "data": "synthetic (seeded weights and activations)",
            "config": {"workload": f"{args.model}-arch one layer's projections at {T} prefill rows", "rows": T},
            "per_class": res, "error_word": ctx.error_word(),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "peak_source": kind}}
    clocks = clk.summary()
    if clocks:
        line["clocks"] = clocks
    print(json.dumps(line), flush=True)


def prefill_flops(cfg: dict, T: int) -> float:
    """FLOPs of a T-token prompt pass: the projections (2 T per weight), the
    causal attention (q.k and p.v over T (T + 1) / 2 query-key pairs per
    head) and the last row's lm_head."""
    H, F, L = cfg["hidden"], cfg["ffn"], cfg["n_layers"]
    qd, kd = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]
    lin = 2.0 * T * L * (H * (qd + 2 * kd) + qd * H + 2 * F * H + F * H)
    att = 4.0 * L * cfg["n_heads"] * cfg["head_dim"] * T * (T + 1) / 2
    return lin + att + 2.0 * H * cfg["vocab"]


def run_prefill(args, cfg):
    """Prompt pass of T uniform random token ids (seed 2) through the public
    API fb_model_forward (batched prefill: tensor-core projections and
    attention), then 64 greedy decode steps (fb_model_decode_greedy; the
    first one captures the decode CUDA graph and is left out of the
    host-timed decode rate)."""
    import numpy as np
    import torch

    import ferrite_b200 as fb

    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream()
    ctx = fb.Context(0, stream.cuda_stream)
    T, ndec = args.prefill, 64
    model = fb.Model(ctx, dict(cfg, max_ctx=T + ndec + 8, max_batch=1))
    model.synth(SEED)
    model.finalize()
    prompt = np.random.default_rng(2).integers(0, cfg["vocab"], T).astype(np.int32)
    for _ in range(args.warmup):
        model.clear_cache()
        model.forward(prompt, 0)
    torch.cuda.synchronize()
    times = []
    with ClockSampler(0) as clk:
        for _ in range(args.steps):
            model.clear_cache()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            logits = model.forward(prompt, 0)  # host tokens in, host logits out
            e1.record(stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        ms = statistics.median(times)
        tok = int(np.argmax(logits))
        # the first decode step captures the decode CUDA graph: untimed
        tok = int(model.decode_greedy([tok], [T])[0])
        toks = [tok]
        t0 = time.perf_counter()
        for i in range(1, ndec):
            tok = int(model.decode_greedy([tok], [T + i])[0])
            toks.append(tok)
        dec_s = time.perf_counter() - t0
        # on-device sampling of one vocab row with the reference sampler's
        # default config (fb_sample), the cost a sampled decode step adds
        lg = torch.from_numpy(np.asarray(logits, dtype=np.float32)).cuda()
        smp = fb.Sampler(ctx)
        prev = prompt[-64:].tolist()
        smp.sample(lg.data_ptr(), cfg["vocab"], prev)
        t1 = time.perf_counter()
        for _ in range(32):
            smp.sample(lg.data_ptr(), cfg["vocab"], prev)
        sample_ms = (time.perf_counter() - t1) / 32 * 1e3
    fl = prefill_flops(cfg, T)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, kind = float(json.load(f)["bf16_tflops"]), "measured (burst)"
    except Exception:
        peak, kind = 1590.0, "fallback"
    achieved = fl / (ms * 1e-3) / 1e12
    line = {"metric": f"prefill tok/s ({T}-token prompt, then {ndec} greedy decode steps)", "value": T / (ms * 1e-3),
            "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp16 x fp16 -> f32 (tensor cores) for the prompt; int8 Q8_K for decode",
            "data": "synthetic (random-init weights, uniform random prompt ids, seed 2)",
            "config": {"workload": f"{args.model}-arch Q4_K_M random-init prefill of {T} tokens, batch 1, "
                                   f"then {ndec} greedy decode steps", "prompt_tokens": T, "decode_steps": ndec},
            "e2e": {"value": T / (ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": 4 * T,
                    "d2h_bytes_per_step": 4 * cfg["vocab"]},
            "decode_after_prefill_tok_s": (ndec - 1) / dec_s,
            "sampler_ms_per_token": sample_ms,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "flops_per_step": fl, "peak_source": kind},
            "error_word": ctx.error_word()}
    clocks = clk.summary()
    if clocks:
        line["clocks"] = clocks
    print(json.dumps(line), flush=True)
    model.close()


def use_tp(args) -> bool:
    return int(os.environ.get("WORLD_SIZE", "1")) > 1 and not args.replicas


def timeline_table(tl) -> dict:
    """Per-phase microseconds of the persistent step's timeline [cta][layer
    + 1][16] (fb_model_step_timeline): median and max over CTAs of each
    phase's duration, averaged over the inner layers."""
    import numpy as np

    L = tl.shape[1] - 1
    names = ["qkv", "barrier_qkv", "attention", "barrier_attention", "o", "barrier_o", "norm_ffn", "gate_up",
             "barrier_gate_up", "swiglu", "barrier_swiglu", "down", "barrier_down", "norm_attn"]
    acc = {n: [] for n in names}
    for l in range(1, L - 1):
        prev = tl[:, l, 0]
        for k, n in enumerate(names):
            cur = tl[:, l, k + 1] if k < 13 else tl[:, l + 1, 0]
            acc[n].append((np.median(cur - prev), np.max(cur - prev)))
            prev = cur
    out = {n: {"median_us": float(np.mean([a for a, _ in v]) / 1e3), "max_us": float(np.mean([b for _, b in v]) / 1e3)}
           for n, v in acc.items()}
    out["layer_us"] = float((tl[:, L - 1, 13].max() - tl[:, 0, 0].min()) / 1e3 / L)
    out["lm_head_us"] = float(np.median(tl[:, L, 1] - tl[:, L, 0]) / 1e3)
    return out


def prefill_extra(model, cfg: dict, stream, T: int = 2048) -> dict:
    """The batched prompt pass of the decode model (T uniform random ids,
    seed 2) through fb_model_forward: host tokens in, host logits out; two
    untimed passes, then the median of three (CUDA events).  FLOPs counted as
    prefill_flops (projections, causal attention, last-row lm_head)."""
    import numpy as np
    import torch

    prompt = np.random.default_rng(2).integers(0, cfg["vocab"], T).astype(np.int32)
    for _ in range(2):
        model.clear_cache()
        model.forward(prompt, 0)
    torch.cuda.synchronize()
    times = []
    for _ in range(3):
        model.clear_cache()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        model.forward(prompt, 0)
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    ms = statistics.median(times)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, kind = float(json.load(f)["bf16_tflops"]), "measured (burst)"
    except Exception:
        peak, kind = 1590.0, "fallback"
    tflops = prefill_flops(cfg, T) / (ms * 1e-3) / 1e12
    return {"prompt_tokens": T, "ms": ms, "tok_s": T / (ms * 1e-3), "tflops": tflops,
            "frac_of_bf16_peak": tflops / peak, "peak_source": kind,
            "how": "fb_model_forward of a uniform random prompt (seed 2), host ids in, host logits out"}


def batch_extra(ctx, cfg: dict, stream, ctx_len: int, B: int = 16, steps: int = 10) -> dict:
    """Decode at batch B on its own model (same weights and KV generator):
    device-resident tokens, CUDA-graph steps timed with CUDA events after
    three warm-up steps.  The step reads the weights once and B sequences'
    KV, far above the L2 size."""
    import torch

    import ferrite_b200 as fb

    m = fb.Model(ctx, dict(cfg, max_ctx=ctx_len + steps + 8, max_batch=B))
    m.synth(SEED)
    m.finalize()
    m.synth_kv(SEED + 7, ctx_len)
    tok = torch.randint(0, cfg["vocab"], (B,), dtype=torch.int32, device="cuda",
                        generator=torch.Generator(device="cuda").manual_seed(3))
    pos = torch.arange(ctx_len, ctx_len + steps + 4, dtype=torch.int32, device="cuda")
    pos = pos.repeat_interleave(B).reshape(-1, B).contiguous()
    for i in range(3):
        m.decode_dev(tok.data_ptr(), pos[i].data_ptr(), B, next_ptr=tok.data_ptr())
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(3, 3 + steps):
        m.decode_dev(tok.data_ptr(), pos[i].data_ptr(), B, next_ptr=tok.data_ptr())
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    err = ctx.error_word()
    m.close()
    sb = step_bytes(cfg, B, ctx_len)
    peak, _ = peaks()
    return {"batch": B, "kv_ctx": ctx_len, "tok_s": B / (ms * 1e-3), "ms_per_step": ms,
            "step_roofline_frac": sb["total"] / (ms * 1e-3) / 1e9 / peak, "device_error_word": err,
            "how": f"fb_model_decode_dev, {steps} CUDA-graph steps after 3 warm-up steps, CUDA events"}


def workload_config(args) -> dict:
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    par = f"tp{ws}" if use_tp(args) else ("replicas" if ws > 1 else "single-gpu")
    wl = f"{args.model}-arch Q4_K_M random-init decode, batch {args.batch}, fp16 KV ctx {args.ctx}"
    if use_tp(args):
        wl += f", tensor-parallel over {ws} GPUs"
    return {"workload": wl, "model_arch": args.model, "batch": args.batch, "kv_ctx": args.ctx,
            "weights": "Q4_K (+Q6_K ffn_down, output)", "parallelism": par,
            "l2": "not flushed: each step streams the weights (GBs per GPU), >> 126 MB L2"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="qwen3-8b", choices=sorted(MODELS))
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=32)
    ap.add_argument("--profile-run", type=int, default=0,
                    help="build the workload, run N untimed decode steps and exit (driver for ncu captures)")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (small ncu captures)")
    ap.add_argument("--tp", action="store_true",
                    help="(default under torchrun) one tensor-parallel model over all ranks (strong scaling)")
    ap.add_argument("--replicas", action="store_true",
                    help="under torchrun: an independent replica per GPU instead of tensor parallelism")
    ap.add_argument("--persistent", action="store_true",
                    help="batch 1: run the opt-in persistent decode-step kernel instead of the kernel chain")
    ap.add_argument("--timeline", action="store_true",
                    help="with --persistent: print the per-phase timeline of one eager step and exit")
    ap.add_argument("--no-prefill-extra", action="store_true",
                    help="skip the 2048-token prefill and batch-16 measurements added to the N=1 decode line")
    ap.add_argument("--prefill", type=int, default=0, metavar="T",
                    help="instead of decode: time a T-token prompt pass (then 64 greedy decode steps), 1 GPU")
    ap.add_argument("--prefill-gemm", type=int, default=0, metavar="T",
                    help="instead of decode: time one layer's prefill QMatMuls at T rows (1 GPU)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    cfg = dict(MODELS[args.model])
    if args.layers:
        cfg["n_layers"] = args.layers
    if args.impl == "reference":
        return run_reference(args, cfg)
    if args.prefill_gemm:
        return run_prefill_gemm(args)
    if args.prefill:
        return run_prefill(args, cfg)

    import numpy as np
    import torch

    import ferrite_b200 as fb

    ws, rank, local = dist_setup()
    torch.cuda.set_device(local)
    pg = None
    if ws > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
        pg = dist
    stream = torch.cuda.current_stream()
    ctx = fb.Context(local, stream.cuda_stream)
    B = args.batch
    max_ctx = args.ctx + args.warmup + args.steps + args.e2e_steps + 16
    mcfg = dict(cfg, max_ctx=max_ctx, max_batch=B)
    comm = fb.Comm.connect(ctx, B, cfg["hidden"]) if use_tp(args) else None
    W = ws if comm else 1
    model = fb.Model(ctx, mcfg, comm)
    model.synth(SEED)
    model.finalize()
    model.synth_kv(SEED + 7, args.ctx)
    if args.persistent:
        assert model.set_persistent(True), "the persistent step does not support this model"
    if pg:
        pg.barrier()  # tensor-parallel ranks start stepping together
    nsteps = args.warmup + args.steps
    pos_all = torch.arange(args.ctx, args.ctx + nsteps + 8, dtype=torch.int32, device="cuda")
    pos_all = pos_all.repeat_interleave(B).reshape(-1, B).contiguous()
    tok = torch.randint(0, cfg["vocab"], (B,), dtype=torch.int32, device="cuda",
                        generator=torch.Generator(device="cuda").manual_seed(2))

    def dstep(i):
        model.decode_dev(tok.data_ptr(), pos_all[i].data_ptr(), B, next_ptr=tok.data_ptr())

    if args.timeline:
        for i in range(3):
            dstep(i)
        tl = model.step_timeline(tok.data_ptr(), pos_all[3].data_ptr(), torch.cuda.get_device_properties(local)
                                 .multi_processor_count).astype(np.int64)
        print(json.dumps(timeline_table(tl)))
        return

    if args.profile_run:
        for i in range(args.profile_run):
            dstep(i)
        torch.cuda.synchronize()
        print("profile run ok", tok.cpu().tolist(), "error word", ctx.error_word())
        return

    for i in range(args.warmup):
        dstep(i)
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for i in range(args.warmup, nsteps):
            dstep(i)
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if pg:
        t = torch.tensor([ms], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
        pg.barrier()
    torch.cuda.synchronize()
    ms_per_step = ms / args.steps
    seqs = B if comm else ws * B  # sequences decoded by the whole job per step
    value = seqs * args.steps / (ms / 1e3)
    err = ctx.error_word()

    # ---- e2e through the public host API (pinned H2D + D2H every step)
    toks_h = tok.cpu().numpy().astype(np.int32)
    p0 = args.ctx + nsteps
    for i in range(2):
        toks_h = model.decode_greedy(toks_h, np.full(B, p0 + i, np.int32))
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    t0 = time.perf_counter()
    for i in range(args.e2e_steps):
        toks_h = model.decode_greedy(toks_h, np.full(B, p0 + 2 + i, np.int32))
    e2e_s = time.perf_counter() - t0
    if pg:
        t = torch.tensor([e2e_s], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = seqs * args.e2e_steps / e2e_s

    # ---- live per-kernel profile: CUDA events between kernel classes of
    # eager steps, kernels serialised (no PDL overlap), so the per-class sum
    # exceeds the graph step's time; the dominant class is the one with the
    # most serialised time per step, over every class
    prof = model.profile(tok.data_ptr(), pos_all[0].data_ptr(), B, 3)
    sb = step_bytes(cfg, B, args.ctx, W)
    peak, peak_kind = peaks()
    classes = [k for k in prof if prof[k][1] > 0 and k in sb["per_launch"]]
    dom = max(classes, key=lambda k: prof[k][0])
    dom_ms_per_launch = prof[dom][0] / 3 / max(1, prof[dom][1])
    achieved = sb["per_launch"][dom] / (dom_ms_per_launch * 1e-3) / 1e9
    kname = {"attn": "attn_decode"}.get(dom, f"gemv_{dom}" if dom in ("qkv", "o", "gate_up", "down", "lm_head")
                                        else dom)
    traffic = None
    for tfile in (os.path.join(ROOT, "profiles", f"{kname}_{args.model}_b{B}.md"),
                  os.path.join(ROOT, "profiles", f"{kname}_{args.model}_b{B}_ctx{args.ctx}.md")):
        if os.path.exists(tfile):
            for ln in open(tfile):
                if ln.startswith("dram_bytes_per_launch:"):
                    traffic = float(ln.split(":")[1].split()[0])
    step_achieved = sb["total"] / (ms_per_step * 1e-3) / 1e9
    prof_ms = {k: round(v[0] / 3, 4) for k, v in prof.items()}

    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong" if comm else "weak",
            "vs_baseline": None, "dtype": "int8 (Q4_K/Q6_K weights x Q8_K activations, int8 MMA, f32/f64 combine)",
            "data": "synthetic (random-init weights and KV, seeded)", "config": workload_config(args),
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8 * B, "d2h_bytes_per_step": 4 * B},
            "gpu_launches": model.launches_per_step() * args.steps,
            "roofline": {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
                         "peak_source": peak_kind,
                         "algorithmic_bytes_per_launch": sb["per_launch"][dom],
                         "launch_ms": dom_ms_per_launch},
            "step_roofline": {"achieved": step_achieved, "peak": peak, "unit": "GB/s",
                              "frac": step_achieved / peak, "bytes_per_step": sb["total"],
                              "roofline_tok_s": B * peak * 1e9 / sb["total"]},
            "kernel_ms_per_step_serialised": prof_ms,
            "kernel_ms_note": "eager steps with a CUDA event after every kernel class and no programmatic "
                              "dependent launch: serialised per-class times whose sum exceeds ms_per_step",
            "device_error_word": err}
    clocks = clk.summary()
    if clocks:
        line["clocks"] = clocks
    if ws == 1 and not args.no_prefill_extra and args.model == "qwen3-8b" and B == 1:
        line["prefill_2048"] = prefill_extra(model, cfg, stream)
        line["batch16"] = batch_extra(ctx, cfg, stream, args.ctx)
    if rank == 0 and ws == 1 and not args.no_cpu_baseline and args.model == "qwen3-8b":
        model.close()
        torch.cuda.empty_cache()
        tps, n, cores = cpu_oracle_decode(cfg, args.ctx, 1, budget_s=20.0, max_tokens=8)
        line["cpu_baseline"] = {"value": tps, "unit": "tok/s", "cores": cores, "kind": "port",
                                "sample": f"{n} greedy decode tokens of the same random-init model at ctx "
                                          f"{args.ctx}, batch 1, CPU oracle (C restatement of candle's CPU "
                                          f"quantized path) on all host threads"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    model.close()
    if comm:
        pg.barrier()  # no rank unmaps its region while a peer still steps
        comm.close()
    if pg:
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
