"""Tensor-parallel decode on 2, 4 and 8 GPUs against the oracle.

Each rank is a child process on its own GPU (one process per GPU, gloo for
the host-side handle exchange and barriers); ranks map each other's fb_comm
regions through CUDA IPC.  The sharded random-init model must give the
oracle's logits (tolerance of the parity bar, over the gathered vocab
slices) and the oracle's greedy tokens, at batch 1 and batch 2.  The greedy
chain is teacher-forced: every step feeds the oracle's token to the ranks,
so a near tie (oracle top-2 margin below TIE_MARGIN) is reported and the
comparison continues.  A second model has the Llama-3-70B widths (hidden
8192, 64 q / 8 kv heads, SwiGLU 28672, vocab 128256) at 2 layers.  The
failure test lets one rank never step: the other rank's bounded device waits
run out (nothing writes the tagged partial sums it polls for), the step
reports FB_ERR_DEVICE
with the peer-timeout bit and the context stays usable.  Each world size is
skipped with fewer GPUs.
"""
import os
import socket

import numpy as np
import pytest

from conftest import O, assert_close, synth_weights

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG = dict(n_layers=2, hidden=1024, n_heads=32, n_kv_heads=8, head_dim=128, ffn=2048, vocab=4096, max_ctx=128,
           max_batch=4, rope_theta=1e6, eps=1e-6, qk_norm=1, rope_mode=1, kv_f16=1)
# Llama-3-70B widths at 2 layers (interleaved RoPE, no QK-norm)
CFG70 = dict(n_layers=2, hidden=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn=28672, vocab=128256, max_ctx=64,
             max_batch=1, rope_theta=5e5, eps=1e-5, qk_norm=0, rope_mode=0, kv_f16=1)
SEED = 77
PROMPT = [11, 400, 7, 3000, 25]
STEPS = 24
STEPS70 = 8
TIE_MARGIN = 2e-2
ERRBIT_PEER_TIMEOUT = 1 << 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, mode, q, cfg, forced):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "ferrite-llm_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch
    import torch.distributed as dist

    import ferrite_b200 as fb

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    out = {}
    try:
        ctx = fb.Context(rank, torch.cuda.current_stream().cuda_stream)
        comm = fb.Comm.connect(ctx, cfg["max_batch"], cfg["hidden"])
        model = fb.Model(ctx, cfg, comm)
        model.synth(SEED)
        model.finalize()
        if mode == "timeout":
            comm.set_timeout_ms(300)
            dist.barrier()
            if rank == 0:  # rank 1 never steps: every wait of rank 0 runs out
                try:
                    model.decode_greedy([5], [0])
                    out["rc"] = 0
                except fb.FerriteError as e:
                    out["rc"] = e.code
                    out["msg"] = str(e)
                out["err_after"] = ctx.error_word()  # context still answers
            dist.barrier()
        else:
            dist.barrier()
            lg = model.forward(PROMPT, 0)
            parts = [None] * world
            dist.all_gather_object(parts, (model.vocab_range, lg))
            full = np.concatenate([p[1] for p in sorted(parts, key=lambda p: p[0][0])])
            # greedy steps, each fed the oracle's token (teacher forcing)
            toks = [int(np.argmax(full))]
            for i, tok in enumerate(forced[:-1]):
                toks.append(int(model.decode_greedy([tok], [len(PROMPT) + i])[0]))
            b2 = []
            if cfg["max_batch"] >= 2:
                # batch 2: slot 1 decodes the same prompt token by token
                t1 = PROMPT[0]
                for i in range(len(PROMPT) + 4):
                    nxt = model.decode_greedy([forced[0], t1], [len(PROMPT) + len(forced) - 1, i])
                    t1 = PROMPT[i + 1] if i + 1 < len(PROMPT) else int(nxt[1])
                    b2.append(int(nxt[1]))
            out.update(logits=full, tokens=toks, batch2=b2, err=ctx.error_word())
        model.close()
        comm.close()
        ctx.close()
    finally:
        dist.destroy_process_group()
    if rank == 0:
        q.put(out)


def _run(world, mode, cfg=CFG, forced=()):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, q, cfg, list(forced))) for r in range(world)]
    for p in procs:
        p.start()
    import queue
    import time
    res, t0 = None, time.time()
    while res is None and time.time() - t0 < 600:
        try:
            res = q.get(timeout=2)
        except queue.Empty:
            if all(not p.is_alive() for p in procs):
                break
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert res is not None, f"rank 0 returned nothing; exit codes {[p.exitcode for p in procs]}"
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return res


def oracle_chain(cfg, steps, batch2=True):
    """The oracle's prompt logits, its greedy chain (token i+1 = argmax after
    token i, from the prompt's argmax), the top-2 margin of every step and
    the slot-1 sequence of the batch-2 phase."""
    om = O.Model(cfg, synth_weights(cfg, SEED), nthreads=os.cpu_count() or 1)
    lg = om.forward(PROMPT, 0)
    toks, margins = [int(np.argmax(lg))], [float(np.diff(np.sort(lg)[-2:])[0])]
    for i in range(steps - 1):
        l2 = om.forward([toks[-1]], len(PROMPT) + i)
        margins.append(float(np.diff(np.sort(l2)[-2:])[0]))
        toks.append(int(np.argmax(l2)))
    om.close()
    b2 = []
    if batch2:
        om2 = O.Model(cfg, synth_weights(cfg, SEED))
        t1 = PROMPT[0]
        for i in range(len(PROMPT) + 4):
            nxt = int(np.argmax(om2.forward([t1], i)))
            t1 = PROMPT[i + 1] if i + 1 < len(PROMPT) else nxt
            b2.append(nxt)
        om2.close()
    return lg, toks, margins, b2


def check_chain(res, lg_ref, toks_ref, margins, what):
    assert res["err"] == 0
    assert_close(res["logits"], lg_ref, what=f"{what} prompt logits (gathered vocab slices)")
    ties = []
    for i, (a, b) in enumerate(zip(res["tokens"], toks_ref)):
        if a != b:
            assert margins[i] < TIE_MARGIN, f"{what} greedy token {i}: {a} != {b} (oracle margin {margins[i]:.3g})"
            ties.append(i)
    assert len(res["tokens"]) == len(toks_ref)
    return ties


@pytest.fixture(scope="module")
def oracle_run():
    return oracle_chain(CFG, STEPS)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_decode_matches_oracle(world, oracle_run):
    lg_ref, toks_ref, margins, b2_ref = oracle_run
    res = _run(world, "decode", CFG, toks_ref)
    check_chain(res, lg_ref, toks_ref, margins, f"tp{world}")
    assert res["batch2"] == b2_ref, "batch-2 slot-1 greedy sequence"


@pytest.mark.parametrize("world", [2, 8])
def test_tp_llama70b_widths_two_layers(world):
    """Llama-3-70B-width shards (at TP8: 8 q + 1 kv head, 3584 ffn columns =
    14 super-blocks of ffn_down, 16032 vocab rows per rank)."""
    import torch

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    lg_ref, toks_ref, margins, _ = oracle_chain(CFG70, STEPS70, batch2=False)
    res = _run(world, "decode", CFG70, toks_ref)
    check_chain(res, lg_ref, toks_ref, margins, f"70B-width tp{world}")


def test_tp_peer_timeout_reports_error():
    res = _run(2, "timeout")
    assert res["rc"] == -4, res  # FB_ERR_DEVICE
    assert "0x" in res.get("msg", "")
    assert res["err_after"] == 0
