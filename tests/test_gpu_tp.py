"""Tensor-parallel decode on 2 (and 4) GPUs against the oracle.

Each rank is a child process on its own GPU (one process per GPU, gloo for
the host-side handle exchange and barriers); ranks map each other's fb_comm
regions through CUDA IPC.  The sharded random-init model must give the
oracle's logits (tolerance of the parity bar, over the gathered vocab
slices) and the oracle's greedy tokens, at batch 1 and batch 2.  The
failure test lets one rank never step: the other rank's bounded device waits
run out (nothing sets the flag it waits on), the step reports FB_ERR_DEVICE
with the peer-timeout bit and the context stays usable.  Skipped with fewer
than two GPUs.
"""
import os
import socket

import numpy as np
import pytest

from conftest import O, assert_close, synth_weights

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG = dict(n_layers=2, hidden=1024, n_heads=16, n_kv_heads=4, head_dim=128, ffn=2048, vocab=4096, max_ctx=128,
           max_batch=4, rope_theta=1e6, eps=1e-6, qk_norm=1, rope_mode=1, kv_f16=1)
SEED = 77
PROMPT = [11, 400, 7, 3000, 25]
STEPS = 24
ERRBIT_PEER_TIMEOUT = 1 << 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, mode, q):
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
        comm = fb.Comm.connect(ctx, CFG["max_batch"], CFG["hidden"])
        model = fb.Model(ctx, CFG, comm)
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
            tok = int(np.argmax(full))
            toks = [tok]
            for i in range(STEPS - 1):
                tok = int(model.decode_greedy([tok], [len(PROMPT) + i])[0])
                toks.append(tok)
            # batch 2: slot 1 decodes the same prompt token by token
            b2 = []
            t1 = PROMPT[0]
            for i in range(len(PROMPT) + 4):
                nxt = model.decode_greedy([toks[0], t1], [len(PROMPT) + STEPS - 1, i])
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


def _run(world, mode):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, q)) for r in range(world)]
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


@pytest.fixture(scope="module")
def oracle_run():
    om = O.Model(CFG, synth_weights(CFG, SEED))
    lg = om.forward(PROMPT, 0)
    toks, margins = [], []
    tok = int(np.argmax(lg))
    toks.append(tok)
    for i in range(STEPS - 1):
        l2 = om.forward([tok], len(PROMPT) + i)
        s = np.sort(l2)
        margins.append(float(s[-1] - s[-2]))
        tok = int(np.argmax(l2))
        toks.append(tok)
    om.close()
    # slot-1 sequence of the batch-2 phase: prompt, then greedy continuation
    om2 = O.Model(CFG, synth_weights(CFG, SEED))
    b2, t1 = [], PROMPT[0]
    for i in range(len(PROMPT) + 4):
        l2 = om2.forward([t1], i)
        nxt = int(np.argmax(l2))
        t1 = PROMPT[i + 1] if i + 1 < len(PROMPT) else nxt
        b2.append(nxt)
    om2.close()
    return lg, toks, margins, b2


@pytest.mark.parametrize("world", [2, 4])
def test_tp_decode_matches_oracle(world, oracle_run):
    lg_ref, toks_ref, margins, b2_ref = oracle_run
    res = _run(world, "decode")
    assert res["err"] == 0
    assert_close(res["logits"], lg_ref, what=f"tp{world} prompt logits (gathered vocab slices)")
    got = res["tokens"]
    for i, (a, b) in enumerate(zip(got, toks_ref)):
        if a != b:
            assert i > 0 and margins[i - 1] < 2e-2, f"tp{world} greedy token {i}: {a} != {b}"
            break
    assert res["batch2"] == b2_ref, "batch-2 slot-1 greedy sequence"


def test_tp_peer_timeout_reports_error():
    res = _run(2, "timeout")
    assert res["rc"] == -4, res  # FB_ERR_DEVICE
    assert "0x" in res.get("msg", "")
    assert res["err_after"] == 0
