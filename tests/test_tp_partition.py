"""Tensor-parallel partitioning of the decode path, checked on the CPU.

The device shards a model the way fb_model_create_tp documents: column-
parallel projections (attn_q/k/v, ffn_gate/up, output) keep a slice of the
output rows and need no exchange; row-parallel ones (attn_output, ffn_down)
keep a slice of the input columns -- whole 256-value super-blocks, so the
Q8_K blocks of the activations are the same blocks -- and each rank's
binary64 partial row sums are added in rank order and rounded to f32 once.
These tests restate that with the oracle (oracle/kquant.c or_qmatmul64) and
require the result to equal the unsharded QMatMul bit for bit, for the
Llama-3-70B and Qwen3-8B projection widths at 2, 4 and 8 ranks.  The last
test runs the same partition as two gloo ranks (world size 2, CPU), with the
exchange as a torch.distributed all-gather, and the fb_comm handle exchange
helper over the same process group.
"""
import os

import numpy as np
import pytest

from conftest import O, gaussian_qweight


def row_parallel(dtype, w, n, k, x, world):
    kc = k // world
    parts = [O.qmatmul64(dtype, O.shard_blocks(dtype, w, n, k, 0, n, r * kc, kc), n, kc, x[:, r * kc:(r + 1) * kc])
             for r in range(world)]
    acc = np.zeros_like(parts[0])
    for p in parts:  # rank order, as the device's residual + RMSNorm kernel
        acc = acc + p
    return acc.astype(np.float32)


# (dtype, n, k): attn_output and ffn_down of Llama-3-70B (k = 8192, 28672) and
# Qwen3-8B (k = 4096, 12288), with n reduced (rows are independent)
ROW_PARALLEL = [(O.Q4_K, 64, 8192), (O.Q6_K, 64, 28672), (O.Q4_K, 64, 4096), (O.Q6_K, 64, 12288)]


@pytest.mark.parametrize("dtype,n,k", ROW_PARALLEL)
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("batch", [1, 4])
def test_row_parallel_sum_is_exact(dtype, n, k, world, batch):
    w = gaussian_qweight(dtype, n, k, seed=k + dtype)
    x = np.random.default_rng(k + batch).normal(0, 1, (batch, k)).astype(np.float32)
    full = O.qmatmul(dtype, w, n, k, x)
    got = row_parallel(dtype, w, n, k, x, world)
    assert np.array_equal(got.view(np.uint32), full.view(np.uint32)), \
        f"{int((got != full).sum())} elements differ from the unsharded QMatMul"


def test_row_parallel_partials_round_like_full():
    """The unrounded full sum equals the rank-order sum of the partials."""
    dtype, n, k = O.Q6_K, 32, 28672
    w = gaussian_qweight(dtype, n, k, seed=3)
    x = np.random.default_rng(9).normal(0, 1, (2, k)).astype(np.float32)
    full64 = O.qmatmul64(dtype, w, n, k, x)
    assert np.array_equal(full64.astype(np.float32), O.qmatmul(dtype, w, n, k, x))
    got = row_parallel(dtype, w, n, k, x, 8)
    assert np.array_equal(got, full64.astype(np.float32))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_column_parallel_is_a_row_slice(world):
    dtype, n, k = O.Q4_K, 512, 2048
    w = gaussian_qweight(dtype, n, k, seed=5)
    x = np.random.default_rng(1).normal(0, 1, (3, k)).astype(np.float32)
    full = O.qmatmul(dtype, w, n, k, x)
    nr = n // world
    for r in range(world):
        part = O.qmatmul(dtype, O.shard_blocks(dtype, w, n, k, r * nr, nr, 0, k), nr, k, x)
        assert np.array_equal(part, full[:, r * nr:(r + 1) * nr])


def test_vocab_parallel_argmax():
    """Global argmax = merge of the ranks' (max, first index) pairs, ties to
    the smaller global index (the device merge)."""
    rng = np.random.default_rng(0)
    for world in (2, 4, 8):
        logits = rng.normal(0, 1, 1024).astype(np.float32)
        logits[[100, 900]] = 7.0  # a tie across ranks
        per = 1024 // world
        pairs = []
        for r in range(world):
            s = logits[r * per:(r + 1) * per]
            i = int(np.argmax(s))
            pairs.append((float(s[i]), r * per + i))
        best = min(pairs, key=lambda p: (-p[0], p[1]))
        assert best[1] == int(np.argmax(logits)) == 100


def _gloo_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dtype, n, k = O.Q6_K, 32, 12288
        w = gaussian_qweight(dtype, n, k, seed=21)
        x = np.random.default_rng(4).normal(0, 1, (2, k)).astype(np.float32)
        kc = k // world
        mine = O.qmatmul64(dtype, O.shard_blocks(dtype, w, n, k, 0, n, rank * kc, kc), n, kc,
                           x[:, rank * kc:(rank + 1) * kc])
        parts = [torch.zeros(mine.shape, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(mine))
        acc = np.zeros_like(mine)
        for p in parts:
            acc = acc + p.numpy()
        ok = np.array_equal(acc.astype(np.float32), O.qmatmul(dtype, w, n, k, x))
        # handle exchange of the fb_comm setup (64-byte blobs, rank order)
        import sys
        sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                        "ferrite-llm_b200"))
        import ferrite_b200 as fb
        hs = fb.Comm.gather_handles(bytes([rank]) * fb.COMM_HANDLE_BYTES, world)
        ok = ok and hs == [bytes([r]) * fb.COMM_HANDLE_BYTES for r in range(world)]
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_partition_and_handles():
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(2))
    assert res == [(0, True), (1, True)]
