"""Shared pytest setup: the `gpu` marker, import paths, and helpers that
build identical weights for the CUDA path and the CPU oracle."""
from __future__ import annotations

import functools
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "ferrite-llm_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

from oracle import oracle as O  # noqa: E402

# float tolerance of the north-star parity bar: 1e-3 relative / 1e-2 absolute
RTOL, ATOL = 1e-3, 1e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def assert_close(got, ref, rtol=RTOL, atol=ATOL, what=""):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(got - ref)
    bound = atol + rtol * np.abs(ref)
    bad = err > bound
    if bad.any():
        i = int(np.argmax(err - bound))
        raise AssertionError(f"{what}: {int(bad.sum())}/{bad.size} outside tol; worst idx {i}: got {got.flat[i]} "
                             f"ref {ref.flat[i]} (max abs err {err.max():.3g})")


@functools.lru_cache(maxsize=16)
def gaussian_qweight(dtype: int, n: int, k: int, seed: int, sigma: float = 0.02) -> np.ndarray:
    """W[n, k] ~ N(0, sigma) (numpy PCG64 seed) quantized by the oracle.
    Cached: callers must not modify the returned array."""
    w = np.random.default_rng(seed).normal(0.0, sigma, size=(n, k)).astype(np.float32)
    q = O.quantize(dtype, w)
    q.setflags(write=False)
    return q


def tiny_config(**over) -> dict:
    cfg = dict(n_layers=2, hidden=1024, n_heads=8, n_kv_heads=2, head_dim=128, ffn=2048, vocab=4096,
               max_ctx=256, max_batch=4, rope_theta=1e6, eps=1e-6, qk_norm=1, rope_mode=1, kv_f16=1)
    cfg.update(over)
    return cfg


def tiny_weights(cfg: dict, seed: int = 7, down_q6: bool = True) -> dict:
    """Gaussian weights quantized like Q4_K_M (ffn_down / output Q6_K) for a
    small model; returns oracle-style specs (dtype, rows, cols, array)."""
    rng = np.random.default_rng(seed)
    H, F, V = cfg["hidden"], cfg["ffn"], cfg["vocab"]
    qd, kd = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]

    def q(dtype, n, k):
        w = rng.normal(0.0, 0.02, size=(n, k)).astype(np.float32)
        return (dtype, n, k, O.quantize(dtype, w))

    def v(n):
        return (O.F32, 1, n, (1.0 + rng.normal(0.0, 0.02, size=n)).astype(np.float32))

    layers = []
    for _ in range(cfg["n_layers"]):
        layers.append(dict(
            attn_norm=v(H), wq=q(O.Q4_K, qd, H), wk=q(O.Q4_K, kd, H), wv=q(O.Q4_K, kd, H),
            wo=q(O.Q4_K, H, qd), q_norm=v(cfg["head_dim"]), k_norm=v(cfg["head_dim"]), ffn_norm=v(H),
            w_gate=q(O.Q4_K, F, H), w_up=q(O.Q4_K, F, H), w_down=q(O.Q6_K if down_q6 else O.Q4_K, H, F)))
    return dict(tok_embd=q(O.Q4_K, V, H), out_norm=v(H), output=q(O.Q6_K, V, H), layers=layers)


# oracle layer keys -> GGUF tensor names
GGUF_NAMES = dict(attn_norm="attn_norm", wq="attn_q", wk="attn_k", wv="attn_v", wo="attn_output",
                  q_norm="attn_q_norm", k_norm="attn_k_norm", ffn_norm="ffn_norm", w_gate="ffn_gate",
                  w_up="ffn_up", w_down="ffn_down")


def load_into_device_model(model, weights: dict):
    for name, key in (("token_embd", "tok_embd"), ("output_norm", "out_norm"), ("output", "output")):
        dt, r, c, a = weights[key]
        model.set_tensor(name, -1, dt, r, c, a)
    for li, lw in enumerate(weights["layers"]):
        for key, name in GGUF_NAMES.items():
            dt, r, c, a = lw[key]
            model.set_tensor(name, li, dt, r, c, a)
    model.finalize()


def synth_weights(cfg: dict, seed: int) -> dict:
    """Oracle-side copy of fb_model_synth's random-init tensors."""
    return O.synth_model_weights(cfg, seed)


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="session")
def fbctx(torch_cuda):
    import ferrite_b200 as fb
    torch = torch_cuda
    torch.cuda.init()
    ctx = fb.Context(0, torch.cuda.current_stream().cuda_stream)
    yield ctx
    ctx.sync()
