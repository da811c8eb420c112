"""The persistent batch-1 decode step (one cooperative kernel per step,
csrc/decode_step.cu) against the per-op kernel chain and the oracle.

Both paths must produce the same bits: logits of every step, the KV rows
the step writes, the residual stream and the attention output, over
qwen3 and llama-compat semantics and GQA groups 2, 4 and 8 (the 8-group
shape at Llama-3-70B widths: hidden 8192, 64 q / 8 kv heads, three ring
stages), with contexts that give the splits several chunks each.
"""
import numpy as np
import pytest

import ferrite_b200 as fb
from conftest import O, synth_weights, tiny_config

pytestmark = pytest.mark.gpu

SHAPES = {
    "qwen3-g4": dict(),
    "llama-g4": dict(qk_norm=0, rope_mode=0),
    "g2": dict(n_heads=8, n_kv_heads=4),
    "g8-wide": dict(hidden=8192, n_heads=64, n_kv_heads=8, ffn=28672, qk_norm=0, rope_mode=0,
                    rope_theta=5e5, eps=1e-5),
}


@pytest.mark.parametrize("shape", sorted(SHAPES))
def test_persistent_step_equals_kernel_chain(fbctx, shape):
    cfg = tiny_config(max_ctx=1200, max_batch=1, vocab=2048, **SHAPES[shape])
    models = []
    for persistent in (True, False):
        m = fb.Model(fbctx, cfg)
        m.synth(seed=13)
        m.finalize()
        supported = m.set_persistent(persistent)
        assert supported, f"{shape}: the persistent step should support this shape"
        m.synth_kv(seed=4, ctx=1000)
        models.append(m)
    toks = [int(t) for t in O.synth_tokens(6, 5, cfg["vocab"])]
    for i, t in enumerate(toks):
        got, want = (m.forward([t], 1000 + i) for m in models)
        assert np.array_equal(got, want), f"{shape} step {i}: logits differ"
        for name in ("x", "attn", "q"):
            a, b = (m.read_activation(name) for m in models)
            assert np.array_equal(a, b), f"{shape} step {i}: activation {name} differs"
    for layer in (0, cfg["n_layers"] - 1):
        for which in (0, 1):
            a, b = (m.read_kv(layer, which, 1000 + len(toks) - 1) for m in models)
            assert np.array_equal(a, b), f"{shape}: kv row l{layer} {which}"
    assert models[0].launches_per_step() == 2  # the persistent kernel + argmax
    assert models[1].launches_per_step() > 2
    for m in models:
        m.close()
    assert fbctx.error_word() == 0


def test_persistent_step_matches_oracle_70b_widths(fbctx):
    """Llama-3-70B widths at 2 layers on one GPU (three ring stages, 8-head
    GQA groups) against the oracle, bit for bit, from a 600-token context."""
    cfg = tiny_config(n_layers=2, hidden=8192, n_heads=64, n_kv_heads=8, ffn=28672, vocab=4096, max_ctx=640,
                      max_batch=1, qk_norm=0, rope_mode=0, rope_theta=5e5, eps=1e-5)
    dm = fb.Model(fbctx, cfg)
    dm.synth(seed=8)
    dm.finalize()
    assert dm.set_persistent(True)
    dm.synth_kv(seed=2, ctx=600)
    om = O.Model(cfg, synth_weights(cfg, 8))
    om.synth_kv(2, 600)
    for i, t in enumerate([7, 1000, 4095]):
        got, want = dm.forward([t], 600 + i), om.forward([t], 600 + i)
        assert np.array_equal(got, want), f"step {i}: not bit-identical to the oracle"
    om.close()
    dm.close()
    assert fbctx.error_word() == 0
