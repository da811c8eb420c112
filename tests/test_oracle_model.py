"""CPU checks of the oracle's Llama/Qwen3 forward (no GPU)."""
import numpy as np
import pytest

from conftest import O, tiny_config, tiny_weights, synth_weights


@pytest.fixture(scope="module")
def small():
    cfg = tiny_config(n_layers=2, hidden=512, n_heads=4, n_kv_heads=2, ffn=768, vocab=1024, max_ctx=64)
    return cfg, tiny_weights(cfg, seed=3)


def test_prefill_equals_token_by_token(small):
    cfg, w = small
    toks = O.synth_tokens(2, 9, cfg["vocab"])
    a = O.Model(cfg, w, nthreads=4)
    all_logits = a.forward(toks, 0, all_logits=True)
    b = O.Model(cfg, w, nthreads=4)
    step = [b.forward([t], i) for i, t in enumerate(toks)]
    np.testing.assert_allclose(all_logits, np.stack(step), rtol=1e-5, atol=1e-5)
    assert a.length == 9 and b.length == 9


def test_kv_cache_rounding_and_overwrite(small):
    cfg, w = small
    m = O.Model(cfg, w, nthreads=2)
    m.forward([1, 2, 3], 0)
    k = m.read_kv(0, 0, 2)
    assert np.array_equal(k, k.astype(np.float16).astype(np.float32))
    # re-running position 2 with another token overwrites it (cache truncation)
    m.forward([5], 2)
    assert m.length == 3
    assert not np.array_equal(m.read_kv(0, 0, 2), k)


def test_llama_compat_mode_differs(small):
    cfg, w = small
    toks = [3, 4, 5]
    q = O.Model(cfg, w).forward(toks, 0)
    l = O.Model(dict(cfg, qk_norm=0, rope_mode=0), w).forward(toks, 0)
    assert not np.allclose(q, l)


def test_rope_modes():
    x = np.arange(2 * 8, dtype=np.float32).reshape(2, 8) / 10
    for mode in (0, 1):
        y = x.copy()
        O.lib().or_rope(O._p(y), 2, 8, 0, 1e4, mode)
        assert np.array_equal(y, x)  # position 0 is the identity
        y = x.copy()
        O.lib().or_rope(O._p(y), 2, 8, 5, 1e4, mode)
        # rotation preserves the norm of each pair
        if mode == 0:
            pa, pb = x.reshape(2, 4, 2), y.reshape(2, 4, 2)
            np.testing.assert_allclose(np.linalg.norm(pa, axis=2), np.linalg.norm(pb, axis=2), rtol=1e-6)
        else:
            n0 = np.hypot(x[:, :4], x[:, 4:])
            n1 = np.hypot(y[:, :4], y[:, 4:])
            np.testing.assert_allclose(n0, n1, rtol=1e-6)


def test_synth_model_runs():
    cfg = tiny_config(n_layers=1, hidden=256, n_heads=2, n_kv_heads=1, ffn=512, vocab=512, max_ctx=32)
    w = synth_weights(cfg, seed=1)
    m = O.Model(cfg, w)
    lg = m.forward([1, 2], 0)
    assert np.isfinite(lg).all() and lg.std() > 0.1
    m.synth_kv(9, 16)
    assert m.length == 16
    m.forward([7], 16)
    assert m.length == 17


def test_tensor_parallel_sharding_identity():
    """Column-split (output rows) and row-split (input super-blocks, summed
    partials) reproduce the unsharded QMatMul — the TP plan for the 70B
    config, simulated on CPU ranks."""
    from conftest import gaussian_qweight
    n, k = 64, 2048
    w = gaussian_qweight(O.Q4_K, n, k, seed=8)
    x = np.random.default_rng(9).normal(0, 1, (3, k)).astype(np.float32)
    full = O.qmatmul(O.Q4_K, w, n, k, x)
    for tp in (2, 4, 8):
        cols = np.concatenate([O.qmatmul(O.Q4_K, w[r * n // tp:(r + 1) * n // tp], n // tp, k, x)
                               for r in range(tp)], axis=1)
        assert np.array_equal(cols, full)
        nb = k // 256 // tp
        parts = []
        for r in range(tp):
            ws = np.ascontiguousarray(w.reshape(n, -1, 144)[:, r * nb:(r + 1) * nb].reshape(n, -1))
            parts.append(O.qmatmul(O.Q4_K, ws, n, k // tp, x[:, r * nb * 256:(r + 1) * nb * 256]))
        np.testing.assert_allclose(np.sum(parts, axis=0), full, rtol=1e-4, atol=1e-4)
