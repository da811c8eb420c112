"""Full decode-step parity of the device model against the oracle forward:
logits per step within tolerance, KV rows, greedy token identity over 64
steps (qwen3 and llama-compat semantics), batched decode, and the on-device
random-init model against the oracle's copy of the same generator."""
import numpy as np
import pytest

import ferrite_b200 as fb
from conftest import O, assert_close, load_into_device_model, synth_weights, tiny_config, tiny_weights

pytestmark = pytest.mark.gpu

# Logits of a random-init model: keep a tie guard.  A greedy step whose
# top-2 oracle margin is below this is reported, not failed.
TIE_MARGIN = 2e-2


def device_model(fbctx, cfg, weights):
    m = fb.Model(fbctx, cfg)
    load_into_device_model(m, weights)
    return m


@pytest.fixture(scope="module", params=["qwen3", "llama"])
def pair(request, fbctx):
    over = {} if request.param == "qwen3" else dict(qk_norm=0, rope_mode=0)
    cfg = tiny_config(**over)
    w = tiny_weights(cfg, seed=11)
    return cfg, w, device_model(fbctx, cfg, w), O.Model(cfg, w)


def test_logits_first_tokens(pair):
    cfg, w, dm, om = pair
    dm.clear_cache()
    om.clear()
    toks = O.synth_tokens(5, 6, cfg["vocab"])
    for i, t in enumerate(toks):
        got = dm.forward([int(t)], i)
        ref = om.forward([int(t)], i)
        assert_close(got, ref, what=f"step {i}")


def test_kv_rows_match(pair):
    cfg, w, dm, om = pair
    dm.clear_cache()
    om.clear()
    toks = [3, 17, 99]
    dm.forward(toks, 0)
    om.forward(toks, 0)
    for layer in range(cfg["n_layers"]):
        for which in (0, 1):
            for p in range(3):
                assert_close(dm.read_kv(layer, which, p), om.read_kv(layer, which, p), rtol=2e-3, atol=2e-3,
                             what=f"kv l{layer} {which} p{p}")


def test_greedy_64_steps_identical(pair):
    cfg, w, dm, om = pair
    dm.clear_cache()
    om.clear()
    prompt = [int(t) for t in O.synth_tokens(2, 8, cfg["vocab"])]
    ref_logits = om.forward(prompt, 0)
    dm.forward(prompt, 0)
    tok_o = int(np.argmax(ref_logits))
    tok_d = tok_o
    ties = 0
    pos = len(prompt)
    for step in range(64):
        nxt_d = int(dm.decode_greedy([tok_d], [pos])[0])
        lg = om.forward([tok_o], pos)
        nxt_o = int(np.argmax(lg))
        top2 = np.sort(lg)[-2:]
        if nxt_d != nxt_o:
            assert top2[1] - top2[0] < TIE_MARGIN, f"step {step}: device {nxt_d} vs oracle {nxt_o}"
            ties += 1
            break
        tok_d = tok_o = nxt_o
        pos += 1
    assert ties == 0 or step > 0


def test_batched_decode_matches_single(fbctx):
    cfg = tiny_config()
    w = tiny_weights(cfg, seed=5)
    dm = device_model(fbctx, cfg, w)
    prompts = [[1, 2, 3], [40, 41, 42], [7, 8, 9]]
    # batch: slot i holds prompt i
    for j in range(3):
        nxt = dm.decode_greedy([p[j] for p in prompts], [j, j, j])
    singles = []
    for p in prompts:
        om = O.Model(cfg, w)
        singles.append(int(np.argmax(om.forward(p, 0))))
    assert list(nxt) == singles


def test_synth_model_parity(fbctx):
    cfg = tiny_config(n_layers=2, vocab=2048)
    dm = fb.Model(fbctx, cfg)
    dm.synth(seed=42)
    dm.finalize()
    om = O.Model(cfg, synth_weights(cfg, seed=42))
    for i, t in enumerate([5, 6, 7]):
        assert_close(dm.forward([t], i), om.forward([t], i), what=f"synth step {i}")


def test_synth_kv_then_decode(fbctx):
    cfg = tiny_config(max_ctx=512, vocab=2048)
    dm = fb.Model(fbctx, cfg)
    dm.synth(seed=3)
    dm.finalize()
    om = O.Model(cfg, synth_weights(cfg, seed=3))
    dm.synth_kv(seed=8, ctx=300)
    om.synth_kv(8, 300)
    for layer in (0, 1):
        assert np.array_equal(dm.read_kv(layer, 1, 299), om.read_kv(layer, 1, 299))
    assert_close(dm.forward([11], 300), om.forward([11], 300), what="decode at ctx 300")


@pytest.mark.parametrize("n_kv,ctx", [(2, 1500), (1, 3000), (4, 2100), (8, 4500)])
def test_long_context_many_splits(fbctx, n_kv, ctx):
    """Few kv heads and long contexts: the attention grid takes 32 or 64
    splits per kv head (one wave of CTAs); with 8 kv heads at ctx 4500 it
    keeps 16 splits of 5 chunks each, more than the ring's 4 stages.  The
    result must not change."""
    cfg = tiny_config(n_heads=4 * n_kv, n_kv_heads=n_kv, max_ctx=ctx + 8, vocab=2048)
    dm = fb.Model(fbctx, cfg)
    dm.synth(seed=5)
    dm.finalize()
    om = O.Model(cfg, synth_weights(cfg, seed=5))
    dm.synth_kv(seed=9, ctx=ctx)
    om.synth_kv(9, ctx)
    for i, t in enumerate([17, 4]):
        got, want = dm.forward([t], ctx + i), om.forward([t], ctx + i)
        assert_close(got, want, what=f"decode at ctx {ctx + i}")
        assert np.array_equal(got, want), f"ctx {ctx + i}: not bit-identical to the oracle"


def test_bad_inputs_rejected(fbctx):
    cfg = tiny_config()
    dm = fb.Model(fbctx, cfg)
    with pytest.raises(fb.FerriteError):
        dm.forward([1], 0)  # not finalized
    dm.synth(1)
    dm.finalize()
    with pytest.raises(fb.FerriteError):
        dm.forward([cfg["vocab"]], 0)
    with pytest.raises(fb.FerriteError):
        dm.decode_greedy([1], [cfg["max_ctx"]])
    assert fbctx.error_word() == 0


@pytest.mark.parametrize("batch,ragged", [(16, False), (32, False), (16, True)])
def test_large_batch_single_split_per_kv_head(fbctx, torch_cuda, batch, ragged):
    """16 or 32 sequences x 8 kv heads fill one wave (or two) of attention
    CTAs with one split each: every CTA walks the whole context (18 chunks,
    several passes over its 4-stage shared-memory ring); at 32 rows the
    projections take the widest MMA consumer (four 8-column n-tiles).  With
    `ragged` every sequence decodes at its own position (1 to 1100 tokens of
    context).  Each sequence's logits must equal the oracle's single-sequence
    forward bit for bit."""
    torch = torch_cuda
    ctx = 1100
    cfg = tiny_config(n_heads=32, n_kv_heads=8, max_ctx=ctx + 8, max_batch=batch, vocab=2048)
    dm = fb.Model(fbctx, cfg)
    dm.synth(seed=5)
    dm.finalize()
    dm.synth_kv(seed=9, ctx=ctx)
    w = synth_weights(cfg, seed=5)
    toks = [(7 * i + 3) % cfg["vocab"] for i in range(batch)]
    tok_d = torch.tensor(toks, dtype=torch.int32, device="cuda")
    positions = [ctx - 73 * i for i in range(batch)] if ragged else [ctx] * batch
    if ragged:
        positions[-1] = 0  # a sequence with only the new token
    pos_d = torch.tensor(positions, dtype=torch.int32, device="cuda")
    logits = torch.empty((batch, cfg["vocab"]), dtype=torch.float32, device="cuda")
    dm.decode_dev(tok_d.data_ptr(), pos_d.data_ptr(), batch, logits_ptr=logits.data_ptr())
    torch.cuda.synchronize()
    got = logits.cpu().numpy()
    for i, t in enumerate(toks):
        om = O.Model(cfg, w)
        om.synth_kv(9, ctx)
        want = om.forward([t], positions[i])
        assert_close(got[i], want, what=f"sequence {i} at position {positions[i]}")
        assert np.array_equal(got[i], want), f"sequence {i}: not bit-identical to the oracle"
    assert fbctx.error_word() == 0
