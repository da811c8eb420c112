"""Batched prefill: the causal prefill attention op against an f64 reference,
and the model's batched prompt forward against the oracle.

The model test feeds prompts of 17..300 tokens (one and several 64-token
pages, a continuation at pos > 0) through fb_model_forward's batched path --
the float form of every projection (as candle's CUDA QMatMul runs more than
8 rows: dequantized weights, float matmul; here tensor cores with fp16
operands) and tensor-core attention, the last row's lm_head in float too --
and compares the last token's logits with the oracle's float forward
(matmul_mode 1) at the parity bar (1e-3 relative / 1e-2 absolute), the KV
rows at 1e-2 (16-bit operands of the projections and fp16 storage), and the
greedy tokens of the integer
decode steps that follow (identical unless the oracle's top-2 margin is a
near tie).  candle's CPU build runs the prompt through the integer Q8_K path
instead, which differs from the float path by the 8-bit activation rounding
(several percent on these random-init logits).
"""
import math

import numpy as np
import pytest

import ferrite_b200 as fb
from conftest import O, assert_close, load_into_device_model, tiny_config, tiny_weights

pytestmark = pytest.mark.gpu

TIE_MARGIN = 2e-2


def causal_reference(q, kp, vp, bt, pos0, page):
    """q [T, nh, hd] f32, kp/vp [num_pages, nkv, page, hd] fp16 (token-major)."""
    T, nh, hd = q.shape
    nkv = kp.shape[1]
    g = nh // nkv
    L = pos0 + T
    K = np.stack([kp[bt[i // page], :, i % page] for i in range(L)]).astype(np.float64)
    V = np.stack([vp[bt[i // page], :, i % page] for i in range(L)]).astype(np.float64)
    out = np.zeros((T, nh, hd))
    for t in range(T):
        n = pos0 + t + 1
        for h in range(nh):
            sc = K[:n, h // g] @ q[t, h].astype(np.float64) / math.sqrt(hd)
            p = np.exp(sc - sc.max())
            out[t, h] = (p / p.sum()) @ V[:n, h // g]
    return out


@pytest.mark.parametrize("nh,nkv", [(32, 8), (64, 8), (8, 8)])
@pytest.mark.parametrize("pos0,T", [(0, 1), (0, 17), (0, 64), (37, 100), (130, 200)])
def test_attn_prefill_op(fbctx, torch_cuda, nh, nkv, pos0, T):
    torch = torch_cuda
    rng = np.random.default_rng(nh + 7 * pos0 + T)
    hd, page = 128, 64
    max_pages = (pos0 + T + page - 1) // page + 1
    num_pages = max_pages + 4
    bt = rng.permutation(num_pages)[:max_pages].astype(np.int32)
    kp = rng.normal(0, 1, (num_pages, nkv, page, hd)).astype(np.float16)
    vp = rng.normal(0, 1, (num_pages, nkv, page, hd)).astype(np.float16)
    q = rng.normal(0, 1, (T, nh, hd)).astype(np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    qd, kd, vd, btd = t(q), t(kp.transpose(0, 1, 3, 2)), t(vp), t(bt)
    out = torch.full((T, nh, hd), float("nan"), dtype=torch.float32, device="cuda")
    fb.attn_prefill(fbctx, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), btd.data_ptr(), max_pages, num_pages, pos0, T,
                    nh, nkv, hd, page, 1.0 / math.sqrt(hd), out.data_ptr())
    ref = causal_reference(q, kp, vp, bt, pos0, page)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-4, atol=1e-5)
    assert fbctx.error_word() == 0


@pytest.fixture(scope="module", params=["qwen3", "llama"])
def pair(request, fbctx):
    over = dict(max_ctx=512) if request.param == "qwen3" else dict(max_ctx=512, qk_norm=0, rope_mode=0)
    cfg = tiny_config(**over)
    w = tiny_weights(cfg, seed=23)
    dm = fb.Model(fbctx, cfg)
    load_into_device_model(dm, w)
    return cfg, dm, O.Model(cfg, w)


@pytest.mark.parametrize("n", [17, 64, 150, 300])
def test_batched_prefill_logits(pair, n):
    cfg, dm, om = pair
    dm.clear_cache()
    om.clear()
    toks = O.synth_tokens(n + 3, n, cfg["vocab"])
    got = dm.forward(toks, 0)
    ref = om.forward(toks, 0, matmul_mode=1)
    assert_close(got, ref, what=f"batched prefill of {n} tokens: last-token logits")
    for layer in (0, cfg["n_layers"] - 1):
        for p in (0, n // 2, n - 1):
            for which in (0, 1):
                # intermediate values: 16-bit operands compound over the layer stack
                assert_close(dm.read_kv(layer, which, p), om.read_kv(layer, which, p), rtol=1e-2, atol=1e-2,
                             what=f"kv l{layer} {which} p{p}")


def test_prefill_continuation_and_decode(pair):
    """20 prompt tokens, then 45 more at pos 20 (both batched), then greedy decode."""
    cfg, dm, om = pair
    dm.clear_cache()
    om.clear()
    toks = O.synth_tokens(99, 65, cfg["vocab"])
    dm.forward(toks[:20], 0)
    om.forward(toks[:20], 0, matmul_mode=1)
    got = dm.forward(toks[20:], 20)
    ref = om.forward(toks[20:], 20, matmul_mode=1)
    assert_close(got, ref, what="continued prefill logits")
    tok_d = tok_o = int(np.argmax(ref))
    pos = 65
    for i in range(16):
        lo = om.forward([tok_o], pos)
        nd = int(dm.decode_greedy([tok_d], [pos])[0])
        no = int(np.argmax(lo))
        if nd != no:
            s = np.sort(lo)
            assert s[-1] - s[-2] < TIE_MARGIN, f"decode step {i} after prefill: {nd} != {no}"
            break
        tok_d = tok_o = no
        pos += 1


@pytest.mark.parametrize("n", [5, 40, 300])
def test_forward_all_logits(pair, n):
    """Multi-token forward: the logits of every token against the oracle's
    (float forward for the batched path, integer decode steps for short
    inputs)."""
    cfg, dm, om = pair
    dm.clear_cache()
    om.clear()
    toks = O.synth_tokens(n + 11, n, cfg["vocab"])
    got = dm.forward_all(toks, 0)
    ref = om.forward(toks, 0, all_logits=True, matmul_mode=1 if n >= 17 else 0)
    assert got.shape == ref.shape == (n, cfg["vocab"])
    assert_close(got, ref, what=f"all logits of {n} tokens")
