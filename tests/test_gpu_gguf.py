"""GGUF ingest on the device: a file written from the parity weights loads
into a model whose decode steps equal the oracle model built from the same
weights (qwen3 and llama semantics), tied embeddings (no output tensor) use
token_embd as the lm_head, and an unsupported tensor type is rejected."""
import os

import numpy as np
import pytest

import ferrite_b200 as fb
from conftest import O, assert_close, tiny_config, tiny_weights
from gguf_writer import model_tensors, write_gguf

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("arch", ["qwen3", "llama"])
def test_load_and_decode(fbctx, tmp_path, arch):
    cfg = tiny_config() if arch == "qwen3" else tiny_config(qk_norm=0, rope_mode=0)
    w = tiny_weights(cfg, seed=31)
    p = os.path.join(tmp_path, "m.gguf")
    write_gguf(p, arch, cfg, model_tensors(w))
    dm = fb.Model.from_gguf(fbctx, p, max_ctx=cfg["max_ctx"], max_batch=1)
    om = O.Model(cfg, w)
    for i, t in enumerate([9, 100, 7]):
        got, want = dm.forward([t], i), om.forward([t], i)
        assert np.array_equal(got, want), f"step {i}: max err {np.abs(got - want).max()}"
    dm.close()


def test_tied_embeddings(fbctx, tmp_path):
    cfg = tiny_config()
    w = tiny_weights(cfg, seed=32)
    w_tied = dict(w, output=w["tok_embd"])
    p = os.path.join(tmp_path, "tied.gguf")
    write_gguf(p, "qwen3", cfg, model_tensors(w, tied=True))
    dm = fb.Model.from_gguf(fbctx, p, max_ctx=cfg["max_ctx"])
    om = O.Model(cfg, w_tied)
    assert_close(dm.forward([5], 0), om.forward([5], 0), what="tied lm_head")
    dm.close()


def test_unsupported_tensor_type(fbctx, tmp_path):
    cfg = tiny_config()
    w = tiny_weights(cfg, seed=33)
    ts = model_tensors(w)
    name, _, r, c, a = ts[5]
    ts[5] = (name, 8, r, c, a)  # Q8_0
    p = os.path.join(tmp_path, "q8.gguf")
    write_gguf(p, "qwen3", cfg, ts)
    with pytest.raises(fb.FerriteError, match="ggml type 8"):
        fb.Model.from_gguf(fbctx, p, max_ctx=cfg["max_ctx"])
