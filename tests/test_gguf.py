"""GGUF metadata parsing (CPU): the model config of llama / qwen3 files,
array-valued metadata skipped, and malformed files rejected with an error
status (no crash)."""
import os
import struct

import numpy as np
import pytest

import ferrite_b200 as fb
from conftest import O, tiny_config, tiny_weights
from gguf_writer import model_tensors, write_gguf


@pytest.mark.parametrize("arch", ["qwen3", "llama"])
def test_config_from_metadata(tmp_path, arch):
    cfg = tiny_config(max_ctx=777, rope_theta=5e5, eps=1e-5)
    w = tiny_weights(cfg, seed=3)
    p = os.path.join(tmp_path, "m.gguf")
    write_gguf(p, arch, cfg, model_tensors(w))
    got = fb.gguf_config(p)
    for k in ("n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab", "max_ctx"):
        assert got[k] == cfg[k], k
    assert got["max_batch"] == 1
    assert got["rope_theta"] == np.float32(5e5) and got["eps"] == np.float32(1e-5)
    assert got["arch"] == arch
    assert (got["qk_norm"], got["rope_mode"]) == ((1, 1) if arch == "qwen3" else (0, 0))


def test_version2_and_alignment(tmp_path):
    cfg = tiny_config()
    p = os.path.join(tmp_path, "v2.gguf")
    write_gguf(p, "llama", cfg, model_tensors(tiny_weights(cfg, seed=4)), align=64, version=2)
    assert fb.gguf_config(p)["hidden"] == cfg["hidden"]


def test_rejects_bad_files(tmp_path):
    cfg = tiny_config()
    good = os.path.join(tmp_path, "good.gguf")
    write_gguf(good, "qwen3", cfg, model_tensors(tiny_weights(cfg, seed=5)))
    raw = open(good, "rb").read()
    cases = {
        "bad magic": b"GGUX" + raw[4:],
        "bad version": raw[:4] + struct.pack("<I", 7) + raw[8:],
        "truncated": raw[:200],
    }
    for what, data in cases.items():
        p = os.path.join(tmp_path, what.replace(" ", "_") + ".gguf")
        open(p, "wb").write(data)
        with pytest.raises(fb.FerriteError):
            fb.gguf_config(p)
    p = os.path.join(tmp_path, "arch.gguf")
    write_gguf(p, "mamba", cfg, model_tensors(tiny_weights(cfg, seed=5)))
    with pytest.raises(fb.FerriteError, match="not supported"):
        fb.gguf_config(p)
    with pytest.raises(fb.FerriteError, match="cannot open"):
        fb.gguf_config(os.path.join(tmp_path, "missing.gguf"))
