"""Minimal GGUF v3 writer for the ingest tests (the published file layout:
magic, version, counts, typed metadata, tensor infos with innermost-first
dims, data section aligned to general.alignment)."""
from __future__ import annotations

import struct

import numpy as np

from conftest import GGUF_NAMES

U32, F32, STRING, ARRAY = 4, 6, 8, 9


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, value) -> bytes:
    out = _str(key) + struct.pack("<I", vtype)
    if vtype == STRING:
        out += _str(value)
    elif vtype == U32:
        out += struct.pack("<I", value)
    elif vtype == F32:
        out += struct.pack("<f", value)
    elif vtype == ARRAY:
        etype, items = value
        out += struct.pack("<IQ", etype, len(items))
        for it in items:
            out += _str(it) if etype == STRING else struct.pack("<f" if etype == F32 else "<I", it)
    else:
        raise ValueError(vtype)
    return out


def write_gguf(path: str, arch: str, cfg: dict, tensors: list, align: int = 32, extra_kv: bytes = b"",
               version: int = 3) -> None:
    """tensors: (name, ggml_type, rows, cols, data array) -- dims are written
    innermost first (cols, rows), 1-D tensors as (cols,)."""
    kv = [
        _kv("general.architecture", STRING, arch),
        _kv("general.alignment", U32, align),
        _kv(f"{arch}.block_count", U32, cfg["n_layers"]),
        _kv(f"{arch}.embedding_length", U32, cfg["hidden"]),
        _kv(f"{arch}.feed_forward_length", U32, cfg["ffn"]),
        _kv(f"{arch}.attention.head_count", U32, cfg["n_heads"]),
        _kv(f"{arch}.attention.head_count_kv", U32, cfg["n_kv_heads"]),
        _kv(f"{arch}.attention.key_length", U32, cfg["head_dim"]),
        _kv(f"{arch}.rope.freq_base", F32, cfg["rope_theta"]),
        _kv(f"{arch}.attention.layer_norm_rms_epsilon", F32, cfg["eps"]),
        _kv(f"{arch}.context_length", U32, cfg["max_ctx"]),
        _kv("tokenizer.ggml.tokens", ARRAY, (STRING, [f"t{i}" for i in range(16)])),
        _kv("tokenizer.ggml.scores", ARRAY, (F32, [0.5] * 16)),
    ]
    infos, blobs, off = [], [], 0
    for name, gtype, rows, cols, data in tensors:
        raw = np.ascontiguousarray(data).tobytes()
        dims = [cols] if rows == 1 else [cols, rows]
        infos.append(_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) +
                     struct.pack("<IQ", gtype, off))
        pad = (-len(raw)) % align
        blobs.append(raw + b"\0" * pad)
        off += len(raw) + pad
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kv) + (1 if extra_kv else 0))
    body = head + b"".join(kv) + extra_kv + b"".join(infos)
    body += b"\0" * ((-len(body)) % align)
    with open(path, "wb") as f:
        f.write(body + b"".join(blobs))


def model_tensors(weights: dict, tied: bool = False) -> list:
    """GGUF tensor list of an oracle-style weight dict (conftest.tiny_weights)."""
    out = []

    def add(name, spec):
        dt, r, c, a = spec
        out.append((name + ".weight", dt, r, c, a))

    add("token_embd", weights["tok_embd"])
    add("output_norm", weights["out_norm"])
    if not tied:
        add("output", weights["output"])
    for li, lw in enumerate(weights["layers"]):
        for key, name in GGUF_NAMES.items():
            add(f"blk.{li}.{name}", lw[key])
    return out
