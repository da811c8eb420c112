"""ctypes view of the CPU oracle (oracle/liboracle.so).

Test infrastructure only: tests/, the smoke check and the CPU-baseline leg of
bench.py use it as the checker.  The product path never imports this module.
The C sources cite the reference lines they restate (oracle.h).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, F16, Q4_K, Q6_K, Q8_K = 0, 1, 12, 14, 15
QK_K = 256
BLOCK_BYTES = {Q4_K: 144, Q6_K: 210, Q8_K: 292}

_lib = None


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


class Config(C.Structure):
    _fields_ = [(n, C.c_int) for n in
                ("n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab", "max_ctx")] + [
        ("rope_theta", C.c_float), ("eps", C.c_float),
        ("qk_norm", C.c_int), ("rope_mode", C.c_int), ("kv_f16", C.c_int)]


class Tensor(C.Structure):
    _fields_ = [("dtype", C.c_int), ("rows", C.c_int64), ("cols", C.c_int64), ("data", C.c_void_p)]


class Layer(C.Structure):
    _fields_ = [(n, Tensor) for n in ("attn_norm", "wq", "wk", "wv", "wo", "q_norm", "k_norm",
                                      "ffn_norm", "w_gate", "w_up", "w_down")]


def _declare(L):
    vp, i64, i32, f32 = C.c_void_p, C.c_int64, C.c_int32, C.c_float
    u64 = C.c_uint64
    L.or_quantize_q4k.argtypes = [vp, i64, vp]
    L.or_quantize_q6k.argtypes = [vp, i64, vp]
    L.or_quantize_q8k.argtypes = [vp, i64, vp, C.c_int]
    L.or_dequantize.argtypes = [C.c_int, vp, i64, vp]
    L.or_dequant_parts.argtypes = [C.c_int, vp, i64, vp, vp, vp]
    L.or_vec_dot.argtypes = [C.c_int, i64, vp, vp]
    L.or_vec_dot.restype = f32
    L.or_block_dots.argtypes = [C.c_int, i64, i64, vp, vp, vp, vp]
    L.or_qmatmul.argtypes = [C.c_int, vp, i64, i64, vp, i64, vp, C.c_int]
    L.or_qmatmul_f32.argtypes = [C.c_int, vp, i64, i64, vp, i64, vp, C.c_int]
    L.or_qmatmul64.argtypes = [C.c_int, vp, i64, i64, vp, i64, vp, C.c_int]
    L.or_f16_to_f32.argtypes = [C.c_uint16]
    L.or_f16_to_f32.restype = f32
    L.or_f32_to_f16.argtypes = [f32]
    L.or_f32_to_f16.restype = C.c_uint16
    L.or_rmsnorm.argtypes = [vp, vp, vp, i64, i64, f32]
    L.or_rope.argtypes = [vp, i64, i64, i64, f32, C.c_int]
    L.or_softmax.argtypes = [vp, i64]
    L.or_silu.argtypes = [f32]
    L.or_silu.restype = f32
    L.or_exp64.argtypes = [C.c_double]
    L.or_exp64.restype = C.c_double
    L.or_synth_q4k.argtypes = [u64, i64, f32, vp]
    L.or_synth_q6k.argtypes = [u64, i64, f32, vp]
    L.or_synth_f32.argtypes = [u64, i64, f32, f32, vp]
    L.or_synth_tokens.argtypes = [u64, i64, i32, vp]
    L.or_model_create.argtypes = [C.POINTER(Config), C.POINTER(Tensor), C.POINTER(Layer),
                                  C.POINTER(Tensor), C.POINTER(Tensor), C.c_int]
    L.or_model_create.restype = vp
    L.or_model_free.argtypes = [vp]
    L.or_model_clear.argtypes = [vp]
    L.or_model_forward.argtypes = [vp, vp, C.c_int, C.c_int, vp, C.c_int, C.c_int]
    L.or_model_forward.restype = C.c_int
    L.or_model_synth_kv.argtypes = [vp, u64, C.c_int, f32]
    L.or_model_synth_kv.restype = C.c_int
    L.or_model_read_kv.argtypes = [vp, C.c_int, C.c_int, C.c_int, vp]
    L.or_model_read_kv.restype = C.c_int
    L.or_model_length.argtypes = [vp]
    L.or_model_length.restype = C.c_int


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- formats --
def f16_to_f32(bits: int) -> float:
    return lib().or_f16_to_f32(bits)


def f32_to_f16(x: float) -> int:
    return lib().or_f32_to_f16(x)


def quantize(dtype: int, x: np.ndarray) -> np.ndarray:
    """f32 [.., k] -> raw GGUF blocks (uint8, [.., k/256*block_bytes])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    assert n % QK_K == 0
    out = np.zeros(n // QK_K * BLOCK_BYTES[dtype], dtype=np.uint8)
    if dtype == Q4_K:
        lib().or_quantize_q4k(_p(x), n, _p(out))
    elif dtype == Q6_K:
        lib().or_quantize_q6k(_p(x), n, _p(out))
    else:
        raise ValueError(dtype)
    return out.reshape(x.shape[:-1] + (x.shape[-1] // QK_K * BLOCK_BYTES[dtype],))


def quantize_q8k(x: np.ndarray, round_mode: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // QK_K * 292, dtype=np.uint8)
    lib().or_quantize_q8k(_p(x), x.size, _p(out), round_mode)
    return out.reshape(x.shape[:-1] + (x.shape[-1] // QK_K * 292,))


def dequantize(dtype: int, blocks: np.ndarray, n: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks)
    y = np.zeros(n, dtype=np.float32)
    lib().or_dequantize(dtype, _p(blocks), n, _p(y))
    return y


def dequant_parts(dtype: int, blocks: np.ndarray, n: int):
    """Per-weight (scale, offset, integer code) with w = scale * q - offset."""
    blocks = np.ascontiguousarray(blocks)
    sc = np.zeros(n, dtype=np.float32)
    off = np.zeros(n, dtype=np.float32)
    q = np.zeros(n, dtype=np.int8)
    lib().or_dequant_parts(dtype, _p(blocks), n, _p(sc), _p(off), _p(q))
    return sc, off, q


def vec_dot(dtype: int, k: int, w_row: np.ndarray, a_q8k: np.ndarray) -> float:
    return lib().or_vec_dot(dtype, k, _p(np.ascontiguousarray(w_row)), _p(np.ascontiguousarray(a_q8k)))


def block_dots(dtype: int, w: np.ndarray, nrows: int, k: int, a_q8k: np.ndarray):
    nb = k // QK_K
    sc = np.zeros((nrows, nb), dtype=np.int32)
    mn = np.zeros((nrows, nb), dtype=np.int32)
    lib().or_block_dots(dtype, nrows, k, _p(np.ascontiguousarray(w)), _p(np.ascontiguousarray(a_q8k)),
                        _p(sc), _p(mn))
    return sc, mn


def qmatmul(dtype: int, w: np.ndarray, n: int, k: int, x: np.ndarray, nthreads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    y = np.zeros((x.shape[0], n), dtype=np.float32)
    lib().or_qmatmul(dtype, _p(np.ascontiguousarray(w)), n, k, _p(x), x.shape[0], _p(y), nthreads)
    return y


def qmatmul64(dtype: int, w: np.ndarray, n: int, k: int, x: np.ndarray, nthreads: int = 0) -> np.ndarray:
    """qmatmul's binary64 row sums before the final rounding to f32."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    y = np.zeros((x.shape[0], n), dtype=np.float64)
    lib().or_qmatmul64(dtype, _p(np.ascontiguousarray(w)), n, k, _p(x), x.shape[0], _p(y), nthreads)
    return y


def shard_blocks(dtype: int, w: np.ndarray, n: int, k: int, row0: int, rows: int, col0: int, cols: int) -> np.ndarray:
    """GGUF blocks of W[row0:row0+rows, col0:col0+cols] (col0, cols multiples
    of 256): the tensor-parallel shard a rank keeps."""
    bb = {Q4_K: 144, Q6_K: 210}[dtype]
    rowsv = np.asarray(w, dtype=np.uint8).reshape(n, k // 256 * bb)
    return np.ascontiguousarray(rowsv[row0:row0 + rows, col0 // 256 * bb:(col0 + cols) // 256 * bb]).reshape(-1)


def qmatmul_f32(dtype: int, w: np.ndarray, n: int, k: int, x: np.ndarray, nthreads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    y = np.zeros((x.shape[0], n), dtype=np.float32)
    lib().or_qmatmul_f32(dtype, _p(np.ascontiguousarray(w)), n, k, _p(x), x.shape[0], _p(y), nthreads)
    return y


def silu(x: np.ndarray) -> np.ndarray:
    f = lib().or_silu
    return np.array([f(float(v)) for v in np.asarray(x, dtype=np.float32).reshape(-1)],
                    dtype=np.float32).reshape(np.shape(x))


def rmsnorm(x: np.ndarray, g: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    g = np.ascontiguousarray(g, dtype=np.float32)
    y = np.zeros_like(x)
    lib().or_rmsnorm(_p(x), _p(g), _p(y), x.size // x.shape[-1], x.shape[-1], eps)
    return y


def synth_q4k(seed: int, nblocks: int, sigma: float = 0.02) -> np.ndarray:
    out = np.zeros(nblocks * 144, dtype=np.uint8)
    lib().or_synth_q4k(seed, nblocks, sigma, _p(out))
    return out


def synth_q6k(seed: int, nblocks: int, sigma: float = 0.02) -> np.ndarray:
    out = np.zeros(nblocks * 210, dtype=np.uint8)
    lib().or_synth_q6k(seed, nblocks, sigma, _p(out))
    return out


def synth_f32(seed: int, n: int, mean: float, std: float) -> np.ndarray:
    out = np.zeros(n, dtype=np.float32)
    lib().or_synth_f32(seed, n, mean, std, _p(out))
    return out


def synth_tokens(seed: int, n: int, vocab: int) -> np.ndarray:
    out = np.zeros(n, dtype=np.int32)
    lib().or_synth_tokens(seed, n, vocab, _p(out))
    return out


# Per-tensor seeds of a random-init model: the convention the product's
# fb_model_synth uses (seed + 0x1000 * (layer + 1) + kind id, layer = -1 for
# global tensors).
KIND_ID = {"token_embd": 1, "output_norm": 2, "output": 3, "attn_norm": 10, "attn_q": 11, "attn_k": 12,
           "attn_v": 13, "attn_output": 14, "attn_q_norm": 15, "attn_k_norm": 16, "ffn_norm": 17, "ffn_gate": 18,
           "ffn_up": 19, "ffn_down": 20}


def tensor_seed(seed: int, layer: int, name: str) -> int:
    return (seed + 0x1000 * (layer + 1) + KIND_ID[name]) & 0xFFFFFFFFFFFFFFFF


def synth_model_weights(cfg: dict, seed: int) -> dict:
    """Oracle-side copy of the random-init model (Q4_K linear layers, Q6_K
    ffn_down and output, f32 norms), generated with the restated generator."""
    H, F, V = cfg["hidden"], cfg["ffn"], cfg["vocab"]
    qd, kd = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]

    def q4(n, k, s):
        return (Q4_K, n, k, synth_q4k(s, n * k // 256, 0.02))

    def q6(n, k, s):
        return (Q6_K, n, k, synth_q6k(s, n * k // 256, 0.02))

    def v(n, s):
        return (F32, 1, n, synth_f32(s, n, 1.0, 0.02))

    layers = []
    for l in range(cfg["n_layers"]):
        def ts(name, l=l):
            return tensor_seed(seed, l, name)
        layers.append(dict(
            attn_norm=v(H, ts("attn_norm")), wq=q4(qd, H, ts("attn_q")), wk=q4(kd, H, ts("attn_k")),
            wv=q4(kd, H, ts("attn_v")), wo=q4(H, qd, ts("attn_output")), q_norm=v(cfg["head_dim"], ts("attn_q_norm")),
            k_norm=v(cfg["head_dim"], ts("attn_k_norm")), ffn_norm=v(H, ts("ffn_norm")),
            w_gate=q4(F, H, ts("ffn_gate")), w_up=q4(F, H, ts("ffn_up")), w_down=q6(H, F, ts("ffn_down"))))
    return dict(tok_embd=q4(V, H, tensor_seed(seed, -1, "token_embd")),
                out_norm=v(H, tensor_seed(seed, -1, "output_norm")),
                output=q6(V, H, tensor_seed(seed, -1, "output")), layers=layers)


# ------------------------------------------------------------------ model --
class Model:
    """Oracle quantized Llama/Qwen3 model over caller-supplied weight arrays.

    weights: dict with 'tok_embd', 'out_norm', 'output' and 'layers' (list of
    dicts with attn_norm, wq, wk, wv, wo, q_norm, k_norm, ffn_norm, w_gate,
    w_up, w_down); each entry is (dtype, rows, cols, ndarray)."""

    def __init__(self, cfg: dict, weights: dict, nthreads: int = 0):
        self.cfg = dict(cfg)
        self._keep = []
        c = Config(**{k: cfg[k] for k, _ in Config._fields_})
        self._c = c
        layers = (Layer * cfg["n_layers"])()
        for i, lw in enumerate(weights["layers"]):
            for name, _ in Layer._fields_:
                setattr(layers[i], name, self._t(lw[name]))
        te, on, out = self._t(weights["tok_embd"]), self._t(weights["out_norm"]), self._t(weights["output"])
        self._h = lib().or_model_create(C.byref(c), C.byref(te), layers, C.byref(on), C.byref(out), nthreads)
        if not self._h:
            raise MemoryError("or_model_create failed")

    def _t(self, spec):
        dtype, rows, cols, arr = spec
        arr = np.ascontiguousarray(arr)
        self._keep.append(arr)
        return Tensor(dtype, rows, cols, arr.ctypes.data)

    def forward(self, tokens, pos: int, all_logits: bool = False, matmul_mode: int = 0) -> np.ndarray:
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        n = toks.size
        V = self.cfg["vocab"]
        out = np.zeros((n if all_logits else 1, V), dtype=np.float32)
        rc = lib().or_model_forward(self._h, _p(toks), n, pos, _p(out), int(all_logits), matmul_mode)
        if rc:
            raise RuntimeError(f"or_model_forward failed ({rc})")
        return out if all_logits else out[0]

    def synth_kv(self, seed: int, ctx: int, scale: float = 0.5):
        if lib().or_model_synth_kv(self._h, seed, ctx, scale):
            raise ValueError("bad ctx")

    def read_kv(self, layer: int, which: int, pos: int) -> np.ndarray:
        out = np.zeros(self.cfg["n_kv_heads"] * self.cfg["head_dim"], dtype=np.float32)
        if lib().or_model_read_kv(self._h, layer, which, pos, _p(out)):
            raise ValueError("bad kv index")
        return out

    def clear(self):
        lib().or_model_clear(self._h)

    @property
    def length(self) -> int:
        return lib().or_model_length(self._h)

    def close(self):
        if self._h:
            lib().or_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
