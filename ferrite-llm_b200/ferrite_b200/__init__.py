"""Python view of libferrite_b200.so (the sm_100a quantized decode path).

Mirrors the reference's operator surface for this path:
  QTensor / QMatMul      candle-core 0.8.4 quantized API as used by
                         quantized_llama (crates/ferrite-wasm-host/src/adapter.rs:41-70)
  Model.forward/prefill/clear_cache
                         ferrite_core::InferenceModel
                         (crates/ferrite-core/src/generation.rs:187-195)
  Model.decode_greedy    Sampler::argmax greedy path
                         (crates/ferrite-core/src/sampling.rs:108-112)

Device buffers are passed as integer device pointers (e.g. torch's
``tensor.data_ptr()``); host buffers as numpy arrays.  Every call goes through
the C ABI declared in include/ferrite_b200.h and raises FerriteError on a
non-zero status.  There is no CPU fallback: importing this module on a machine
without the built library raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "libferrite_b200.so")

F32, F16, Q4_K, Q6_K, Q8_K, BF16 = 0, 1, 12, 14, 15, 30
BLOCK_BYTES = {Q4_K: 144, Q6_K: 210, Q8_K: 292}

# Every symbol include/ferrite_b200.h declares (checked by the CPU tests).
EXPORTED = (
    "fb_last_error", "fb_abi_version", "fb_ctx_create", "fb_ctx_destroy", "fb_ctx_set_stream", "fb_ctx_stream",
    "fb_sync", "fb_ctx_error_word", "fb_ctx_set_pdl", "fb_ctx_set_prefill_weight_cache", "fb_qtensor_upload", "fb_qtensor_upload_dev",
    "fb_qtensor_synth", "fb_qtensor_concat_rows", "fb_qtensor_info", "fb_qtensor_download", "fb_qtensor_destroy",
    "fb_dequantize", "fb_qmatmul", "fb_qmatmul_q8k", "fb_quantize_q8k", "fb_block_dots", "fb_rmsnorm", "fb_rope",
    "fb_swiglu", "fb_attn_decode", "fb_model_create", "fb_model_destroy", "fb_model_set_tensor", "fb_model_synth",
    "fb_model_finalize", "fb_model_forward", "fb_model_decode_greedy", "fb_model_decode_dev", "fb_model_prefill",
    "fb_model_clear_cache", "fb_model_synth_kv", "fb_model_read_kv", "fb_model_weight_bytes",
    "fb_model_read_activation", "fb_model_profile", "fb_model_launches_per_step", "fb_attn_decode_noalloc",
    "fb_qtensor_upload_slice", "fb_comm_create", "fb_comm_handle", "fb_comm_open", "fb_comm_destroy",
    "fb_model_create_tp", "fb_model_tp_info", "fb_comm_set_timeout_ms", "fb_attn_prefill", "fb_gguf_config",
    "fb_model_load_gguf", "fb_model_forward_all", "fb_sample", "fb_top_logits", "fb_model_set_persistent",
    "fb_model_step_timeline",
)
COMM_HANDLE_BYTES = 64

PROF_KINDS = ("embed_norm", "qkv", "rope_kv", "attn", "o", "norm", "gate_up", "swiglu", "down", "lm_head", "argmax")


class FerriteError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class SamplerConfig(C.Structure):
    _fields_ = [("temperature", C.c_double), ("top_p", C.c_double), ("top_k", C.c_int), ("min_p", C.c_float),
                ("repetition_penalty", C.c_float)]


class ModelConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in
                ("n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab", "max_ctx", "max_batch")] + [
        ("rope_theta", C.c_float), ("eps", C.c_float), ("qk_norm", C.c_int), ("rope_mode", C.c_int)]


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run ferrite-llm_b200/build.py")
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(L):
    vp, i64, i32, f32, u64 = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_uint64
    P = C.POINTER
    sig = {
        "fb_last_error": (C.c_char_p, []),
        "fb_abi_version": (i32, []),
        "fb_ctx_create": (i32, [i32, vp, P(vp)]),
        "fb_ctx_destroy": (i32, [vp]),
        "fb_ctx_set_stream": (i32, [vp, vp]),
        "fb_ctx_stream": (vp, [vp]),
        "fb_sync": (i32, [vp]),
        "fb_ctx_error_word": (i32, [vp, P(C.c_uint32)]),
        "fb_ctx_set_pdl": (i32, [vp, i32]),
        "fb_ctx_set_prefill_weight_cache": (i32, [vp, i32]),
        "fb_qtensor_upload": (i32, [vp, i32, i64, i64, vp, P(vp)]),
        "fb_qtensor_upload_dev": (i32, [vp, i32, i64, i64, vp, P(vp)]),
        "fb_qtensor_synth": (i32, [vp, i32, i64, i64, u64, f32, P(vp)]),
        "fb_qtensor_concat_rows": (i32, [vp, P(vp), i32, P(vp)]),
        "fb_qtensor_info": (i32, [vp, P(i32), P(i64), P(i64), P(i64)]),
        "fb_qtensor_download": (i32, [vp, vp, vp]),
        "fb_qtensor_destroy": (i32, [vp]),
        "fb_dequantize": (i32, [vp, vp, vp, i32]),
        "fb_qmatmul": (i32, [vp, vp, vp, vp, i64]),
        "fb_qmatmul_q8k": (i32, [vp, vp, vp, vp, i64]),
        "fb_quantize_q8k": (i32, [vp, vp, i64, i64, vp]),
        "fb_block_dots": (i32, [vp, vp, vp, vp, vp]),
        "fb_rmsnorm": (i32, [vp, vp, vp, vp, i64, i64, f32]),
        "fb_rope": (i32, [vp, vp, i64, i64, i64, i64, f32, i32]),
        "fb_swiglu": (i32, [vp, vp, vp, vp, i64, i64]),
        "fb_attn_decode": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, i32, f32]),
        "fb_attn_decode_noalloc": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, i32, f32]),
        "fb_model_create": (i32, [vp, P(ModelConfig), P(vp)]),
        "fb_model_destroy": (i32, [vp]),
        "fb_model_set_tensor": (i32, [vp, C.c_char_p, i32, i32, i64, i64, vp]),
        "fb_model_synth": (i32, [vp, u64]),
        "fb_model_finalize": (i32, [vp]),
        "fb_model_forward": (i32, [vp, vp, i32, i32, vp]),
        "fb_model_decode_greedy": (i32, [vp, vp, vp, i32, vp]),
        "fb_model_decode_dev": (i32, [vp, vp, vp, i32, vp, vp]),
        "fb_model_prefill": (i32, [vp, vp, i32, vp]),
        "fb_model_clear_cache": (i32, [vp]),
        "fb_model_synth_kv": (i32, [vp, u64, i32, f32]),
        "fb_model_read_kv": (i32, [vp, i32, i32, i32, vp]),
        "fb_model_weight_bytes": (i32, [vp, P(i64)]),
        "fb_model_read_activation": (i32, [vp, C.c_char_p, i32, vp, i64]),
        "fb_model_profile": (i32, [vp, vp, vp, i32, i32, vp, vp]),
        "fb_model_launches_per_step": (i32, [vp, P(i32)]),
        "fb_qtensor_upload_slice": (i32, [vp, i32, i64, i64, vp, i32, i64, i64, i64, i64, P(vp)]),
        "fb_comm_create": (i32, [vp, i32, i32, i32, i32, P(vp)]),
        "fb_comm_handle": (i32, [vp, vp]),
        "fb_comm_open": (i32, [vp, vp]),
        "fb_comm_destroy": (i32, [vp]),
        "fb_comm_set_timeout_ms": (i32, [vp, i32]),
        "fb_attn_prefill": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, i32, f32, vp]),
        "fb_gguf_config": (i32, [C.c_char_p, P(ModelConfig), P(i32)]),
        "fb_model_load_gguf": (i32, [vp, C.c_char_p]),
        "fb_model_forward_all": (i32, [vp, vp, i32, i32, vp]),
        "fb_sample": (i32, [vp, vp, i32, P(SamplerConfig), vp, i32, P(C.c_uint64), P(i32)]),
        "fb_top_logits": (i32, [vp, vp, i32, i64, i32, vp, vp]),
        "fb_model_set_persistent": (i32, [vp, i32, P(i32)]),
        "fb_model_step_timeline": (i32, [vp, vp, vp, vp, i64, P(i32), P(i32)]),
        "fb_model_create_tp": (i32, [vp, P(ModelConfig), vp, P(vp)]),
        "fb_model_tp_info": (i32, [vp, P(i32), P(i32), P(i32), P(i32)]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args


def _check(rc: int):
    if rc != 0:
        raise FerriteError(rc, lib().fb_last_error().decode(errors="replace"))


def _np(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


class Context:
    """fb_ctx: device + stream (defaults to torch's current stream when given)."""

    def __init__(self, device: int = 0, stream: int | None = None):
        h = C.c_void_p()
        _check(lib().fb_ctx_create(device, stream, C.byref(h)))
        self.h = h
        self.device = device

    def sync(self):
        _check(lib().fb_sync(self.h))

    def set_pdl(self, enable: bool):
        _check(lib().fb_ctx_set_pdl(self.h, int(enable)))

    def set_prefill_weight_cache(self, enable: bool):
        """Keep fp16 copies of the projection weights for long prompt passes
        (the default) or dequantize them on every pass."""
        _check(lib().fb_ctx_set_prefill_weight_cache(self.h, int(enable)))

    def error_word(self) -> int:
        v = C.c_uint32()
        _check(lib().fb_ctx_error_word(self.h, C.byref(v)))
        return v.value

    @property
    def stream(self) -> int:
        return lib().fb_ctx_stream(self.h) or 0

    def set_stream(self, stream: int):
        """Order later work on `stream` (the old stream is synchronised first)."""
        _check(lib().fb_ctx_set_stream(self.h, stream or None))

    def close(self):
        if self.h:
            lib().fb_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class QTensor:
    """Device-resident k-quant weight W[n, k] (candle QTensor counterpart)."""

    def __init__(self, ctx: Context, handle: C.c_void_p):
        self.ctx, self.h = ctx, handle
        dt, n, k, nbytes = C.c_int(), C.c_int64(), C.c_int64(), C.c_int64()
        _check(lib().fb_qtensor_info(handle, C.byref(dt), C.byref(n), C.byref(k), C.byref(nbytes)))
        self.dtype, self.n, self.k, self.device_bytes = dt.value, n.value, k.value, nbytes.value

    @classmethod
    def upload(cls, ctx: Context, dtype: int, n: int, k: int, blocks: np.ndarray) -> "QTensor":
        blocks = np.ascontiguousarray(blocks)
        h = C.c_void_p()
        _check(lib().fb_qtensor_upload(ctx.h, dtype, n, k, _np(blocks), C.byref(h)))
        return cls(ctx, h)

    @classmethod
    def upload_slice(cls, ctx: Context, dtype: int, n: int, k: int, blocks: np.ndarray, row0: int, rows: int,
                     col0: int, cols: int) -> "QTensor":
        """W[row0:row0+rows, col0:col0+cols] of the full GGUF tensor W[n, k]
        (host blocks); cols and col0 are multiples of 256."""
        blocks = np.ascontiguousarray(blocks)
        h = C.c_void_p()
        _check(lib().fb_qtensor_upload_slice(ctx.h, dtype, n, k, _np(blocks), 0, row0, rows, col0, cols,
                                             C.byref(h)))
        return cls(ctx, h)

    @classmethod
    def synth(cls, ctx: Context, dtype: int, n: int, k: int, seed: int, sigma: float = 0.02) -> "QTensor":
        h = C.c_void_p()
        _check(lib().fb_qtensor_synth(ctx.h, dtype, n, k, seed, sigma, C.byref(h)))
        return cls(ctx, h)

    @classmethod
    def concat_rows(cls, ctx: Context, parts: list["QTensor"]) -> "QTensor":
        arr = (C.c_void_p * len(parts))(*[p.h for p in parts])
        h = C.c_void_p()
        _check(lib().fb_qtensor_concat_rows(ctx.h, arr, len(parts), C.byref(h)))
        return cls(ctx, h)

    def download(self) -> np.ndarray:
        nbytes = self.n * self.k // 256 * BLOCK_BYTES[self.dtype] if self.dtype != F32 else self.n * self.k * 4
        out = np.zeros(nbytes, dtype=np.uint8)
        _check(lib().fb_qtensor_download(self.ctx.h, self.h, _np(out)))
        return out

    def dequantize(self, out_ptr: int, out_dtype: int = F32):
        _check(lib().fb_dequantize(self.ctx.h, self.h, out_ptr, out_dtype))

    def close(self):
        if self.h:
            lib().fb_qtensor_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class QMatMul:
    """y[m, n] = x[m, k] . W^T for a device QTensor (candle QMatMul::forward)."""

    def __init__(self, w: QTensor):
        self.w = w

    def forward(self, x_ptr: int, y_ptr: int, m: int):
        _check(lib().fb_qmatmul(self.w.ctx.h, self.w.h, x_ptr, y_ptr, m))

    def forward_q8k(self, x_ptr: int, y_ptr: int, m: int):
        _check(lib().fb_qmatmul_q8k(self.w.ctx.h, self.w.h, x_ptr, y_ptr, m))


def quantize_q8k(ctx: Context, x_ptr: int, m: int, k: int, out_ptr: int):
    _check(lib().fb_quantize_q8k(ctx.h, x_ptr, m, k, out_ptr))


def block_dots(ctx: Context, w: QTensor, x_ptr: int, sc_ptr: int, mn_ptr: int):
    _check(lib().fb_block_dots(ctx.h, w.h, x_ptr, sc_ptr, mn_ptr))


def rmsnorm(ctx: Context, x_ptr, g_ptr, y_ptr, rows, dim, eps):
    _check(lib().fb_rmsnorm(ctx.h, x_ptr, g_ptr, y_ptr, rows, dim, eps))


def rope(ctx: Context, x_ptr, n_tok, n_heads, head_dim, pos0, theta, mode):
    _check(lib().fb_rope(ctx.h, x_ptr, n_tok, n_heads, head_dim, pos0, theta, mode))


def swiglu(ctx: Context, g_ptr, u_ptr, o_ptr, m, f):
    _check(lib().fb_swiglu(ctx.h, g_ptr, u_ptr, o_ptr, m, f))


def attn_decode(ctx: Context, q_ptr, k_ptr, v_ptr, bt_ptr, lens_ptr, out_ptr, batch, n_heads, n_kv, head_dim,
                page_size, max_pages, num_pages, max_seq_len, scale):
    """num_pages: pages the K / V pools hold; block-table ids outside
    [0, num_pages) are skipped and set the error word's bad-page bit."""
    _check(lib().fb_attn_decode(ctx.h, q_ptr, k_ptr, v_ptr, bt_ptr, lens_ptr, out_ptr, batch, n_heads, n_kv,
                                head_dim, page_size, max_pages, num_pages, max_seq_len, scale))


def attn_prefill(ctx: Context, q_ptr, k_ptr, v_ptr, bt_ptr, max_pages, num_pages, pos0, n_tokens, n_heads, n_kv,
                 head_dim, page_size, scale, out_ptr):
    _check(lib().fb_attn_prefill(ctx.h, q_ptr, k_ptr, v_ptr, bt_ptr, max_pages, num_pages, pos0, n_tokens, n_heads,
                                 n_kv, head_dim, page_size, scale, out_ptr))


def attn_decode_noalloc(ctx: Context, q_ptr, k_ptr, v_ptr, bt_ptr, lens_ptr, out_ptr, batch, n_heads, n_kv,
                        head_dim, page_size, max_pages, num_pages, max_seq_len, scale):
    """fb_attn_decode without any device allocation (fixed 4 MiB scratch in
    the library's device image; see include/ferrite_b200.h)."""
    _check(lib().fb_attn_decode_noalloc(ctx.h, q_ptr, k_ptr, v_ptr, bt_ptr, lens_ptr, out_ptr, batch, n_heads, n_kv,
                                        head_dim, page_size, max_pages, num_pages, max_seq_len, scale))


# GGUF tensor names of one layer / of the whole model.
LAYER_TENSORS = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "attn_q_norm", "attn_k_norm",
                 "ffn_norm", "ffn_gate", "ffn_up", "ffn_down")
KIND_ID = {"token_embd": 1, "output_norm": 2, "output": 3, "attn_norm": 10, "attn_q": 11, "attn_k": 12,
           "attn_v": 13, "attn_output": 14, "attn_q_norm": 15, "attn_k_norm": 16, "ffn_norm": 17, "ffn_gate": 18,
           "ffn_up": 19, "ffn_down": 20}


def tensor_seed(seed: int, layer: int, name: str) -> int:
    """Per-tensor seed used by Model.synth (layer = -1 for global tensors)."""
    return (seed + 0x1000 * (layer + 1) + KIND_ID[name]) & 0xFFFFFFFFFFFFFFFF


class Sampler:
    """Sampler::sample of the reference on the device (fb_sample); the RNG
    state advances like the reference's xorshift64."""

    def __init__(self, ctx: Context, temperature=0.7, top_p=0.9, top_k=0, min_p=0.05, repetition_penalty=1.1,
                 seed=42):
        self.ctx = ctx
        self.cfg = SamplerConfig(temperature, top_p, top_k, min_p, repetition_penalty)
        self.state = C.c_uint64(seed)

    def sample(self, logits_ptr: int, vocab: int, previous_tokens=()) -> int:
        prev = np.ascontiguousarray(np.asarray(previous_tokens, dtype=np.int32))
        out = C.c_int32()
        _check(lib().fb_sample(self.ctx.h, logits_ptr, vocab, C.byref(self.cfg), _np(prev) if prev.size else None,
                               prev.size, C.byref(self.state), C.byref(out)))
        return out.value


def top_logits(ctx: Context, logits_ptr: int, rows: int, vocab: int, k: int, ids_ptr: int, vals_ptr: int):
    """The k (1..16) largest logits of each row, ordered like the reference
    hook's stable descending sort: ids [rows][k] int32, vals [rows][k] f32 on
    the device (fb_top_logits)."""
    _check(lib().fb_top_logits(ctx.h, logits_ptr, rows, vocab, k, ids_ptr, vals_ptr))


def gguf_config(path: str) -> dict:
    """Model config from a GGUF file's metadata (plus 'arch': llama / qwen3)."""
    c = ModelConfig()
    arch = C.c_int()
    _check(lib().fb_gguf_config(os.fsencode(path), C.byref(c), C.byref(arch)))
    d = {k: getattr(c, k) for k, _ in ModelConfig._fields_}
    d["arch"] = "qwen3" if arch.value == 1 else "llama"
    return d


class Comm:
    """Tensor-parallel exchange region of one rank (fb_comm).

    create -> handle() on every rank -> exchange the handles -> open(all).
    ``Comm.connect`` does the exchange over an initialised torch.distributed
    process group (any backend; the handles are 64-byte host blobs)."""

    def __init__(self, ctx: Context, rank: int, world: int, max_batch: int, hidden: int):
        self.ctx, self.rank, self.world = ctx, rank, world
        h = C.c_void_p()
        _check(lib().fb_comm_create(ctx.h, rank, world, max_batch, hidden, C.byref(h)))
        self.h = h

    def set_timeout_ms(self, ms: int):
        _check(lib().fb_comm_set_timeout_ms(self.h, ms))

    def handle(self) -> bytes:
        buf = (C.c_uint8 * COMM_HANDLE_BYTES)()
        _check(lib().fb_comm_handle(self.h, buf))
        return bytes(buf)

    def open(self, handles: list[bytes]):
        if len(handles) != self.world or any(len(x) != COMM_HANDLE_BYTES for x in handles):
            raise ValueError("need one 64-byte handle per rank, in rank order")
        blob = b"".join(handles)
        _check(lib().fb_comm_open(self.h, C.c_char_p(blob)))

    @staticmethod
    def gather_handles(mine: bytes, world: int, group=None) -> list[bytes]:
        """All ranks' handles in rank order through torch.distributed."""
        import torch.distributed as dist

        out = [None] * world
        dist.all_gather_object(out, mine, group=group)
        return out

    @classmethod
    def connect(cls, ctx: Context, max_batch: int, hidden: int, group=None) -> "Comm":
        import torch.distributed as dist

        rank, world = dist.get_rank(group), dist.get_world_size(group)
        c = cls(ctx, rank, world, max_batch, hidden)
        c.open(cls.gather_handles(c.handle(), world, group))
        dist.barrier(group)
        return c

    def close(self):
        if self.h:
            lib().fb_comm_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Model:
    """Quantized Llama/Qwen3 model (ferrite_core::InferenceModel counterpart).

    With ``comm`` the model is this rank's tensor-parallel shard: cfg and the
    tensors given to set_tensor are the full model's; forward returns the
    rank's vocab slice of the logits (``vocab_range``)."""

    def __init__(self, ctx: Context, cfg: dict, comm: Comm | None = None):
        self.ctx = ctx
        self.cfg = dict(cfg)
        self.comm = comm
        c = ModelConfig(**{k: cfg[k] for k, _ in ModelConfig._fields_})
        h = C.c_void_p()
        if comm is None:
            _check(lib().fb_model_create(ctx.h, C.byref(c), C.byref(h)))
        else:
            _check(lib().fb_model_create_tp(ctx.h, C.byref(c), comm.h, C.byref(h)))
        self.h = h
        r, w, vo, vn = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        _check(lib().fb_model_tp_info(h, C.byref(r), C.byref(w), C.byref(vo), C.byref(vn)))
        self.rank, self.world, self.vocab_range = r.value, w.value, (vo.value, vo.value + vn.value)
        self.local = dict(self.cfg, n_heads=cfg["n_heads"] // w.value, n_kv_heads=cfg["n_kv_heads"] // w.value,
                          ffn=cfg["ffn"] // w.value, vocab=vn.value)

    @classmethod
    def from_gguf(cls, ctx: Context, path: str, max_ctx: int | None = None, max_batch: int = 1,
                  comm: "Comm | None" = None) -> "Model":
        """Model with the config and tensors of a llama / qwen3 GGUF file."""
        cfg = gguf_config(path)
        if max_ctx:
            cfg["max_ctx"] = max_ctx
        cfg["max_batch"] = max_batch
        m = cls(ctx, cfg, comm)
        _check(lib().fb_model_load_gguf(m.h, os.fsencode(path)))
        return m

    def set_tensor(self, name: str, layer: int, dtype: int, rows: int, cols: int, data: np.ndarray):
        data = np.ascontiguousarray(data)
        _check(lib().fb_model_set_tensor(self.h, name.encode(), layer, dtype, rows, cols, _np(data)))

    def synth(self, seed: int):
        _check(lib().fb_model_synth(self.h, seed))

    def finalize(self):
        _check(lib().fb_model_finalize(self.h))

    def forward(self, tokens, pos: int) -> np.ndarray:
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        out = np.zeros(self.local["vocab"], dtype=np.float32)
        _check(lib().fb_model_forward(self.h, _np(toks), toks.size, pos, _np(out)))
        return out

    def forward_all(self, tokens, pos: int) -> np.ndarray:
        """Logits of every token, [n, vocab] (multi-token verification)."""
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        out = np.zeros((toks.size, self.local["vocab"]), dtype=np.float32)
        _check(lib().fb_model_forward_all(self.h, _np(toks), toks.size, pos, _np(out)))
        return out

    def prefill(self, tokens) -> np.ndarray:
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        out = np.zeros(self.local["vocab"], dtype=np.float32)
        _check(lib().fb_model_prefill(self.h, _np(toks), toks.size, _np(out)))
        return out

    def decode_greedy(self, tokens, positions) -> np.ndarray:
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        pos = np.ascontiguousarray(np.asarray(positions, dtype=np.int32))
        out = np.zeros(toks.size, dtype=np.int32)
        _check(lib().fb_model_decode_greedy(self.h, _np(toks), _np(pos), toks.size, _np(out)))
        return out

    def decode_dev(self, tok_ptr: int, pos_ptr: int, batch: int, next_ptr: int = 0, logits_ptr: int = 0):
        _check(lib().fb_model_decode_dev(self.h, tok_ptr, pos_ptr, batch, next_ptr or None, logits_ptr or None))

    def clear_cache(self):
        _check(lib().fb_model_clear_cache(self.h))

    def synth_kv(self, seed: int, ctx: int, scale: float = 0.5):
        _check(lib().fb_model_synth_kv(self.h, seed, ctx, scale))

    def read_kv(self, layer: int, which: int, pos: int) -> np.ndarray:
        out = np.zeros(self.local["n_kv_heads"] * self.cfg["head_dim"], dtype=np.float32)
        _check(lib().fb_model_read_kv(self.h, layer, which, pos, _np(out)))
        return out

    def read_activation(self, name: str, row: int = 0) -> np.ndarray:
        c = self.local
        qd, kd = c["n_heads"] * c["head_dim"], c["n_kv_heads"] * c["head_dim"]
        n = {"x": c["hidden"], "qkv": qd + 2 * kd, "q": qd, "attn": qd, "o": c["hidden"], "gate_up": 2 * c["ffn"],
             "down": c["hidden"], "logits": c["vocab"]}[name]
        out = np.zeros(n, dtype=np.float32)
        _check(lib().fb_model_read_activation(self.h, name.encode(), row, _np(out), n))
        return out

    def profile(self, tok_ptr: int, pos_ptr: int, batch: int, steps: int) -> dict:
        """Per-kernel-class milliseconds (summed over `steps` eager steps) and
        launches per step."""
        ms = np.zeros(len(PROF_KINDS), dtype=np.float32)
        nl = np.zeros(len(PROF_KINDS), dtype=np.int32)
        _check(lib().fb_model_profile(self.h, tok_ptr, pos_ptr, batch, steps, _np(ms), _np(nl)))
        return {k: (float(ms[i]), int(nl[i])) for i, k in enumerate(PROF_KINDS)}

    def set_persistent(self, enable: bool) -> bool:
        """Batch-1 decode as one persistent kernel (True) or as the per-op
        kernel chain (False, the default); returns whether the model supports
        the persistent kernel."""
        sup = C.c_int32()
        _check(lib().fb_model_set_persistent(self.h, int(bool(enable)), C.byref(sup)))
        return bool(sup.value)

    def step_timeline(self, tok_ptr: int, pos_ptr: int, n_sms: int = 148) -> np.ndarray:
        """Phase timeline of one eager persistent step: uint64 ns stamps
        [cta][layer + 1][16] (fb_model_step_timeline)."""
        per = (self.cfg["n_layers"] + 1) * 16
        buf = np.zeros(n_sms * per + 1024 * per, dtype=np.uint64)
        ctas, slots = C.c_int32(), C.c_int32()
        _check(lib().fb_model_step_timeline(self.h, tok_ptr, pos_ptr, _np(buf), buf.size, C.byref(ctas),
                                            C.byref(slots)))
        return buf[: ctas.value * per].reshape(ctas.value, self.cfg["n_layers"] + 1, slots.value)

    def launches_per_step(self) -> int:
        v = C.c_int()
        _check(lib().fb_model_launches_per_step(self.h, C.byref(v)))
        return v.value

    def weight_bytes(self) -> int:
        v = C.c_int64()
        _check(lib().fb_model_weight_bytes(self.h, C.byref(v)))
        return v.value

    def close(self):
        if self.h:
            lib().fb_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
