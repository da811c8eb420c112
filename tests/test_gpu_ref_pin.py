"""Pins the oracle (and this library) against the reference's own code.

The reference's CUDA dequantization kernels (ferrite-os/crates/internal/
ptx-kernels/kernels/candle/quantized.cu:936-1151, `dequantize_block_q4_K_f32`
and `dequantize_block_q6_K_f32`), compiled from the reference sources by
oracle/ref/Makefile into oracle/_ref/libref_quant.so, dequantize the same
GGUF blocks as the CPU oracle and this library's device kernels; all three
must agree bit for bit.  Blocks come from the oracle's quantizer (Gaussian
weights of several scales) and from the synthetic-weight generator (fp16
subnormal super-block scales), plus hand-made extremes.
"""
import ctypes as C
import os

import numpy as np
import pytest

import ferrite_b200 as fb
from conftest import O, gaussian_qweight

pytestmark = pytest.mark.gpu

REF_SO = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "libref_quant.so")


@pytest.fixture(scope="module")
def ref_lib():
    if not os.path.exists(REF_SO):
        pytest.skip("oracle/_ref/libref_quant.so is not built (needs the reference sources at build time)")
    lib = C.CDLL(REF_SO)
    lib.ref_dequantize_host.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_void_p]
    lib.ref_dequantize_host.restype = C.c_int
    return lib


def ref_dequantize(lib, dtype, blocks, nblocks):
    blocks = np.ascontiguousarray(blocks)
    out = np.empty(nblocks * 256, dtype=np.float32)
    rc = lib.ref_dequantize_host(dtype, blocks.ctypes.data, nblocks, out.ctypes.data)
    assert rc == 0, f"reference kernel launch failed: cudaError {rc}"
    return out


def extreme_blocks(dtype, nblocks, seed):
    """Random bytes with the fp16 scales forced to finite values (GGUF allows any)."""
    rng = np.random.default_rng(seed)
    bb = 144 if dtype == O.Q4_K else 210
    raw = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    scales = rng.choice(np.array([0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0x8001, 0xFBFF, 0x1234, 0x0000],
                                 dtype=np.uint16), size=(nblocks, 2))
    if dtype == O.Q4_K:
        raw[:, 0:4] = scales.view(np.uint8).reshape(nblocks, 4)
    else:
        raw[:, 208:210] = scales[:, :1].view(np.uint8).reshape(nblocks, 2)
    return raw.reshape(-1)


@pytest.mark.parametrize("dtype", [O.Q4_K, O.Q6_K])
def test_dequant_matches_reference_cuda(fbctx, torch_cuda, ref_lib, dtype):
    torch = torch_cuda
    cases = []
    for sigma in (0.02, 1.0, 300.0):
        cases.append(("gaussian sigma=%g" % sigma, gaussian_qweight(dtype, 32, 1024, seed=int(sigma * 7) + dtype,
                                                                    sigma=sigma), 32, 1024))
    t = fb.QTensor.synth(fbctx, dtype, 16, 2048, seed=21, sigma=0.02)
    cases.append(("synthetic subnormal scales", t.download(), 16, 2048))
    cases.append(("random bytes, extreme scales", extreme_blocks(dtype, 64, seed=dtype), 16, 1024))
    for what, blocks, n, k in cases:
        nbl = n * k // 256
        ref = ref_dequantize(ref_lib, dtype, blocks, nbl)
        orc = O.dequantize(dtype, blocks, n * k)
        assert np.array_equal(orc.view(np.uint32), ref.view(np.uint32)), f"oracle vs reference CUDA ({what})"
        dev = fb.QTensor.upload(fbctx, dtype, n, k, blocks)
        out = torch.empty(n * k, dtype=torch.float32, device="cuda")
        dev.dequantize(out.data_ptr(), fb.F32)
        got = out.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), f"device vs reference CUDA ({what})"


def ref_qmatmul(lib, dtype, mode, w, n, k, x):
    lib.ref_qmatmul_vec_host.argtypes = [C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    lib.ref_qmatmul_vec_host.restype = C.c_int
    w = np.ascontiguousarray(w)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(n, dtype=np.float32)
    rc = lib.ref_qmatmul_vec_host(dtype, mode, w.ctypes.data, n, k, x.ctypes.data, y.ctypes.data)
    assert rc == 0, f"reference kernel launch failed: cudaError {rc}"
    return y


@pytest.mark.parametrize("dtype,n,k", [(O.Q4_K, 4096, 4096), (O.Q4_K, 1024, 4096), (O.Q6_K, 4096, 12288),
                                       (O.Q6_K, 2048, 4096)])
def test_qmatmul_vs_reference_cuda(fbctx, torch_cuda, ref_lib, dtype, n, k):
    """The reference's own decode QMatMul kernels on the same weights and
    activation: its float DMMV kernel (dequantize_mul_mat_vec_q*_k) against
    the oracle's float QMatMul (f32 accumulation order only: 1e-5 relative of
    the row's scale), and its integer MMVQ kernel (Q8_1 activations, blocks of
    32) against this library's integer GEMV (Q8_K activations, the CPU
    path's): the two 8-bit activation roundings differ, so the bar is their
    quantization noise -- a relative RMS difference below 1%."""
    torch = torch_cuda
    w = gaussian_qweight(dtype, n, k, seed=n + k + dtype)
    x = np.random.default_rng(k).normal(0, 1, k).astype(np.float32)
    ref_float = ref_qmatmul(ref_lib, dtype, 1, w, n, k, x)
    orc_float = O.qmatmul_f32(dtype, w, n, k, x[None])[0]
    scale = np.abs(orc_float).max()
    assert np.abs(ref_float - orc_float).max() <= 1e-5 * scale, "oracle float QMatMul vs the reference's DMMV kernel"
    ref_int = ref_qmatmul(ref_lib, dtype, 0, w, n, k, x)
    t = fb.QTensor.upload(fbctx, dtype, n, k, w)
    xd = torch.from_numpy(x[None].copy()).cuda()
    yd = torch.empty((1, n), dtype=torch.float32, device="cuda")
    fb.QMatMul(t).forward(xd.data_ptr(), yd.data_ptr(), 1)
    dev = yd.cpu().numpy()[0]
    rel = np.sqrt(np.mean((dev - ref_int) ** 2)) / np.sqrt(np.mean(ref_int.astype(np.float64) ** 2))
    assert rel < 1e-2, f"integer paths: relative RMS difference {rel:.3g}"
    # and each integer path stays that close to the float product
    for what, v in (("device", dev), ("reference MMVQ", ref_int)):
        r = np.sqrt(np.mean((v - orc_float) ** 2)) / np.sqrt(np.mean(orc_float.astype(np.float64) ** 2))
        assert r < 1e-2, f"{what} vs float product: {r:.3g}"


# configs[1]-style decode shapes at batch 1 (n x k): attention q/o, k/v,
# gate and up (each), down (Q6_K), lm_head (Q6_K)
SPEED_SHAPES = [(O.Q4_K, 4096, 4096), (O.Q4_K, 1024, 4096), (O.Q4_K, 12288, 4096), (O.Q6_K, 4096, 12288),
                (O.Q6_K, 151936, 4096)]


def test_gemv_speed_vs_reference_cuda(fbctx, torch_cuda, ref_lib):
    """Device time of one decode QMatMul (activation quantization + GEMV) of
    this library vs the reference's MMVQ kernels on the same B200, both with
    resident inputs and back-to-back launches; prints a table (run with -s)
    and requires this library to be faster on every shape.  The reference
    is launched from a C loop; this library's calls are captured in a CUDA
    graph and replayed, so both columns are device time (the Python-launched
    column is shown beside it: at 1024 rows it is ctypes-bound)."""
    torch = torch_cuda
    ref_lib.ref_qmatmul_vec_time.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int,
                                             C.c_void_p]
    ref_lib.ref_qmatmul_vec_time.restype = C.c_int
    rows = []
    for dtype, n, k in SPEED_SHAPES:
        w = fb.QTensor.synth(fbctx, dtype, n, k, seed=n + k)
        blocks = w.download()
        x = np.random.default_rng(1).normal(0, 1, k).astype(np.float32)
        ms = np.zeros(1, dtype=np.float32)
        rc = ref_lib.ref_qmatmul_vec_time(dtype, blocks.ctypes.data, n, k, x.ctypes.data, 5, 50, ms.ctypes.data)
        assert rc == 0
        xd = torch.from_numpy(x[None].copy()).cuda()
        yd = torch.empty((1, n), dtype=torch.float32, device="cuda")
        mm = fb.QMatMul(w)
        for _ in range(5):
            mm.forward(xd.data_ptr(), yd.data_ptr(), 1)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(50):
            mm.forward(xd.data_ptr(), yd.data_ptr(), 1)
        e1.record()
        torch.cuda.synchronize()
        eager = e0.elapsed_time(e1) / 50
        # the same 50 calls captured once and replayed: device time without
        # the Python/ctypes launch cost the reference's C loop does not pay
        old_stream, cap = fbctx.stream, torch.cuda.Stream()
        fbctx.set_stream(cap.cuda_stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            for _ in range(50):
                mm.forward(xd.data_ptr(), yd.data_ptr(), 1)
        fbctx.set_stream(old_stream)
        g.replay()
        torch.cuda.synchronize()
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        ours = e0.elapsed_time(e1) / 50
        del g
        gb = n * k / 256 * (144 if dtype == O.Q4_K else 210) / 1e9
        rows.append((dtype, n, k, float(ms[0]), ours, eager, gb / (ms[0] * 1e-3), gb / (ours * 1e-3)))
    print("\n| weight | n x k | reference MMVQ us | this library us (graph) | this library us (Python launches) | "
          "reference GB/s | this library GB/s | speed-up |")
    print("|---|---|---|---|---|---|---|---|")
    for dtype, n, k, r, o, ea, rg, og in rows:
        print(f"| {'Q4_K' if dtype == O.Q4_K else 'Q6_K'} | {n} x {k} | {r * 1e3:.1f} | {o * 1e3:.1f} | {ea * 1e3:.1f} | "
              f"{rg:.0f} | {og:.0f} | {r / o:.2f}x |")
    for row in rows:
        assert row[4] < row[3], f"slower than the reference on {row[:3]}"
