"""Pins the oracle against the reference's own code.

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
