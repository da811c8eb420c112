"""Prefill QMatMul (m > 16 rows) on the tensor cores.

Two checks per case, on identical seeded inputs:
* kernel arithmetic: against an exact f64 restatement of the kernel's
  operands -- weights w = fp16(fp16(d*sc) * q - fp16(dmin*m)) (Q4_K) or
  fp16(fp16(d*sc) * (q - 32)) (Q6_K) from the oracle's exact per-weight
  factors, X scaled by the kernel's power-of-two row scale and rounded to
  fp16 -- only the f32 accumulation order differs, so the bound is tight;
* parity with the oracle's float QMatMul (f32 dequantized W times f32 X,
  binary64 accumulation): the fp16 operands are the only difference;
  tolerance 1e-3 relative / 1e-2 absolute per element.
"""
import numpy as np
import pytest

import ferrite_b200 as fb
from conftest import O, assert_close, gaussian_qweight

pytestmark = pytest.mark.gpu


def run(fbctx, torch, dtype, n, k, w, x):
    m = x.shape[0]
    t = fb.QTensor.upload(fbctx, dtype, n, k, w)
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    fb.QMatMul(t).forward(xd.data_ptr(), y.data_ptr(), m)
    torch.cuda.synchronize()
    assert fbctx.error_word() == 0
    return y.cpu().numpy()


def fp16_weights(dtype, w, n, k):
    sc, off, q = O.dequant_parts(dtype, w, n * k)
    s16 = sc.astype(np.float16).astype(np.float64)
    o16 = off.astype(np.float16).astype(np.float64)
    return (s16 * q.astype(np.float64) - o16).astype(np.float16).reshape(n, k)


def emulate(dtype, w, n, k, x):
    wf = fp16_weights(dtype, w, n, k).astype(np.float64)
    amax = np.abs(x).max(axis=1)
    e = np.zeros(x.shape[0], dtype=np.int64)
    while True:  # smallest e >= 0 with amax / 2^e <= 32768
        over = amax > np.ldexp(np.float64(32768.0), e)
        if not over.any():
            break
        e += over
    s = np.ldexp(1.0, e)
    xh = (x / s[:, None].astype(np.float32)).astype(np.float16).astype(np.float64)
    return (xh @ wf.T) * s[:, None]


@pytest.mark.parametrize("dtype,n,k,m", [(O.Q4_K, 512, 1024, 200), (O.Q4_K, 128, 256, 17),
                                         (O.Q6_K, 256, 2048, 130), (O.Q4_K, 1024, 4096, 333),
                                         (O.Q6_K, 4096, 12288, 64),
                                         # from 512 rows: weights dequantized once, then the fp16 GEMM
                                         (O.Q4_K, 1024, 4096, 512), (O.Q6_K, 4096, 12288, 600),
                                         (O.Q4_K, 6144, 4096, 2048), (O.Q4_K, 8192, 1024, 777)])
def test_prefill_gemm(fbctx, torch_cuda, dtype, n, k, m):
    w = gaussian_qweight(dtype, n, k, seed=n + 3 * k + dtype)
    x = np.random.default_rng(m + n).normal(0, 1, (m, k)).astype(np.float32)
    got = run(fbctx, torch_cuda, dtype, n, k, w, x)
    emu = emulate(dtype, w, n, k, x)
    scale = np.abs(emu).max()
    err = np.abs(got - emu).max()
    assert err <= 2e-5 * scale + 1e-6, f"kernel vs fp16-operand emulation: max err {err:.3g} (scale {scale:.3g})"
    ref = O.qmatmul_f32(dtype, w, n, k, x)
    assert_close(got, ref, what=f"prefill {dtype} {n}x{k} m={m} vs oracle f32 QMatMul")


def test_prefill_gemm_large_rows(fbctx, torch_cuda):
    """Rows beyond the fp16 range take a power-of-two scale (exact)."""
    dtype, n, k, m = O.Q4_K, 256, 1024, 40
    w = gaussian_qweight(dtype, n, k, seed=11)
    x = np.random.default_rng(5).normal(0, 1, (m, k)).astype(np.float32)
    x[3] *= 1e5
    x[17] *= 3e6
    got = run(fbctx, torch_cuda, dtype, n, k, w, x)
    emu = emulate(dtype, w, n, k, x)
    rel = np.abs(got - emu) / (np.abs(emu).max(axis=1, keepdims=True) + 1e-30)
    assert rel.max() <= 2e-5, f"max row-relative err {rel.max():.3g}"
    assert np.isfinite(got).all()


@pytest.mark.parametrize("dtype,n,k", [(O.Q4_K, 1024, 4096), (O.Q6_K, 512, 12288)])
def test_two_pass_equals_fused(fbctx, torch_cuda, dtype, n, k):
    """Below 512 rows the weights are dequantized inside the GEMM (once per
    256-row tile); from 512 rows they are dequantized once into fp16 and
    multiplied by the plain fp16 GEMM.  Same fp16 operands, same MMA shape
    and k order: the rows the two runs share must be bit-identical."""
    w = gaussian_qweight(dtype, n, k, seed=n + k)
    x = np.random.default_rng(9).normal(0, 1, (700, k)).astype(np.float32)
    fused = run(fbctx, torch_cuda, dtype, n, k, w, x[:333])
    two = run(fbctx, torch_cuda, dtype, n, k, w, x)
    assert np.array_equal(fused, two[:333])


@pytest.mark.parametrize("dtype,n,k", [(O.Q4_K, 1024, 4096), (O.Q6_K, 4096, 12288)])
def test_prefill_weight_cache_bit_identical(fbctx, torch_cuda, dtype, n, k):
    """From 512 rows the first pass over a tensor keeps its fp16 copy
    (fb_ctx_set_prefill_weight_cache, on by default) and later passes skip the
    dequantization: the cache-filling pass, a cached pass and a run with the
    cache off must give the same bits."""
    torch = torch_cuda
    w = gaussian_qweight(dtype, n, k, seed=2 * n + k)
    x = np.random.default_rng(21).normal(0, 1, (640, k)).astype(np.float32)
    t = fb.QTensor.upload(fbctx, dtype, n, k, w)
    xd = torch.from_numpy(x).cuda()

    def once():
        y = torch.full((640, n), float("nan"), dtype=torch.float32, device="cuda")
        fb.QMatMul(t).forward(xd.data_ptr(), y.data_ptr(), 640)
        torch.cuda.synchronize()
        return y.cpu().numpy()

    try:
        fbctx.set_prefill_weight_cache(False)
        off = once()
        fbctx.set_prefill_weight_cache(True)
        fill, cached = once(), once()
    finally:
        fbctx.set_prefill_weight_cache(True)
    assert fbctx.error_word() == 0
    assert np.array_equal(off, fill) and np.array_equal(fill, cached)
