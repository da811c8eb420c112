"""GPU QMatMul (decode GEMV, m <= 16) against the oracle's candle-CPU
QMatMul on identical seeded inputs: tolerance 1e-3 relative / 1e-2 absolute
per element (the integer partials are bit-exact; only the f32 combination
order differs)."""
import numpy as np
import pytest

import ferrite_b200 as fb
from conftest import O, assert_close, gaussian_qweight

pytestmark = pytest.mark.gpu


def run(fbctx, torch, dtype, n, k, m, w, x):
    t = fb.QTensor.upload(fbctx, dtype, n, k, w)
    xd = torch.from_numpy(x).cuda()
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    fb.QMatMul(t).forward(xd.data_ptr(), y.data_ptr(), m)
    return y.cpu().numpy()


def test_c1_q4k_4096x4096_m1(fbctx, torch_cuda):
    """Config C1: W 4096x4096 ~ N(0, 0.02) seed 0 -> Q4_K; x 1x4096 ~ N(0, 1) seed 1."""
    n = k = 4096
    w = gaussian_qweight(O.Q4_K, n, k, seed=0)
    x = np.random.default_rng(1).normal(0, 1, (1, k)).astype(np.float32)
    got = run(fbctx, torch_cuda, O.Q4_K, n, k, 1, w, x)
    assert_close(got, O.qmatmul(O.Q4_K, w, n, k, x), what="C1")


@pytest.mark.parametrize("m", [1, 4, 16])
@pytest.mark.parametrize("dtype,n,k", [(O.Q4_K, 4096, 4096), (O.Q4_K, 1024, 4096), (O.Q4_K, 12288, 4096),
                                       (O.Q6_K, 4096, 12288)])
def test_c2_sweep(fbctx, torch_cuda, dtype, n, k, m):
    w = gaussian_qweight(dtype, n, k, seed=n + k + dtype)
    x = np.random.default_rng(m).normal(0, 1, (m, k)).astype(np.float32)
    got = run(fbctx, torch_cuda, dtype, n, k, m, w, x)
    assert_close(got, O.qmatmul(dtype, w, n, k, x), what=f"{dtype} {n}x{k} m={m}")


@pytest.mark.parametrize("m", [1, 16])
def test_c2_lm_head_q6k(fbctx, torch_cuda, m):
    """4096 -> 151936 Q6_K (random-init blocks from the shared generator)."""
    n, k = 151936, 4096
    w = O.synth_q6k(77, n * k // 256, 0.02)
    x = np.random.default_rng(3).normal(0, 1, (m, k)).astype(np.float32)
    got = run(fbctx, torch_cuda, O.Q6_K, n, k, m, w, x)
    assert_close(got, O.qmatmul(O.Q6_K, w, n, k, x), what=f"lm_head m={m}")


@pytest.mark.parametrize("dtype", [O.Q4_K, O.Q6_K])
@pytest.mark.parametrize("n,k,m", [(1, 256, 1), (17, 256, 3), (1000, 768, 9), (333, 2560, 13), (40, 512, 8)])
def test_ragged_shapes(fbctx, torch_cuda, dtype, n, k, m):
    w = gaussian_qweight(dtype, n, k, seed=n * 31 + k)
    x = np.random.default_rng(n).normal(0, 1, (m, k)).astype(np.float32)
    x[0, :256] = 0.0  # an all-zero activation block
    got = run(fbctx, torch_cuda, dtype, n, k, m, w, x)
    assert_close(got, O.qmatmul(dtype, w, n, k, x), what=f"{dtype} {n}x{k} m={m}")


@pytest.mark.parametrize("m", [5, 9, 13, 16])
@pytest.mark.parametrize("n,k", [(2368, 4096), (2400, 2560), (4096, 1024)])
def test_mma_path_many_tiles(fbctx, torch_cuda, n, k, m):
    """Q4_K with m = 5..16 (the tensor-core consumer) and at least one
    16-row tile per SM, so CTAs loop over several tiles and the record ring
    wraps across tiles (k = 2560: 10 super-blocks, not a multiple of the
    warps per CTA).  The row sums are the oracle's binary64 sums rounded
    once, element for element."""
    w = gaussian_qweight(O.Q4_K, n, k, seed=3 * n + k)
    x = np.random.default_rng(m + n).normal(0, 1, (m, k)).astype(np.float32)
    x[m - 1, 256:512] = 0.0  # an all-zero activation block in the last row
    got = run(fbctx, torch_cuda, O.Q4_K, n, k, m, w, x)
    ref = O.qmatmul(O.Q4_K, w, n, k, x)
    assert_close(got, ref, what=f"staged {n}x{k} m={m}")
    same = np.mean(got.view(np.uint32) == ref.view(np.uint32))
    assert same >= 0.9999, f"{same:.6f} of the outputs bit-identical"


def test_batch_rows_independent(fbctx, torch_cuda):
    """Each activation row's result does not depend on the other rows."""
    n, k = 512, 1024
    w = gaussian_qweight(O.Q4_K, n, k, seed=2)
    x = np.random.default_rng(4).normal(0, 1, (16, k)).astype(np.float32)
    full = run(fbctx, torch_cuda, O.Q4_K, n, k, 16, w, x)
    for r in (0, 7, 15):
        one = run(fbctx, torch_cuda, O.Q4_K, n, k, 1, w, np.ascontiguousarray(x[r:r + 1]))
        np.testing.assert_allclose(one[0], full[r], rtol=1e-6, atol=1e-6)


def test_qmatmul_large_m_chunks(fbctx, torch_cuda):
    n, k, m = 256, 512, 40
    w = gaussian_qweight(O.Q4_K, n, k, seed=6)
    x = np.random.default_rng(6).normal(0, 1, (m, k)).astype(np.float32)
    t = fb.QTensor.upload(fbctx, O.Q4_K, n, k, w)
    torch = torch_cuda
    xd = torch.from_numpy(x).cuda()
    y = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    fb.QMatMul(t).forward_q8k(xd.data_ptr(), y.data_ptr(), m)
    assert_close(y.cpu().numpy(), O.qmatmul(O.Q4_K, w, n, k, x), what="m=40 q8k")
