"""GPU parity of the format kernels against the CPU oracle: upload/download,
bit-exact dequantization, Q8_K activation quantization, integer block dots,
and the random-init generator."""
import numpy as np
import pytest

import ferrite_b200 as fb
from conftest import O, gaussian_qweight

pytestmark = pytest.mark.gpu


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("dtype", [O.Q4_K, O.Q6_K])
@pytest.mark.parametrize("n,k", [(16, 256), (37, 1024), (64, 4096)])
def test_upload_download_roundtrip(fbctx, dtype, n, k):
    w = gaussian_qweight(dtype, n, k, seed=n + k)
    t = fb.QTensor.upload(fbctx, dtype, n, k, w)
    assert np.array_equal(t.download(), w.reshape(-1))


@pytest.mark.parametrize("dtype", [O.Q4_K, O.Q6_K])
def test_dequantize_bit_exact(fbctx, torch_cuda, dtype):
    torch = torch_cuda
    n, k = 48, 2048
    w = gaussian_qweight(dtype, n, k, seed=5)
    t = fb.QTensor.upload(fbctx, dtype, n, k, w)
    ref = O.dequantize(dtype, w, n * k).reshape(n, k)
    out = torch.empty(n, k, dtype=torch.float32, device="cuda")
    t.dequantize(out.data_ptr(), fb.F32)
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    for odt, tdt in ((fb.F16, torch.float16), (fb.BF16, torch.bfloat16)):
        o16 = torch.empty(n, k, dtype=tdt, device="cuda")
        t.dequantize(o16.data_ptr(), odt)
        assert torch.equal(o16.cpu(), torch.from_numpy(ref).to(tdt))


def test_dequantize_synth_subnormal_scales(fbctx, torch_cuda):
    """Q6_K super-block scales of sigma = 0.02 weights are fp16 subnormals."""
    torch = torch_cuda
    t = fb.QTensor.synth(fbctx, O.Q6_K, 32, 1024, seed=3, sigma=0.02)
    blocks = t.download()
    ref = O.dequantize(O.Q6_K, blocks, 32 * 1024)
    out = torch.empty(32 * 1024, dtype=torch.float32, device="cuda")
    t.dequantize(out.data_ptr(), fb.F32)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_quantize_q8k_bytes(fbctx, torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(9)
    x = rng.normal(0, 1, (5, 1024)).astype(np.float32)
    x[1, 256:512] = 0.0                       # all-zero block
    x[2, 10], x[2, 20] = 3.5, -3.5            # magnitude tie (first wins)
    x[3, :256] = np.round(rng.normal(0, 4, 256))  # exact .5 products are likely
    x[4] *= 1e-3
    xd = _dev(torch, x)
    out = torch.zeros(5 * 4 * 292, dtype=torch.uint8, device="cuda")
    fb.quantize_q8k(fbctx, xd.data_ptr(), 5, 1024, out.data_ptr())
    got = out.cpu().numpy()
    ref = O.quantize_q8k(x).reshape(-1)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("dtype", [O.Q4_K, O.Q6_K])
@pytest.mark.parametrize("n,k", [(16, 256), (45, 2048), (128, 4096)])
def test_block_dots_bit_exact(fbctx, torch_cuda, dtype, n, k):
    torch = torch_cuda
    w = gaussian_qweight(dtype, n, k, seed=n * 7 + k)
    x = np.random.default_rng(k).normal(0, 1, k).astype(np.float32)
    t = fb.QTensor.upload(fbctx, dtype, n, k, w)
    xd = _dev(torch, x)
    sc = torch.zeros(n, k // 256, dtype=torch.int32, device="cuda")
    mn = torch.zeros(n, k // 256, dtype=torch.int32, device="cuda")
    fb.block_dots(fbctx, t, xd.data_ptr(), sc.data_ptr(), mn.data_ptr())
    rsc, rmn = O.block_dots(dtype, w, n, k, O.quantize_q8k(x))
    assert np.array_equal(sc.cpu().numpy(), rsc)
    assert np.array_equal(mn.cpu().numpy(), rmn)


@pytest.mark.parametrize("dtype", [O.Q4_K, O.Q6_K])
def test_synth_matches_oracle_generator(fbctx, dtype):
    t = fb.QTensor.synth(fbctx, dtype, 24, 1024, seed=1234, sigma=0.02)
    ref = (O.synth_q4k if dtype == O.Q4_K else O.synth_q6k)(1234, 24 * 4, 0.02)
    assert np.array_equal(t.download(), ref)
