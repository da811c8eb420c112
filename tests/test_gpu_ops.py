"""GPU RMSNorm / RoPE / SwiGLU / paged flash-decode attention vs CPU
references (oracle for the elementwise ops, float64 numpy for attention)."""
import math

import numpy as np
import pytest

import ferrite_b200 as fb
from conftest import O, assert_close

pytestmark = pytest.mark.gpu


def test_rmsnorm(fbctx, torch_cuda):
    torch = torch_cuda
    x = np.random.default_rng(1).normal(0, 3, (6, 4096)).astype(np.float32)
    g = (1 + np.random.default_rng(2).normal(0, 0.02, 4096)).astype(np.float32)
    xd, gd = torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda()
    yd = torch.empty_like(xd)
    fb.rmsnorm(fbctx, xd.data_ptr(), gd.data_ptr(), yd.data_ptr(), 6, 4096, 1e-6)
    ref = O.rmsnorm(x, g, 1e-6)
    # sums of squares in binary64 on both sides: bit-identical
    assert np.array_equal(yd.cpu().numpy(), ref)


@pytest.mark.parametrize("mode", [0, 1])
def test_rope(fbctx, torch_cuda, mode):
    torch = torch_cuda
    x = np.random.default_rng(mode).normal(0, 1, (3, 8, 128)).astype(np.float32)
    xd = torch.from_numpy(x.copy()).cuda()
    fb.rope(fbctx, xd.data_ptr(), 3, 8, 128, 4090, 1e6, mode)
    ref = x.copy()
    for t in range(3):
        O.lib().or_rope(O._p(ref[t]), 8, 128, 4090 + t, 1e6, mode)
    assert np.array_equal(xd.cpu().numpy(), ref)  # same tables, same rounding


def test_swiglu(fbctx, torch_cuda):
    torch = torch_cuda
    g = np.random.default_rng(3).normal(0, 2, (4, 1024)).astype(np.float32)
    u = np.random.default_rng(4).normal(0, 2, (4, 1024)).astype(np.float32)
    gd, ud = torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda()
    od = torch.empty_like(gd)
    fb.swiglu(fbctx, gd.data_ptr(), ud.data_ptr(), od.data_ptr(), 4, 1024)
    ref = O.silu(g) * u
    assert np.array_equal(od.cpu().numpy(), ref)  # same binary64 exp on both sides
    # and within CUDA's own SiLU (expf-based) error bounds
    want = torch.nn.functional.silu(gd) * ud
    np.testing.assert_allclose(od.cpu().numpy(), want.cpu().numpy(), rtol=2e-6, atol=1e-7)


def attn_reference(q, kp, vp, bt, lens, page):
    b, nh, hd = q.shape
    nkv = kp.shape[1]
    g = nh // nkv
    out = np.zeros_like(q, dtype=np.float64)
    for s in range(b):
        L = lens[s]
        pages = [bt[s, i // page] for i in range(L)]
        K = np.stack([kp[pages[i], :, i % page] for i in range(L)]).astype(np.float64)  # [L, nkv, hd]
        V = np.stack([vp[pages[i], :, i % page] for i in range(L)]).astype(np.float64)
        for h in range(nh):
            sc = K[:, h // g] @ q[s, h].astype(np.float64) / math.sqrt(hd)
            p = np.exp(sc - sc.max())
            out[s, h] = (p / p.sum()) @ V[:, h // g]
    return out


@pytest.mark.parametrize("nh,nkv", [(32, 8), (64, 8), (8, 8), (16, 8)])
@pytest.mark.parametrize("page", [32, 64])
def test_attn_decode_paged(fbctx, torch_cuda, nh, nkv, page):
    torch = torch_cuda
    rng = np.random.default_rng(nh + page)
    hd, b = 128, 5
    lens = np.array([1, page - 1, page + 1, 2 * page + 3, 700], dtype=np.int32)
    max_pages = int(math.ceil(lens.max() / page))
    num_pages = b * max_pages + 3
    perm = rng.permutation(num_pages)[: b * max_pages].reshape(b, max_pages).astype(np.int32)
    kp = rng.normal(0, 1, (num_pages, nkv, page, hd)).astype(np.float16)
    vp = rng.normal(0, 1, (num_pages, nkv, page, hd)).astype(np.float16)
    q = rng.normal(0, 1, (b, nh, hd)).astype(np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    # K pages are dim-major on the device: [page][kv head][hd][page tokens]
    qd, kd, vd, btd, ld = t(q), t(kp.transpose(0, 1, 3, 2)), t(vp), t(perm), t(lens)
    out = torch.zeros((b, nh, hd), dtype=torch.float32, device="cuda")
    fb.attn_decode(fbctx, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), btd.data_ptr(), ld.data_ptr(),
                   out.data_ptr(), b, nh, nkv, hd, page, max_pages, num_pages, int(lens.max()), 1.0 / math.sqrt(hd))
    ref = attn_reference(q, kp, vp, perm, lens, page)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-4, atol=1e-5)
    assert fbctx.error_word() == 0


@pytest.mark.parametrize("nh,nkv", [(32, 8), (8, 1)])
@pytest.mark.parametrize("page", [32, 64])
def test_attn_decode_long_ring_reuse(fbctx, torch_cuda, nh, nkv, page):
    """Contexts whose splits hold more 64-token chunks than the shared-memory
    ring has stages (16 splits: > 4 chunks without clusters, > 2 with), so
    stages are refilled while other warps still work on the ring; both entry
    points (cluster merge where the GPU holds one, and the cluster-free merge
    of the allocation-free entry) against an f64 reference and each other."""
    torch = torch_cuda
    rng = np.random.default_rng(nh * 7 + page)
    hd, lens = 128, np.array([4100, 2500, 1, 5000 - page + 3], dtype=np.int32)
    b = lens.size
    max_pages = int(math.ceil(lens.max() / page))
    num_pages = b * max_pages + 5
    perm = rng.permutation(num_pages)[: b * max_pages].reshape(b, max_pages).astype(np.int32)
    kp = rng.normal(0, 1, (num_pages, nkv, page, hd)).astype(np.float16)
    vp = rng.normal(0, 1, (num_pages, nkv, page, hd)).astype(np.float16)
    q = rng.normal(0, 1, (b, nh, hd)).astype(np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    qd, kd, vd, btd, ld = t(q), t(kp.transpose(0, 1, 3, 2)), t(vp), t(perm), t(lens)
    ref = attn_reference(q, kp, vp, perm, lens, page)
    outs = []
    for fn in (fb.attn_decode, fb.attn_decode_noalloc):
        out = torch.full((b, nh, hd), float("nan"), dtype=torch.float32, device="cuda")
        fn(fbctx, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), btd.data_ptr(), ld.data_ptr(), out.data_ptr(), b, nh,
           nkv, hd, page, max_pages, num_pages, int(lens.max()), 1.0 / math.sqrt(hd))
        outs.append(out.cpu().numpy())
        np.testing.assert_allclose(outs[-1], ref, rtol=1e-4, atol=1e-5)
    # binary64 softmax and P.V: the split and warp layout does not show in the f32 result
    assert np.array_equal(outs[0], outs[1])
    assert fbctx.error_word() == 0


@pytest.mark.parametrize("entry", ["attn_decode", "attn_decode_noalloc"])
def test_attn_decode_rejects_page_ids_outside_the_pool(fbctx, torch_cuda, entry):
    """A block-table entry outside [0, num_pages) (a stale or corrupt id from
    the caller) is never dereferenced: the kernel skips that page and sets
    the error word's bad-page bit.  The pools here are exactly num_pages
    pages long, so a read through the bad id would leave the allocation."""
    torch = torch_cuda
    rng = np.random.default_rng(77)
    hd, nh, nkv, page, b = 128, 32, 8, 64, 2
    lens = np.array([200, 130], dtype=np.int32)
    max_pages = 4
    num_pages = b * max_pages
    bt = np.arange(num_pages, dtype=np.int32).reshape(b, max_pages)
    bt[1, 1] = num_pages + 1000  # sequence 1's second page: outside the pool
    kp = rng.normal(0, 1, (num_pages, nkv, page, hd)).astype(np.float16)
    vp = rng.normal(0, 1, (num_pages, nkv, page, hd)).astype(np.float16)
    q = rng.normal(0, 1, (b, nh, hd)).astype(np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    qd, kd, vd, btd, ld = t(q), t(kp.transpose(0, 1, 3, 2)), t(vp), t(bt), t(lens)
    out = torch.zeros((b, nh, hd), dtype=torch.float32, device="cuda")
    assert fbctx.error_word() == 0
    getattr(fb, entry)(fbctx, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), btd.data_ptr(), ld.data_ptr(),
                       out.data_ptr(), b, nh, nkv, hd, page, max_pages, num_pages, int(lens.max()),
                       1.0 / math.sqrt(hd))
    torch.cuda.synchronize()
    assert fbctx.error_word() & 0x8, "bad-page bit not set"
    # sequence 0 only uses pages inside the pool: its result is unaffected
    ref = attn_reference(q[:1], kp, vp, bt[:1], lens[:1], page)
    np.testing.assert_allclose(out.cpu().numpy()[:1], ref, rtol=1e-4, atol=1e-5)
    assert fbctx.error_word() == 0
