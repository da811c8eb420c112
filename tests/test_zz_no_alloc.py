"""Allocation-free decode attention (fb_attn_decode_noalloc).

Callers running under a pooled or hooked device allocator (ferrite-os routes
device allocations through its TLSF pool) or in loops that must not take the
synchronisation cudaMalloc/cudaFree can imply cannot let the library grow a
workspace; the no-alloc entry point keeps its split-K scratch in a fixed
device array instead.  These tests call it through the C ABI and check it
against the allocating entry point, fb_attn_decode, on the same inputs; this
file is collected last so a failure here leaves every other result in place.
"""
import math

import numpy as np
import pytest

import ferrite_b200 as fb
from conftest import assert_close

pytestmark = pytest.mark.gpu


def make_inputs(torch, seed, b, nh, nkv, page, lens):
    rng = np.random.default_rng(seed)
    hd = 128
    max_pages = int(math.ceil(max(lens) / page))
    num_pages = b * max_pages + 2
    bt = rng.permutation(num_pages)[: b * max_pages].reshape(b, max_pages).astype(np.int32)
    kp = rng.normal(0, 1, (num_pages, nkv, page, hd)).astype(np.float16)
    vp = rng.normal(0, 1, (num_pages, nkv, page, hd)).astype(np.float16)
    q = rng.normal(0, 1, (b, nh, hd)).astype(np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    # K pages are dim-major on the device: [page][kv head][hd][page tokens]
    return dict(q=t(q), k=t(kp.transpose(0, 1, 3, 2)), v=t(vp), bt=t(bt), lens=t(np.asarray(lens, np.int32)), b=b,
                nh=nh, nkv=nkv, page=page, max_pages=max_pages, num_pages=num_pages, max_len=int(max(lens)))


def run(fn, ctx, torch, d):
    out = torch.full((d["b"], d["nh"], 128), float("nan"), dtype=torch.float32, device="cuda")
    fn(ctx, d["q"].data_ptr(), d["k"].data_ptr(), d["v"].data_ptr(), d["bt"].data_ptr(), d["lens"].data_ptr(),
       out.data_ptr(), d["b"], d["nh"], d["nkv"], 128, d["page"], d["max_pages"], d["num_pages"], d["max_len"],
       1.0 / math.sqrt(128))
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_noalloc_matches_allocating_entry_point_two_calls(fbctx, torch_cuda):
    torch = torch_cuda
    cases = [(1, dict(b=3, nh=32, nkv=8, page=64, lens=[5, 130, 1000])),
             (2, dict(b=2, nh=64, nkv=8, page=64, lens=[1000, 77]))]
    for seed, shape in cases:  # two calls in a row, second reuses the shared scratch
        d = make_inputs(torch, seed, **shape)
        ref = run(fb.attn_decode, fbctx, torch, d)
        got = run(fb.attn_decode_noalloc, fbctx, torch, d)
        assert np.isfinite(got).all()
        assert_close(got, ref, what=f"noalloc vs fb_attn_decode (seed {seed})")
    assert fbctx.error_word() == 0


def test_noalloc_rejects_oversized_request(fbctx, torch_cuda):
    torch = torch_cuda
    d = make_inputs(torch, 3, b=1, nh=8, nkv=8, page=64, lens=[64])
    # 16 sequences x 64 heads x 16 splits x 1040 B = 17 MB: > 4 MiB
    with pytest.raises(fb.FerriteError, match="exceeds the fixed"):
        fb.attn_decode_noalloc(fbctx, d["q"].data_ptr(), d["k"].data_ptr(), d["v"].data_ptr(), d["bt"].data_ptr(),
                               d["lens"].data_ptr(), d["q"].data_ptr(), 16, 64, 8, 128, 64, 128, 128, 8192,
                               0.088)


def noalloc_bytes(b, nh, nkv):
    """Scratch a call needs: split partials (16 splits x (128 dims + max,
    sum) binary64 per head) plus the merge counters rounded up to 256 bytes."""
    return b * nh * 16 * 130 * 8 + (b * nkv * 4 + 255) // 256 * 256


def test_noalloc_largest_accepted_shape(fbctx, torch_cuda):
    """The largest batch the fixed scratch accepts for 32 heads / 8 kv heads
    runs and matches fb_attn_decode; one more sequence is rejected."""
    torch = torch_cuda
    limit = 4 << 20
    b = max(x for x in range(1, 64) if noalloc_bytes(x, 32, 8) <= limit)
    assert noalloc_bytes(b + 1, 32, 8) > limit
    lens = [1 + (97 * i) % 600 for i in range(b)]
    d = make_inputs(torch, 4, b=b, nh=32, nkv=8, page=64, lens=lens)
    ref = run(fb.attn_decode, fbctx, torch, d)
    got = run(fb.attn_decode_noalloc, fbctx, torch, d)
    assert_close(got, ref, what=f"noalloc at its largest batch ({b})")
    d2 = make_inputs(torch, 5, b=b + 1, nh=32, nkv=8, page=64, lens=lens + [64])
    with pytest.raises(fb.FerriteError, match="exceeds the fixed"):
        run(fb.attn_decode_noalloc, fbctx, torch, d2)
    assert fbctx.error_word() == 0
