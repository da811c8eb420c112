"""Device sampling (fb_sample) against the CPU restatement of the reference
sampler (oracle/sampling.py).

* Against the same rules with binary64 sums (the device's arithmetic): the
  same token and RNG state for every draw, over the reference's default
  config and variations of each filter, at a Qwen3-size vocabulary and a
  small one, on wide distributions (thousands of tokens inside top-p).
* Against the reference's own f32 left-to-right sums: the same tokens when a
  few tokens hold most of the mass (the reference's f32 running sums then
  stay clear of the boundaries; on wide distributions they drift by ~1e-4,
  which moves its top-p and draw boundaries across low-probability tokens).
"""
import numpy as np
import pytest

import ferrite_b200 as fb
from oracle import sampling as S

pytestmark = pytest.mark.gpu

CONFIGS = [
    dict(),  # reference defaults: T 0.7, top_p 0.9, min_p 0.05, rep 1.1
    dict(temperature=0.0),
    dict(temperature=1.0, top_p=1.0, min_p=0.0, top_k=40, repetition_penalty=1.0),
    dict(temperature=1.0, top_p=0.95, min_p=0.0, repetition_penalty=1.0),
    dict(temperature=1.3, top_p=1.0, min_p=0.1, repetition_penalty=1.3),
    dict(temperature=1.5, top_p=0.8, top_k=100, min_p=0.02, repetition_penalty=1.2),
    dict(temperature=0.5, top_p=0.5, top_k=3, min_p=0.0, repetition_penalty=1.0),
]


def run(fbctx, torch, vocab, ci, sums, scale, boost):
    cfg = dict(temperature=0.7, top_p=0.9, top_k=0, min_p=0.05, repetition_penalty=1.1, seed=42)
    cfg.update(CONFIGS[ci])
    rng = np.random.default_rng(vocab + ci)
    dev = fb.Sampler(fbctx, **cfg)
    ref = S.Sampler(**cfg, sums=sums)
    prev = list(rng.integers(0, vocab, 40))
    mism = []
    for step in range(12):
        x = rng.normal(0, scale, vocab).astype(np.float32)
        x[rng.integers(0, vocab, 3)] += boost
        xd = torch.from_numpy(x).cuda()
        got = dev.sample(xd.data_ptr(), vocab, prev)
        want = ref.sample(x, prev)
        assert dev.state.value == ref.state, f"rng state differs at step {step}"
        if got != want:
            mism.append((step, got, want))
        prev.append(want)
    return mism


@pytest.mark.parametrize("vocab", [151936, 4096])
@pytest.mark.parametrize("ci", range(len(CONFIGS)))
def test_sample_matches_rules_f64(fbctx, torch_cuda, vocab, ci):
    mism = run(fbctx, torch_cuda, vocab, ci, "f64", 2.5, 8.0)
    assert not mism, f"draws differ (step, device, oracle): {mism}"


@pytest.mark.parametrize("ci", range(len(CONFIGS)))
def test_sample_matches_reference_f32_concentrated(fbctx, torch_cuda, ci):
    mism = run(fbctx, torch_cuda, 151936, ci, "f32", 1.0, 14.0)
    assert not mism, f"draws differ (step, device, oracle): {mism}"


@pytest.mark.parametrize("vocab,k,rows", [(151936, 16, 1), (151936, 5, 3), (128256, 16, 2), (37, 16, 1), (10, 16, 1),
                                          (4096, 1, 1)])
def test_top_logits_matches_hook_order(fbctx, torch_cuda, vocab, k, rows):
    """fb_top_logits against the restated hook candidate list (stable
    descending sort): ties of the top value across chunks, repeated values
    inside one chunk, +-0.0, -inf entries, and rows shorter than k."""
    torch = torch_cuda
    rng = np.random.default_rng(vocab + k + rows)
    x = rng.normal(0, 3, (rows, vocab)).astype(np.float32)
    for r in range(rows):
        top = float(x[r].max())
        # the row maximum repeated at indices in different 2048-value chunks
        for i in rng.choice(vocab, min(vocab, 5), replace=False):
            x[r, i] = top
        # a run of equal values inside one chunk, and signed zeros
        j = int(rng.integers(0, max(1, vocab - 8)))
        x[r, j:j + 6] = top - 0.25 if vocab > 8 else x[r, j:j + 6]
        x[r, rng.integers(0, vocab)] = -np.inf
    if vocab > 2:
        x[0, 0], x[0, 1] = -0.0, 0.0
    xd = torch.from_numpy(x).cuda()
    ids = torch.full((rows, k), -7, dtype=torch.int32, device="cuda")
    vals = torch.zeros((rows, k), dtype=torch.float32, device="cuda")
    fb.top_logits(fbctx, xd.data_ptr(), rows, vocab, k, ids.data_ptr(), vals.data_ptr())
    torch.cuda.synchronize()
    gi, gv = ids.cpu().numpy(), vals.cpu().numpy()
    for r in range(rows):
        want = S.top_logits_candidates(x[r], k)
        n = len(want)
        assert gi[r, :n].tolist() == [i for i, _ in want], f"row {r}"
        assert np.array_equal(gv[r, :n], np.array([v for _, v in want], np.float32))
        assert (gi[r, n:] == -1).all() and np.isneginf(gv[r, n:]).all()
    with pytest.raises(fb.FerriteError):
        fb.top_logits(fbctx, xd.data_ptr(), rows, vocab, 17, ids.data_ptr(), vals.data_ptr())
