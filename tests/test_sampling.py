"""The CPU restatement of the reference sampler (oracle/sampling.py):
greedy and top-k = 1 pick the (penalized) argmax, the xorshift64 stream,
filters keep what the reference's rules keep, and empirical frequencies of
many draws follow the filtered softmax."""
import numpy as np

from oracle import sampling as S


def test_xorshift_stream():
    st, seq = 42, []
    for _ in range(3):
        st, r = S.xorshift64(st)
        seq.append(st)
        assert 0.0 <= r <= 1.0
    # three steps of x ^= x << 13; x ^= x >> 7; x ^= x << 17 from 42
    m = (1 << 64) - 1
    x = 42
    for want in seq:
        x ^= (x << 13) & m
        x ^= x >> 7
        x ^= (x << 17) & m
        assert x == want


def test_greedy_and_penalty():
    rng = np.random.default_rng(0)
    x = rng.normal(0, 2, 1000).astype(np.float32)
    top = int(np.argmax(x))
    assert S.Sampler(temperature=0.0, repetition_penalty=1.0).sample(x) == top
    # penalizing the argmax (positive logit divided) can move the argmax
    y = x.copy()
    y[top] = y[top] / np.float32(5.0)
    want = int(np.argmax(y))
    got = S.Sampler(temperature=0.0, repetition_penalty=5.0).sample(x, [top, top, 99999])
    assert got == want
    assert S.Sampler(temperature=1.0, top_k=1, min_p=0.0, top_p=1.0, repetition_penalty=1.0).sample(x) == top


def test_empirical_frequencies():
    x = np.linspace(-2, 2, 16).astype(np.float32)
    sm = S.Sampler(temperature=1.0, top_p=1.0, top_k=0, min_p=0.0, repetition_penalty=1.0, seed=7)
    n = 20000
    counts = np.bincount([sm.sample(x) for _ in range(n)], minlength=16) / n
    p = np.exp(x - x.max())
    p /= p.sum()
    assert np.abs(counts - p).max() < 0.015


def test_top_p_keeps_crossing_token():
    p = np.log(np.array([0.5, 0.3, 0.15, 0.05], dtype=np.float32))
    sm = S.Sampler(temperature=1.0, top_p=0.7, top_k=0, min_p=0.0, repetition_penalty=1.0, seed=1)
    seen = {sm.sample(p) for _ in range(400)}
    assert seen == {0, 1}  # 0.5 < 0.7 keeps token 1 as well; 0.8 >= 0.7 stops


def test_top_logits_candidates_stable_order():
    """The hook's candidate list (hooks.rs:19-38): descending logits, equal
    logits in index order, limit 0 taken as 1, a short row returns it all."""
    x = np.array([0.5, 2.0, -1.0, 2.0, 0.5, -0.0, 0.0, 3.0], dtype=np.float32)
    got = S.top_logits_candidates(x, 6)
    assert [i for i, _ in got] == [7, 1, 3, 0, 4, 5]
    assert S.top_logits_candidates(x, 0) == [(7, 3.0)]
    assert len(S.top_logits_candidates(x, 16)) == x.size
    # -0.0 and 0.0 compare equal: index order
    assert [i for i, _ in S.top_logits_candidates(np.array([-0.0, 0.0], np.float32), 2)] == [0, 1]
    rng = np.random.default_rng(3)
    y = rng.normal(0, 1, 5000).astype(np.float32)
    want = np.argsort(-y, kind="stable")[:16]
    assert [i for i, _ in S.top_logits_candidates(y, 16)] == list(want)
