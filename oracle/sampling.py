"""CPU restatement of the reference sampler (test infrastructure only).

Follows crates/ferrite-core/src/sampling.rs:61-239 step by step in f32:
repetition penalty on the distinct previous tokens below vocab (candle's
scalar division / multiplication as affine x * (1/p) + 0 / x * p + 0, then
index_add of pen - x), temperature == 0 -> first index of the maximum,
scaling x * (1/T) + 0, softmax (max, exp, left-to-right f32 sum, divide),
min-p (keep p >= min_p * max_p), top-p (stable descending sort, keep while
the running f32 sum is below top_p), top-k (stable descending sort, first
k), each followed by a left-to-right f32 renormalization, and the draw with
the reference's xorshift64 state and f32 uniform (first index whose running
f32 sum exceeds r, else the last nonzero index).

sums="f64" applies the same rules with binary64 sums (softmax and
renormalization sums, the top-p running sum, the draw's cumulative sum) and
f32 results rounded once: the device sampler's arithmetic.  The two agree
whenever the reference's f32 running sums stay clear of a boundary -- e.g.
when a few tokens hold the mass -- but a wide distribution (thousands of
tokens kept by top-p) accumulates f32 rounding of ~1e-4 in the reference's
running sums, which moves its boundaries by many low-probability tokens.

Parity is unpinned: the reference has no tests or vectors for the sampler
and its Rust toolchain is absent here.
"""
from __future__ import annotations

import numpy as np

F = np.float32


def _seq_sum(x: np.ndarray) -> np.float32:
    # left-to-right f32 accumulation (Iterator::sum over f32)
    return np.cumsum(x, dtype=F)[-1] if x.size else F(0)


def _renorm(p: np.ndarray, f64: bool = False) -> np.ndarray:
    if f64:
        s = float(np.sum(p.astype(np.float64)))
        return (p.astype(np.float64) / s).astype(F) if s > 0 else p
    s = _seq_sum(p)
    return (p / s).astype(F) if s > 0 else p


def xorshift64(state: int) -> tuple[int, float]:
    m = (1 << 64) - 1
    state ^= (state << 13) & m
    state ^= state >> 7
    state ^= (state << 17) & m
    return state, float(F(state) / F(m))


class Sampler:
    def __init__(self, temperature=0.7, top_p=0.9, top_k=0, min_p=0.05, repetition_penalty=1.1, seed=42,
                 sums: str = "f32"):
        self.f64 = sums == "f64"
        self.temperature, self.top_p, self.top_k = float(temperature), float(top_p), int(top_k)
        self.min_p, self.rep = F(min_p), F(repetition_penalty)
        self.state = int(seed)

    def sample(self, logits: np.ndarray, previous_tokens=()) -> int:
        x = np.asarray(logits, dtype=F).copy()
        V = x.size
        if self.rep != F(1.0) and len(previous_tokens):
            toks = sorted({int(t) for t in previous_tokens if 0 <= int(t) < V})
            inv = F(1.0 / float(self.rep))
            for t in toks:
                v = x[t]
                pen = F(v * inv + F(0)) if v > 0 else F(v * self.rep + F(0))
                x[t] = F(v + F(pen - v))
        if self.temperature == 0.0:
            return int(np.argmax(x))
        s = (x * F(1.0 / self.temperature) + F(0)).astype(F)
        e = np.exp((s - s.max()).astype(F)).astype(F)
        p = _renorm(e, self.f64) if self.f64 else (e / _seq_sum(e)).astype(F)
        if self.min_p > 0:
            thr = F(self.min_p * p.max())
            p = np.where(p >= thr, p, F(0)).astype(F)
            p = _renorm(p, self.f64)
        if self.top_p < 1.0:
            order = np.argsort(-p, kind="stable")
            keep = np.zeros(V, dtype=bool)
            if self.f64:
                run = np.cumsum(p[order].astype(np.float64))
                before = np.concatenate([[0.0], run[:-1]])
                keep[order[before < float(F(self.top_p))]] = True
            else:
                cum, tp = F(0), F(self.top_p)
                for i in order:
                    if cum < tp:
                        keep[i] = True
                        cum = F(cum + p[i])
                    else:
                        break
            p = _renorm(np.where(keep, p, F(0)).astype(F), self.f64)
        if self.top_k > 0:
            order = np.argsort(-p, kind="stable")
            keep = np.zeros(V, dtype=bool)
            keep[order[: self.top_k]] = True
            p = _renorm(np.where(keep, p, F(0)).astype(F), self.f64)
        self.state, r = xorshift64(self.state)
        cum = np.cumsum(p.astype(np.float64)) if self.f64 else np.cumsum(p, dtype=F)
        hit = np.nonzero((float(r) if self.f64 else F(r)) < cum)[0]
        if hit.size:
            return int(hit[0])
        nz = np.nonzero(p > 0)[0]
        return int(nz[-1]) if nz.size else 0


def top_logits_candidates(logits: np.ndarray, limit: int):
    """Restates crates/ferrite-core/src/hooks.rs:19-38 for finite logits:
    (index, value) pairs sorted by descending logit with a stable sort (equal
    logits keep index order), the first max(limit, 1) of them.  Written as a
    stable merge sort (Python's sorted), the same kind of sort as Rust's
    slice::sort_by, on the key -logit."""
    x = np.asarray(logits, dtype=np.float32).reshape(-1)
    order = sorted(range(x.size), key=lambda i: -float(x[i]))
    take = order[: max(int(limit), 1)]
    return [(int(i), float(x[i])) for i in take]
