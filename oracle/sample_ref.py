"""CPU restatement of the reference's samplers (TEST INFRASTRUCTURE ONLY).

numpy, fp32 arithmetic with sequential sums, as layer1/tb_tensor.c does:

  tb_sample_top_p  tb_tensor.c:436-504  softmax of logits / t (t = temperature
                   when > 0.01, else 1), candidates >= 1e-4 of the peak
                   probability in index order (at most 2047), sorted largest
                   first by a stable sort (the reference's insertion sort keeps
                   equal probabilities in index order), cut after the first
                   prefix whose sum reaches p, r = u * (sum of the kept), the
                   first kept candidate whose running sum reaches r
  tb_sample_top_k  tb_tensor.c:506-540  k >= vocab: top_p(0.95); else the k
                   largest logits (equal values by lower index here; the
                   reference's selection sort differs only among equal values),
                   softmax of (l - l_max) / t (t = temperature when > 0, else
                   1), r = u * sum, first whose running sum reaches r

u stands for the reference's rand() / ((float)RAND_MAX + 1.0f).

Only tests/ use this module; the shipped library never does.
"""
from __future__ import annotations

import numpy as np

F = np.float32


def _first_reaching(cum: np.ndarray, target) -> int:
    hit = np.nonzero(cum >= target)[0]
    return int(hit[0]) if hit.size else -1


def sample_top_p(logits, p: float, temperature: float, u: float) -> int:
    t = F(temperature) if temperature > 0.01 else F(1.0)
    lg = np.asarray(logits, dtype=F)
    m = lg.max()
    probs = np.exp((lg - m) / t).astype(F)
    s = np.cumsum(probs, dtype=F)[-1]
    inv = F(1.0) / s if s > 0 else F(1.0)
    probs = (probs * inv).astype(F)
    thr = probs.max() * F(1e-4)
    cand = np.nonzero(probs >= thr)[0][:2047]
    if cand.size == 0:
        return 0
    cp = probs[cand]
    order = np.argsort(-cp, kind="stable")
    cp, ci = cp[order], cand[order]
    cut = _first_reaching(np.cumsum(cp, dtype=F), F(p))
    if cut < 0:
        cut = cp.size - 1
    kept = cp[:cut + 1]
    acc = np.cumsum(kept, dtype=F)
    r = F(u) * acc[-1]
    j = _first_reaching(acc, r)
    return int(ci[j] if j >= 0 else ci[cut])


def sample_top_k(logits, k: int, temperature: float, u: float) -> int:
    lg = np.asarray(logits, dtype=F)
    if k >= lg.size:
        return sample_top_p(lg, 0.95, temperature, u)
    t = F(temperature) if temperature > 0 else F(1.0)
    top = np.argsort(-lg, kind="stable")[:k]
    v = lg[top]
    e = np.exp((v - v[0]) / t).astype(F)
    acc = np.cumsum(e, dtype=F)
    r = F(u) * acc[-1]
    j = _first_reaching(acc, r)
    return int(top[j] if j >= 0 else top[0])
