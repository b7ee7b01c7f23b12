"""The oracle's router restatement (tb_route_experts, layer4/tb_infer.c:351-374)
on hand-checked cases: softmax, the replace-the-first-minimum scan (ties keep
the earlier expert unless a larger one evicts it first), and the weights
renormalised over the selected experts."""
import numpy as np

from oracle.decode_ref import route


def test_route_topk_and_weights():
    logits = np.array([0.5, 2.0, -1.0, 1.5, 3.0])
    idx, w = route(logits, 2)
    p = np.exp(logits - logits.max())
    p /= p.sum()
    assert sorted(idx) == [1, 4]
    assert np.isclose(sum(w), 1.0)
    assert np.isclose(w[idx.index(4)], p[4] / (p[4] + p[1]))


def test_route_scan_order_and_ties():
    # slots after experts 0, 1: [e0, e1]; expert 2 evicts the first smallest slot (slot 0)
    idx, w = route(np.array([5.0, 5.0, 7.0]), 2)
    assert idx == [2, 1]
    # an equal probability does not displace the expert already held
    idx, _ = route(np.array([1.0, 3.0, 3.0]), 1)
    assert idx == [1]
    # k = E keeps every expert, weights = the softmax itself
    lg = np.array([0.1, -0.3, 0.7])
    idx, w = route(lg, 3)
    p = np.exp(lg - lg.max())
    p /= p.sum()
    assert sorted(idx) == [0, 1, 2]
    assert np.allclose([w[idx.index(e)] for e in range(3)], p)
