"""GPU parity of the device sampler (tb_cuda_sample_dev) against the oracle's
restatement of tb_sample_top_p / tb_sample_top_k (oracle/sample_ref.py, itself
pinned to the reference's code in tests/test_sample_oracle.py): the same
token for the same logits and the same uniform variate u, at the lm_head's
vocabulary size and smaller; non-finite logits and bad arguments."""
import ctypes

import numpy as np
import pytest

from oracle import sample_ref as S

pytestmark = pytest.mark.gpu


def _sample(kq, lg, k, p, t, u):
    import torch
    d = torch.from_numpy(np.ascontiguousarray(lg, dtype=np.float32)).cuda()
    tok = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    r = kq.L.tb_cuda_sample_dev(ctypes.c_void_p(d.data_ptr()), lg.size, k, p, t, u, ctypes.c_void_p(tok.data_ptr()),
                                None)
    torch.cuda.synchronize()
    return r, int(tok.item())


@pytest.mark.parametrize("case", range(16))
def test_top_p_matches_oracle(kq, case):
    rng = np.random.default_rng(300 + case)
    V = [151936, 1000, 32000, 77][case % 4]
    lg = (rng.standard_normal(V) * [1.0, 2.0, 4.0][case % 3]).astype(np.float32)
    p, t = [0.9, 0.5, 0.99, 1.0][case % 4], [1.0, 0.7, 1.3, 0.005][(case // 4) % 4]
    u = float(rng.random())
    r, tok = _sample(kq, lg, 0, p, t, u)
    assert r == 1 and kq.L.tb_cuda_last_error() == 0
    assert tok == S.sample_top_p(lg, p, t, u), (V, p, t, u)


@pytest.mark.parametrize("case", range(16))
def test_top_k_matches_oracle(kq, case):
    rng = np.random.default_rng(400 + case)
    V = [151936, 1000, 8000, 300][case % 4]
    lg = (rng.standard_normal(V) * 2).astype(np.float32)
    k = [1, 5, 40, 2048, V + 5][case % 5]   # the last: k >= vocab, the nucleus fallback
    t = [1.0, 0.8, 0.0, 1.5][(case // 4) % 4]
    u = float(rng.random())
    r, tok = _sample(kq, lg, k, 0.0, t, u)
    assert r == 1 and kq.L.tb_cuda_last_error() == 0
    assert tok == S.sample_top_k(lg, k, t, u), (V, k, t, u)


def test_top_k_equal_logits_by_lower_index(kq):
    lg = np.zeros(5000, dtype=np.float32)
    lg[[17, 900, 4000]] = 3.0            # three equal largest values
    for u in (0.0, 0.5, 0.999):
        r, tok = _sample(kq, lg, 2, 0.0, 1.0, u)   # the two lower indices, equal weights
        assert r == 1 and tok == S.sample_top_k(lg, 2, 1.0, u) and tok in (17, 900)


def test_sample_rejects_and_reports(kq):
    lg = np.random.default_rng(1).standard_normal(5000).astype(np.float32)
    assert _sample(kq, lg, 6000, 0.0, 1.0, 0.5)[0] == 1    # k >= vocab: the nucleus fallback
    assert _sample(kq, lg, 3000, 0.0, 1.0, 0.5)[0] == 0    # 2048 < k < vocab: refused
    assert _sample(kq, lg, 5, 0.0, 1.0, 1.0)[0] == 0       # u outside [0, 1)
    assert _sample(kq, lg, 5, 0.0, 1.0, -0.1)[0] == 0
    assert _sample(kq, lg, 0, 0.0, 1.0, 0.5)[0] == 0       # nucleus needs 0 < p <= 1
    assert _sample(kq, lg, 0, 1.5, 1.0, 0.5)[0] == 0
    assert kq.L.tb_cuda_last_error() == 0
    bad = lg.copy()
    bad[123] = np.nan
    r, tok = _sample(kq, bad, 0, 0.9, 1.0, 0.5)
    assert r == 1 and tok == 0
    assert kq.L.tb_cuda_last_error() == 2                  # reported once, then cleared
    assert kq.L.tb_cuda_last_error() == 0


@pytest.mark.parametrize("k", [40, 2048])
@pytest.mark.parametrize("bad", [np.nan, np.inf])
def test_top_k_non_finite_reported_once(kq, k, bad):
    """Top-k checks finiteness inside its first radix pass: a NaN or +Inf logit gives
    token 0 and the error word 2, reported once."""
    lg = np.random.default_rng(5).standard_normal(151936).astype(np.float32)
    lg[77777] = bad
    r, tok = _sample(kq, lg, k, 0.0, 1.0, 0.3)
    assert r == 1 and tok == 0
    assert kq.L.tb_cuda_last_error() == 2
    assert kq.L.tb_cuda_last_error() == 0


def test_sampled_decode_step_non_finite_logits(kq):
    """A sampled decode step whose logits are not finite (an output norm of inf) reports
    the error word through the step's 0 return, and the next call works again."""
    import torch
    from test_gpu_decode import GpuDecoder, make_model
    m = make_model(n_layers=1, hidden=256, nh=2, nk=1, ffn=256, vocab=512, max_ctx=16, seed=4)
    m.out_norm = np.full(m.hidden, np.inf, dtype=np.float32)
    g = GpuDecoder(kq, m, quirks=True)
    try:
        assert kq.L.tb_cuda_dec_set_sampling(g.d, 1.0, 40, 0.0) == 1
        u = np.array([0.25], dtype=np.float32)
        toks = (ctypes.c_int * 1)()
        fp = ctypes.POINTER(ctypes.c_float)
        assert kq.L.tb_cuda_dec_generate_u(g.d, 1, 0, 1, u.ctypes.data_as(fp), toks, None, None) == 0
        assert kq.L.tb_cuda_last_error() == 0          # the step's own error word was read and cleared
        torch.cuda.synchronize()
    finally:
        kq.L.tb_cuda_dec_destroy(g.d)
