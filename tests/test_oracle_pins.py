"""CPU: pin the oracle (tb_oracle.c) against the reference's own code and golden vectors.

The reference routines are compiled from its sources into oracle/_ref/; the
golden fixtures were produced by them (tests/golden/make_golden.py).
"""
import numpy as np
import pytest

from oracle.oracle import SEM_CUDA, SEM_DISPATCH, SEM_GGUF_C
from trailblaze_b200 import qtypes as Q, synth

CPU_TYPES = [t for t in Q.ALL if t != Q.IQ3_S]   # the reference CPU path zeroes IQ3_S


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


# ---- known-answer tests of the reference self-test (tb_gguf.c:995-1092) ----------------
def test_kat_converters(oracle, golden):
    assert oracle.h2f(0x3C00) == 1.0 and oracle.h2f(0xBC00) == -1.0
    assert oracle.bf2f(0x4000) == 2.0
    np.testing.assert_array_equal(golden["kat/f16_ref"], [1.0, -1.0])
    np.testing.assert_array_equal(golden["kat/bf16_ref"], [2.0])


def test_kat_fp16_subnormal_quirk(oracle):
    # tb_gguf.c:97 maps exponent 0 to sign|m<<13: m*2^-136, not m*2^-24
    assert oracle.h2f(0x0001) == np.float32(2.0 ** -136)
    assert oracle.h2f(0x8001) == -np.float32(2.0 ** -136)
    assert np.isinf(oracle.h2f(0x7C00)) and np.isnan(oracle.h2f(0x7E00))


def test_kat_q8_0_q4_0(oracle, golden):
    q8 = golden["kat/q8_0_in"]
    d = oracle.dequant(Q.Q8_0, q8, 1, 32).ravel()
    np.testing.assert_array_equal(bits(d), bits(golden["kat/q8_0_ref"]))
    assert d[0] == np.float32(oracle.h2f(0x2E66))
    for tag, want in (("88", 0.0), ("FF", 7.0)):
        out = oracle.dequant(Q.Q4_0, golden[f"kat/q4_0_in{tag}"], 1, 32).ravel()
        np.testing.assert_array_equal(bits(out), bits(golden[f"kat/q4_0_ref{tag}"]))
        assert out[0] == want


def test_kat_q4k_smoke_divergence(oracle, golden):
    """Documented divergence: d=1, dmin=0, scale bytes 0x01, nibbles 8."""
    blk = golden["kat/q4k_smoke_in"]
    gguf_c = oracle.dequant(Q.Q4_K, blk, 1, 256, SEM_GGUF_C).ravel()
    cuda = oracle.dequant(Q.Q4_K, blk, 1, 256, SEM_CUDA).ravel()
    np.testing.assert_array_equal(bits(gguf_c), bits(golden["kat/q4k_smoke_ref"]))
    assert np.all(gguf_c == 8.0)
    assert np.all(cuda[:128] == 8.0) and np.all(cuda[128:] == 32.0)
    np.testing.assert_array_equal(bits(cuda), bits(golden["kat/q4k_smoke_cuda"]))


# ---- bit-exact pins against the reference routines ---------------------------------------
@pytest.mark.parametrize("qt", CPU_TYPES, ids=[Q.NAMES[t] for t in CPU_TYPES])
def test_dequant_matches_tb_gguf_dequant_row(oracle, reference, qt):
    M, K = 7, 1024
    W = synth.weights(qt, M, K, seed=99, tensor=qt)
    rb = Q.row_bytes(qt, K)
    ref = np.stack([reference.dequant_row(qt, W[m * rb:(m + 1) * rb], K) for m in range(M)])
    got = oracle.dequant(qt, W, M, K, SEM_GGUF_C)
    np.testing.assert_array_equal(bits(got), bits(ref))


@pytest.mark.parametrize("qt", CPU_TYPES, ids=[Q.NAMES[t] for t in CPU_TYPES])
def test_matvec_loop_matches_tb_gguf_dequant_matvec(oracle, reference, qt):
    M, K = 9, 512
    W = synth.weights(qt, M, K, seed=5, tensor=qt)
    x = synth.activations(K, seed=6)
    ref = reference.dequant_matvec(qt, W, M, K, x)
    got = oracle.matvec_f32_seq(qt, W, M, K, x, SEM_GGUF_C)
    np.testing.assert_array_equal(bits(got), bits(ref))


@pytest.mark.parametrize("qt,name", [(Q.Q4_K, "tb_dot_q4k_scalar"), (Q.Q3_K, "tb_dot_q3k_scalar")])
def test_cuda_scale_unpack_pinned_by_dispatch_scalar(oracle, reference, qt, name):
    """tb_dot_q4k/q3k_scalar use the CUDA kernels' scale unpack (tb_analog_dispatch.c:204-220)
    with bf16-read d/dmin; the oracle's SEM_DISPATCH is SEM_CUDA with only that converter
    swapped, so equality pins the CUDA-semantics unpack and nibble order bit for bit."""
    K = 2048
    W = synth.weights(qt, 4, K, seed=17, tensor=qt)
    x = synth.activations(K, seed=18)
    rb = Q.row_bytes(qt, K)
    for m in range(4):
        row = W[m * rb:(m + 1) * rb]
        ref = np.float32(reference.dot_scalar(name, row, K, x))
        got = oracle.matvec_f32_seq(qt, row, 1, K, x, SEM_DISPATCH)[0]
        assert bits(np.array([got]))[0] == bits(np.array([ref]))[0]


def test_q8_0_dispatch_scalar(oracle, reference):
    """tb_dot_q8_scalar reads d as fp16 with an IEEE converter; for normal scales it equals
    the oracle's product order d*q*x accumulated sequentially in fp32."""
    K = 1024
    W = synth.weights(Q.Q8_0, 2, K, seed=3, tensor=8)
    x = synth.activations(K, seed=4)
    w = oracle.dequant(Q.Q8_0, W, 2, K, SEM_CUDA)
    rb = Q.row_bytes(Q.Q8_0, K)
    for m in range(2):
        ref = reference.dot_scalar("tb_dot_q8_scalar", W[m * rb:(m + 1) * rb], K, x)
        assert abs(ref - float(np.dot(w[m].astype(np.float64), x))) <= 1e-5 * np.abs(w[m] * x).sum()


# ---- golden fixtures ---------------------------------------------------------------
@pytest.mark.parametrize("qt", Q.ALL, ids=[Q.NAMES[t] for t in Q.ALL])
def test_oracle_reproduces_golden(oracle, golden, qt):
    n = Q.NAMES[qt]
    M, K = (int(v) for v in golden[f"{n}/MK"])
    W, x = golden[f"{n}/W"], golden[f"{n}/x"]
    np.testing.assert_array_equal(bits(oracle.dequant(qt, W, M, K, SEM_CUDA)), bits(golden[f"{n}/cuda_deq"]))
    np.testing.assert_array_equal(oracle.matvec_f64(qt, W, M, K, x, SEM_CUDA), golden[f"{n}/cuda_mv64"])
    if qt != Q.IQ3_S:
        np.testing.assert_array_equal(bits(oracle.dequant(qt, W, M, K, SEM_GGUF_C)), bits(golden[f"{n}/ref_deq"]))
        np.testing.assert_array_equal(bits(oracle.matvec_f32_seq(qt, W, M, K, x, SEM_GGUF_C)),
                                      bits(golden[f"{n}/ref_mv"]))


def test_cuda_and_gguf_c_semantics_differ_only_for_q4k_q5k(golden):
    for qt in CPU_TYPES:
        n = Q.NAMES[qt]
        same = np.array_equal(bits(golden[f"{n}/cuda_deq"]), bits(golden[f"{n}/ref_deq"]))
        assert same == (qt not in (Q.Q4_K, Q.Q5_K)), n


def test_iq3s_is_q3k_alias(oracle):
    W = synth.weights(Q.Q3_K, 2, 512, seed=1)
    a = oracle.dequant(Q.IQ3_S, W, 2, 512, SEM_CUDA)
    b = oracle.dequant(Q.Q3_K, W, 2, 512, SEM_CUDA)
    np.testing.assert_array_equal(bits(a), bits(b))
