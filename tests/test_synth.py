"""CPU: the synthetic generators are seeded, counter-based and shaped like the configs."""
import numpy as np

from trailblaze_b200 import qtypes as Q, synth


def test_deterministic_and_seed_sensitive():
    a = synth.weights(Q.Q4_K, 8, 512, seed=1)
    b = synth.weights(Q.Q4_K, 8, 512, seed=1)
    c = synth.weights(Q.Q4_K, 8, 512, seed=2)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert a.size == Q.matrix_bytes(Q.Q4_K, 8, 512)


def test_counter_based_prefix():
    long = synth.u64(5, 3, 1000)
    part = synth.u64(5, 3, 100, start=400)
    assert np.array_equal(long[400:500], part)


def test_scale_distribution_q4k():
    W = synth.weights(Q.Q4_K, 4096, 1024, seed=0).reshape(-1, 144)
    d = W[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    assert np.all(d >= 0)
    assert 0.006 < float(np.mean(d)) < 0.010      # E|N(0,1)|*0.01 = 0.00798
    sub = np.mean(d < 6.104e-5)                    # fp16 subnormals (reference converter quirk)
    assert 0.002 < sub < 0.01


def test_activations_normal():
    x = synth.activations(1 << 16, seed=3)
    assert x.dtype == np.float32
    assert abs(float(x.mean())) < 0.02 and abs(float(x.std()) - 1) < 0.02
