"""GPU parity: the sm_100a library against the oracle, the golden vectors and the
reference's own CUDA kernels, always through the C ABI.

Tolerances (north star): dequantisation bit-exact; matvec relative L2 error
<= 1e-3 against the fp64-accumulated oracle.  Two activation arithmetics are
checked:
  fp32 (the default): fp32 x, fp32 products and sums, as the reference's
       kernels; only rounding order differs, so FP32_TOL = 2e-5 is asserted
       besides the contract tolerance (a single short row, whose rounding does not average out,
       reaches ~6e-6).
  int16 (opt-in): x rounded to 2^-15 of each 128-slot's largest |x|, exact
       after that (observed 2e-5 to 4e-5 over many rows of Gaussian x, up to
       ~1e-4 for a single short row); STRICT = 3e-4 is asserted besides the
       contract tolerance.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle.oracle import SEM_CUDA, SEM_GGUF_C
from trailblaze_b200 import qtypes as Q, synth

pytestmark = pytest.mark.gpu

TOL = 1e-3
STRICT = 3e-4
FP32_TOL = 2e-5
ARITH = {"fp32": 0, "int16": 1}
QUANT = [Q.Q4_K, Q.Q5_K, Q.Q6_K, Q.Q3_K, Q.Q2_K, Q.Q8_0, Q.Q4_0, Q.Q8_K]
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def torch():
    import torch as t
    return t


def dev_bytes(a: np.ndarray, offset: int = 0):
    """Copy bytes to the GPU at `offset` bytes into a fresh (512-B aligned) buffer."""
    t = torch()
    buf = t.zeros(a.size + offset + 64, dtype=t.uint8, device="cuda")
    buf[offset:offset + a.size] = t.from_numpy(np.ascontiguousarray(a)).cuda()
    return buf, buf.data_ptr() + offset


@pytest.fixture(params=["fp32", "int16"])
def arith(request, kq):
    """Runs the test under each activation arithmetic, restoring the default after."""
    prev = kq.tb_cuda_set_matvec_arith(ARITH[request.param])
    assert prev == 0
    yield request.param
    assert kq.tb_cuda_set_matvec_arith(prev) == ARITH[request.param]


def bound(arith, qt):
    """The tight bound of an arithmetic (the float types are fp32 in both)."""
    return FP32_TOL if arith == "fp32" or qt in (Q.F32, Q.F16, Q.BF16) else STRICT


def gpu_matvec(kq, qt, wptr, M, K, x):
    t = torch()
    dx = t.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    dy = t.full((M,), float("nan"), dtype=t.float32, device="cuda")
    assert kq.tb_cuda_matvec_dev(wptr, qt, M, K, dx.data_ptr(), dy.data_ptr(),
                                 t.cuda.current_stream().cuda_stream) == 1
    t.cuda.synchronize()
    assert kq.tb_cuda_last_error() == 0
    return dy.cpu().numpy()


def gpu_dequant(kq, qt, wptr, M, K, sem=0):
    t = torch()
    out = t.full((M * K,), float("nan"), dtype=t.float32, device="cuda")
    assert kq.tb_cuda_dequant_dev(wptr, qt, M, K, out.data_ptr(), sem,
                                  t.cuda.current_stream().cuda_stream) == 1
    t.cuda.synchronize()
    return out.cpu().numpy().reshape(M, K)


def rel_l2(y, ref):
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.linalg.norm(np.asarray(y, np.float64) - ref) / max(np.linalg.norm(ref), 1e-300))


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def kshape(qt, K):
    bw, _ = Q.geometry(qt)
    return K if K % bw == 0 else (K // bw) * bw or bw


# ---------------------------------------------------------------- dequantisation
DQ_SHAPES = [(1, 256), (3, 512), (17, 1024), (5, 2560)]


@pytest.mark.parametrize("qt", Q.ALL, ids=[Q.NAMES[t] for t in Q.ALL])
@pytest.mark.parametrize("M,K", DQ_SHAPES)
def test_dequant_bitexact(kq, oracle, qt, M, K):
    W = synth.weights(qt, M, K, seed=M * 7 + K, tensor=qt)
    buf, p = dev_bytes(W)
    got = gpu_dequant(kq, qt, p, M, K, 0)
    np.testing.assert_array_equal(bits(got), bits(oracle.dequant(qt, W, M, K, SEM_CUDA)))


@pytest.mark.parametrize("qt", [Q.Q4_K, Q.Q5_K])
def test_dequant_compat_semantics_bitexact(kq, oracle, qt):
    M, K = 9, 1024
    W = synth.weights(qt, M, K, seed=41, tensor=qt)
    buf, p = dev_bytes(W)
    got = gpu_dequant(kq, qt, p, M, K, 1)
    np.testing.assert_array_equal(bits(got), bits(oracle.dequant(qt, W, M, K, SEM_GGUF_C)))


@pytest.mark.parametrize("qt", Q.ALL, ids=[Q.NAMES[t] for t in Q.ALL])
def test_dequant_golden(kq, golden, qt):
    n = Q.NAMES[qt]
    M, K = (int(v) for v in golden[f"{n}/MK"])
    buf, p = dev_bytes(golden[f"{n}/W"])
    np.testing.assert_array_equal(bits(gpu_dequant(kq, qt, p, M, K, 0)), bits(golden[f"{n}/cuda_deq"]))
    if qt != Q.IQ3_S:   # the reference CPU path zeroes IQ3_S
        want = golden[f"{n}/ref_deq"]
        got = gpu_dequant(kq, qt, p, M, K, 1 if qt in (Q.Q4_K, Q.Q5_K) else 0)
        np.testing.assert_array_equal(bits(got), bits(want))


def test_dequant_kats(kq, golden):
    buf, p = dev_bytes(golden["kat/q4k_smoke_in"])
    np.testing.assert_array_equal(gpu_dequant(kq, Q.Q4_K, p, 1, 256, 0).ravel(), golden["kat/q4k_smoke_cuda"])
    np.testing.assert_array_equal(gpu_dequant(kq, Q.Q4_K, p, 1, 256, 1).ravel(), golden["kat/q4k_smoke_ref"])
    buf, p = dev_bytes(golden["kat/q8_0_in"])
    np.testing.assert_array_equal(bits(gpu_dequant(kq, Q.Q8_0, p, 1, 32).ravel()), bits(golden["kat/q8_0_ref"]))
    for tag in ("88", "FF"):
        buf, p = dev_bytes(golden[f"kat/q4_0_in{tag}"])
        np.testing.assert_array_equal(gpu_dequant(kq, Q.Q4_0, p, 1, 32).ravel(), golden[f"kat/q4_0_ref{tag}"])


# ---------------------------------------------------------------- matvec
MV_SHAPES = [(1, 256), (3, 512), (33, 768), (97, 2560), (130, 4096), (7, 12288), (300, 1024)]


@pytest.mark.parametrize("qt", Q.ALL, ids=[Q.NAMES[t] for t in Q.ALL])
@pytest.mark.parametrize("M,K", MV_SHAPES)
def test_matvec_parity(kq, oracle, arith, qt, M, K):
    W = synth.weights(qt, M, K, seed=1000 + M + K, tensor=qt)
    x = synth.activations(K, seed=M)
    buf, p = dev_bytes(W)
    y = gpu_matvec(kq, qt, p, M, K, x)
    ref = oracle.matvec_f64(qt, W, M, K, x, SEM_CUDA)
    e = rel_l2(y, ref)
    assert np.all(np.isfinite(y))
    assert e <= TOL, e
    assert e <= bound(arith, qt), e


@pytest.mark.parametrize("qt", [Q.Q4_K, Q.Q5_K, Q.Q6_K, Q.Q3_K, Q.Q2_K, Q.Q8_0, Q.Q4_0, Q.Q8_K, Q.F16, Q.F32, Q.BF16],
                         ids=lambda t: Q.NAMES[t])
@pytest.mark.parametrize("offset", [1, 2, 3, 6, 14])
def test_matvec_unaligned_base(kq, oracle, arith, qt, offset):
    """W at an arbitrary byte offset (e.g. a packed tensor sliced at a row boundary)."""
    M, K = 45, 1024
    W = synth.weights(qt, M, K, seed=77 + offset, tensor=qt)
    x = synth.activations(K, seed=offset)
    buf, p = dev_bytes(W, offset)
    e = rel_l2(gpu_matvec(kq, qt, p, M, K, x), oracle.matvec_f64(qt, W, M, K, x, SEM_CUDA))
    assert e <= bound(arith, qt), e


@pytest.mark.parametrize("qt", [Q.F32, Q.F16, Q.BF16])
@pytest.mark.parametrize("K", [1, 7, 255, 257, 1001])
def test_matvec_float_ragged_k(kq, oracle, qt, K):
    M = 19
    W = synth.weights(qt, M, K, seed=K, tensor=qt)
    x = synth.activations(K, seed=K + 1)
    buf, p = dev_bytes(W)
    e = rel_l2(gpu_matvec(kq, qt, p, M, K, x), oracle.matvec_f64(qt, W, M, K, x, SEM_CUDA))
    assert e <= STRICT, e


@pytest.mark.parametrize("qt", [Q.Q8_0, Q.Q4_0])
@pytest.mark.parametrize("K", [32, 96, 288, 2080])
def test_matvec_block32_partial_unit(kq, oracle, arith, qt, K):
    M = 23
    W = synth.weights(qt, M, K, seed=K, tensor=qt)
    x = synth.activations(K, seed=K + 2)
    buf, p = dev_bytes(W)
    e = rel_l2(gpu_matvec(kq, qt, p, M, K, x), oracle.matvec_f64(qt, W, M, K, x, SEM_CUDA))
    assert e <= bound(arith, qt), e


def test_matvec_golden(kq, golden, arith):
    for qt in Q.ALL:
        n = Q.NAMES[qt]
        M, K = (int(v) for v in golden[f"{n}/MK"])
        buf, p = dev_bytes(golden[f"{n}/W"])
        y = gpu_matvec(kq, qt, p, M, K, golden[f"{n}/x"])
        assert rel_l2(y, golden[f"{n}/cuda_mv64"]) <= bound(arith, qt), n


# ---------------------------------------------------------------- heavy-tailed activations
def outlier_x(K, seed, big=1000.0):
    """N(0,1) activations with one +-big outlier in every run of 128 (a seeded position and
    sign per run), like the few huge channels of real decode activations."""
    x = synth.activations(K, seed=seed).astype(np.float32)
    rng = np.random.default_rng(seed)
    base = np.arange(0, K, 128)
    pos = base + rng.integers(0, np.minimum(128, K - base))
    x[pos] = np.where(rng.integers(0, 2, pos.size) == 1, big, -big).astype(np.float32)
    return x, pos


def student_t_x(K, seed, dof=3):
    return np.random.default_rng(seed).standard_t(dof, K).astype(np.float32)


@pytest.mark.parametrize("qt", QUANT, ids=lambda t: Q.NAMES[t])
@pytest.mark.parametrize("dist", ["outlier", "student_t3"])
def test_matvec_heavy_tailed(kq, oracle, arith, qt, dist):
    """Heavy-tailed x against the fp64 oracle at the contract tolerance, on both arithmetics;
    the fp32 path also at its own tight bound."""
    M, K = 256, 4096
    W = synth.weights(qt, M, K, seed=61, tensor=qt)
    x = outlier_x(K, 17)[0] if dist == "outlier" else student_t_x(K, 17)
    buf, p = dev_bytes(W)
    e = rel_l2(gpu_matvec(kq, qt, p, M, K, x), oracle.matvec_f64(qt, W, M, K, x, SEM_CUDA))
    assert e <= TOL, e
    if arith == "fp32":
        assert e <= FP32_TOL, e


@pytest.mark.parametrize("qt", QUANT, ids=lambda t: Q.NAMES[t])
def test_small_activations_beside_outliers(kq, oracle, arith, qt):
    """What y's relative L2 hides: the contribution of the ordinary activations in a 128-slot
    that also holds a +-1000 outlier.  y(x) - y(outliers only), both on the GPU, against the
    fp64 matvec of the ordinary activations alone.  The fp32 path keeps it to rounding; the
    int16 path rounds every activation of such a slot to 1000 * 2^-15 (0.03), which leaves
    an error of several percent in that contribution: the documented failure mode of the
    opt-in arithmetic, asserted here so that it stays documented."""
    M, K = 256, 4096
    W = synth.weights(qt, M, K, seed=62, tensor=qt)
    x, pos = outlier_x(K, 23)
    xo = np.zeros_like(x)
    xo[pos] = x[pos]
    buf, p = dev_bytes(W)
    d = gpu_matvec(kq, qt, p, M, K, x).astype(np.float64) - gpu_matvec(kq, qt, p, M, K, xo)
    e = rel_l2(d, oracle.matvec_f64(qt, W, M, K, x - xo, SEM_CUDA))
    if arith == "fp32":
        assert e <= 1e-4, e
    else:
        assert e > TOL, e


def test_matvec_deterministic_and_scale_exact(kq, arith):
    """Run-to-run bitwise identical; x -> 2x gives exactly 2y (power-of-two scaling of x
    only moves the slot exponents, in both arithmetics)."""
    for qt in (Q.Q4_K, Q.Q6_K, Q.Q2_K, Q.Q8_0):
        M, K = 1000, 4096
        W = synth.weights(qt, M, K, seed=5, tensor=qt)
        x = synth.activations(K, seed=9)
        buf, p = dev_bytes(W)
        y1 = gpu_matvec(kq, qt, p, M, K, x)
        y2 = gpu_matvec(kq, qt, p, M, K, x)
        y3 = gpu_matvec(kq, qt, p, M, K, 2 * x)
        np.testing.assert_array_equal(bits(y1), bits(y2))
        np.testing.assert_array_equal(bits(y3), bits(2 * y1))


@pytest.mark.parametrize("qt", [Q.Q4_K, Q.Q6_K, Q.Q8_0, Q.F16], ids=lambda t: Q.NAMES[t])
def test_matvec_long_rows(kq, oracle, arith, qt):
    """Rows longer than one launch's column slots cover (K > 30720 for the fp32 decoders,
    > 15360 for F16) run as column windows; RMSNorm input, which needs the whole row's sum
    of squares, is refused there rather than computed per window.  (The windows stream
    whole rows through the ring: a row must fit half of shared memory, so F32 rows stop
    at about 28000 weights.)"""
    M, K = 40, 32768
    W = synth.weights(qt, M, K, seed=91, tensor=qt)
    x = synth.activations(K, seed=91)
    buf, p = dev_bytes(W)
    e = rel_l2(gpu_matvec(kq, qt, p, M, K, x), oracle.matvec_f64(qt, W, M, K, x, SEM_CUDA))
    assert e <= bound(arith, qt), e
    if arith == "fp32" and qt != Q.F16:
        t = torch()
        dx = t.from_numpy(x).cuda()
        nw = t.ones(K, device="cuda")
        dy = t.empty(M, device="cuda")
        assert kq.tb_cuda_matvec_fused_dev(p, qt, M, K, dx.data_ptr(), dy.data_ptr(), 1, None, nw.data_ptr(),
                                           1e-6, None, 0, 0) == 0


def test_matvec_linearity(kq):
    M, K = 2000, 2560
    qt = Q.Q5_K
    W = synth.weights(qt, M, K, seed=12, tensor=qt)
    x1, x2 = synth.activations(K, seed=1), synth.activations(K, seed=2)
    buf, p = dev_bytes(W)
    y = gpu_matvec(kq, qt, p, M, K, x1 + x2)
    ys = gpu_matvec(kq, qt, p, M, K, x1).astype(np.float64) + gpu_matvec(kq, qt, p, M, K, x2)
    # fp32: rounding only; int16: each of the three results carries its own x rounding
    # (2^-15 of a slot's max)
    assert rel_l2(y, ys) <= (FP32_TOL if kq.tb_cuda_get_matvec_arith() == 0 else STRICT)


def test_expert_slice_rows(kq, oracle):
    """MoE call site (tb_infer.c:797-827): rows of a packed expert tensor via d_data + offset."""
    qt, K, E, F = Q.Q4_K, 2048, 8, 96
    W = synth.weights(qt, E * F, K, seed=8, tensor=qt)
    x = synth.activations(K, seed=3)
    buf, p = dev_bytes(W)
    rb = Q.row_bytes(qt, K)
    for e in (0, 3, 7):
        Ws = W[e * F * rb:(e + 1) * F * rb]
        y = gpu_matvec(kq, qt, p + e * F * rb, F, K, x)
        assert rel_l2(y, oracle.matvec_f64(qt, Ws, F, K, x)) <= STRICT


# ---------------------------------------------------------------- BASELINE-size checks
def test_config1_q4k_4096(kq, oracle):
    """Q4_K 4096 x 4096 from one seed, against the fp64 oracle."""
    M = K = 4096
    W = synth.weights(Q.Q4_K, M, K, seed=1, tensor=0)
    x = synth.activations(K, seed=1)
    buf, p = dev_bytes(W)
    e = rel_l2(gpu_matvec(kq, Q.Q4_K, p, M, K, x), oracle.matvec_f64(Q.Q4_K, W, M, K, x))
    assert e <= STRICT, e


def test_lm_head_q6k_full_size(kq, oracle):
    """Largest single matvec of the sweep: Q6_K lm_head 151936 x 2560 (319.7 MB)."""
    qt, M, K = Q.Q6_K, 151936, 2560
    W = synth.weights(qt, M, K, seed=2, tensor=5)
    x = synth.activations(K, seed=2)
    buf, p = dev_bytes(W)
    y = gpu_matvec(kq, qt, p, M, K, x)
    e = rel_l2(y, oracle.matvec_f64(qt, W, M, K, x))
    assert e <= STRICT, e


# ---------------------------------------------------------------- blocking reference ABI
def test_blocking_abi_and_upload_x(kq, oracle):
    qt, M, K = Q.Q6_K, 200, 2560
    W = synth.weights(qt, M, K, seed=3, tensor=qt)
    x = synth.activations(K, seed=3)
    d = kq.tb_cuda_upload_tensor(W)
    assert d
    out = np.full(M, np.nan, dtype=np.float32)
    assert kq.tb_cuda_matvec_device(d, qt, M, K, x, out) == 1
    ref = oracle.matvec_f64(qt, W, M, K, x)
    assert rel_l2(out, ref) <= STRICT
    # device-resident x: one upload, then x_host = NULL
    assert kq.tb_cuda_upload_x(x) == 1
    out2 = np.full(M, np.nan, dtype=np.float32)
    assert kq.tb_cuda_matvec_device(d, qt, M, K, None, out2) == 1
    np.testing.assert_array_equal(bits(out), bits(out2))
    kq.tb_cuda_set_snap(None)
    kq.tb_cuda_sync_all()
    kq.tb_cuda_free_tensor(d)
    kq.tb_cuda_free_tensor(0)


def test_blocking_abi_large_y(kq):
    """A large y (70000 rows) through the blocking ABI: the same bits as the
    stream-ordered entry point, twice in a row."""
    qt, M, K = Q.Q4_K, 70000, 256
    W = synth.weights(qt, M, K, seed=4, tensor=qt)
    d = kq.tb_cuda_upload_tensor(W)
    assert d
    try:
        for call in range(2):
            x = synth.activations(K, seed=5 + call)
            out = np.full(M, np.nan, dtype=np.float32)
            assert kq.tb_cuda_matvec_device(d, qt, M, K, x, out) == 1
            np.testing.assert_array_equal(bits(out), bits(gpu_matvec(kq, qt, d, M, K, x)))
    finally:
        kq.tb_cuda_free_tensor(d)


def test_abi_rejects_bad_arguments(kq):
    W = synth.weights(Q.Q4_K, 4, 512, seed=1)
    d = kq.tb_cuda_upload_tensor(W)
    out = np.zeros(4, dtype=np.float32)
    x = np.ones(512, dtype=np.float32)
    assert kq.tb_cuda_matvec_device(d, 3, 4, 512, x, out) == 0           # unknown qtype
    assert kq.tb_cuda_matvec_device(d, Q.Q4_K, 4, 500, x[:500], out) == 0  # K % 256 != 0
    assert kq.tb_cuda_matvec_device(d, Q.Q4_K, 0, 512, x, out) == 0      # M = 0
    assert kq.tb_cuda_matvec_device(0, Q.Q4_K, 4, 512, x, out) == 0      # NULL W
    assert kq.tb_cuda_matvec_device(d, Q.Q4_K, 4, 512, x, out) == 1      # still works
    kq.tb_cuda_free_tensor(d)


def test_cleanup_and_reinit(kq, oracle):
    kq.tb_cuda_cleanup()
    kq.tb_cuda_cleanup()                      # safe twice
    assert kq.tb_cuda_init() == 1
    W = synth.weights(Q.Q2_K, 64, 1024, seed=4)
    x = synth.activations(1024, seed=4)
    buf, p = dev_bytes(W)
    assert rel_l2(gpu_matvec(kq, Q.Q2_K, p, 64, 1024, x), oracle.matvec_f64(Q.Q2_K, W, 64, 1024, x)) <= STRICT


# ---------------------------------------------------------------- failure paths (host-made)
CHILD = r"""
import sys, os, numpy as np
sys.path.insert(0, {repo!r})
from trailblaze_b200 import load, synth, qtypes as Q
k = load(); assert k.tb_cuda_init() == 1
W = synth.weights(Q.Q4_K, 64, 2048, seed=1); x = synth.activations(2048, seed=1)
mode = os.environ.get("TB_CUDA_FAULT", "")
if mode == "alloc":
    print("RESULT", k.tb_cuda_upload_tensor(W))
else:
    import torch
    buf = torch.from_numpy(W).cuda(); torch.cuda.synchronize()
    out = np.zeros(64, dtype=np.float32)
    r = k.tb_cuda_matvec_device(buf.data_ptr(), Q.Q4_K, 64, 2048, x, out)
    print("RESULT", r, k.tb_cuda_last_error())
"""


@pytest.mark.parametrize("mode,want", [("alloc", "RESULT 0"), ("copy", "RESULT 0 0"), ("launch", "RESULT 0 0")])
def test_fault_injection_returns_zero(mode, want):
    env = dict(os.environ, TB_CUDA_FAULT=mode)
    r = subprocess.run([sys.executable, "-c", CHILD.format(repo=REPO)], env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert want in r.stdout, r.stdout + r.stderr


def test_bounded_wait_reports_timeout():
    """A one-poll wait limit makes the pipeline wait run out on the first stage; the kernel
    sets the error word, lets its copies land (fixed drain limit) and returns: the call
    returns 0, the error reads 1, and the process exits cleanly."""
    env = dict(os.environ, TB_WAIT_LIMIT="1")
    r = subprocess.run([sys.executable, "-c", CHILD.format(repo=REPO)], env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    res = [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT")][0].split()
    # either every copy had landed by its first poll (no timeout), or the timeout was
    # reported through the 0 return with device error 1 (and cleared afterwards)
    if res[1] == "0":
        assert "device error 1" in r.stderr, r.stderr
    assert res[2] == "0", r.stdout


# ---------------------------------------------------------------- drop-in + reference kernels
def test_dropin_reference_host_links_unmodified():
    exe = os.path.join(REPO, "oracle", "_ref", "tb_dropin")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/tb_dropin not built")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "DROPIN PASS" in r.stdout, r.stdout + r.stderr


def test_against_reference_cuda_kernels(kq):
    """Our result vs the reference's unmodified k_*_matvec kernels built for sm_100a."""
    import ctypes
    from oracle.oracle import ReferenceCuda
    try:
        rc = ReferenceCuda()
    except FileNotFoundError:
        pytest.skip("reference CUDA library not built")
    L = rc.L
    assert L.tb_cuda_init() == 1
    fp = ctypes.POINTER(ctypes.c_float)
    for qt in (Q.Q4_K, Q.Q5_K, Q.Q6_K, Q.Q3_K, Q.Q8_0, Q.Q4_0, Q.Q8_K, Q.F16, Q.BF16, Q.F32):
        M, K = 256, 2048
        W = synth.weights(qt, M, K, seed=31, tensor=qt)
        x = synth.activations(K, seed=31)
        dref = L.tb_cuda_upload_tensor(W.ctypes.data_as(ctypes.c_void_p), W.nbytes)
        yr = np.zeros(M, dtype=np.float32)
        assert L.tb_cuda_matvec_device(dref, qt, M, K, x.ctypes.data_as(fp), yr.ctypes.data_as(fp)) == 1
        buf, p = dev_bytes(W)
        y = gpu_matvec(kq, qt, p, M, K, x)
        assert rel_l2(y, yr) <= TOL, Q.NAMES[qt]
        L.tb_cuda_free_tensor(dref)
