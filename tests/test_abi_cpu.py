"""CPU: the C-ABI library loads and exports every symbol include/*.h declares.

No compute call runs here (there is no GPU); only host-only entry points are
called.
"""
import os
import re
import subprocess

import numpy as np
import pytest

from trailblaze_b200 import qtypes as Q
from trailblaze_b200._lib import LIB_PATH, exported_symbols, lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "tb_gguf_dequant.h")

# reference ABI, layer4/tb_gguf_dequant.h:19-43
REFERENCE_SYMBOLS = ["tb_cuda_init", "tb_cuda_upload_tensor", "tb_cuda_free_tensor", "tb_cuda_upload_x",
                     "tb_cuda_set_snap", "tb_cuda_matvec_device", "tb_cuda_sync_all", "tb_cuda_cleanup"]


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tb_cuda_\w+)\s*\(", src)))


def dynamic_symbols():
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True, text=True, check=True)
    return {ln.split()[-1] for ln in out.stdout.splitlines() if " T " in ln}


def test_library_built_for_sm100a():
    from trailblaze_b200 import build
    assert os.path.exists(LIB_PATH)
    assert "arch=compute_100a,code=sm_100a" in build.NVCC_FLAGS
    assert "-use_fast_math" not in build.NVCC_FLAGS and "--ftz=true" not in build.NVCC_FLAGS


def test_header_symbols_exported():
    declared = header_functions()
    exported = dynamic_symbols()
    assert set(REFERENCE_SYMBOLS) <= set(declared)
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    assert sorted(exported_symbols()) == declared


def test_library_loads_and_host_only_calls():
    L = lib()
    assert L.tb_cuda_version().decode().startswith("tb_cuda_sm100")
    from trailblaze_b200.kquant import KQuantLib
    k = KQuantLib()
    for qt in Q.ALL:
        assert k.tb_cuda_qtype_info(qt) == Q.geometry(qt)
    assert k.tb_cuda_qtype_info(3) is None
    assert k.tb_cuda_launch_count() == 0


def test_no_cpu_fallback_in_product():
    """The product package never imports the oracle, and the library has no host compute path."""
    pkg = os.path.join(REPO, "trailblaze_b200")
    for root, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                text = open(os.path.join(root, f)).read()
                assert "oracle" not in text.replace("Oracle", "").lower() or f == "__init__.py", f


def test_fastdiv_formula():
    """Host restatement of tb_common.cuh's make_fastdiv/fdiv, exhaustive on edges."""
    def make(d):
        l = 0
        while (1 << l) < d:
            l += 1
        m = ((1 << 32) * ((1 << l) - d)) // d + 1
        return d, m & 0xFFFFFFFF, l

    def div(n, f):
        d, m, s = f
        if d == 1:
            return n
        t = (n * m) >> 32
        return (t + ((n - t) >> 1)) >> (s - 1)

    rng = np.random.default_rng(0)
    for d in list(range(1, 300)) + [593, 1187, 151936 * 10, 2**31 - 1, 2**31]:
        f = make(d)
        ns = list(range(0, 2000)) + [2**32 - 1, 2**31, 2**31 - 1] + list(rng.integers(0, 2**32, 200))
        for n in ns:
            assert div(int(n), f) == int(n) // d, (n, d)
