"""trailblaze_b200 — B200 (sm_100a) GGUF K-quant dequant x fp32 matvec.

The product is libtb_cuda_sm100.so (C ABI: include/tb_gguf_dequant.h).  This
package holds its sources (csrc/), its in-tree build (build.py), the ctypes
binding (_lib.py), a thin Python mirror of the ABI (kquant.py), the quant-type
table (qtypes.py) and seeded synthetic tensors (synth.py).
"""
from . import qtypes  # noqa: F401
from .kquant import (  # noqa: F401
    KQuantLib,
    load,
)
