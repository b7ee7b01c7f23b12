"""Generate tests/golden/golden_v1.npz from the REFERENCE's own code.

Run in a container that has the reference tree (its CPU sources are compiled
into oracle/_ref/ by oracle/Makefile); the GPU host only reads the .npz.

Contents, per qtype name N (inputs from trailblaze_b200.synth, seed 20261201):
  N/W            raw GGUF bytes, M x K
  N/x            fp32 activations, K
  N/ref_deq      tb_gguf_dequant_row(W) per row (layer4/tb_gguf.c:293-371),
                 i.e. the reference's shipped CPU decoders
  N/ref_mv       tb_gguf_dequant_matvec(W, x) (layer4/tb_gguf.c:376-419), fp32
  N/cuda_deq     oracle restatement of the reference CUDA-kernel decode
                 (equal to ref_deq except Q4_K / Q5_K, and IQ3_S which the CPU
                 path zeroes)
  N/cuda_mv64    fp64-accumulated matvec of cuda_deq
Known-answer blocks from the reference self-test (tb_gguf.c:995-1092), decoded
by the reference: kat/f16, kat/bf16, kat/q8_0_*, kat/q4_0_*, kat/q4k_smoke_*.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle.oracle import SEM_CUDA, Oracle, Reference  # noqa: E402
from trailblaze_b200 import qtypes as Q, synth  # noqa: E402

SEED = 20261201
SHAPES = {Q.F32: (3, 256), Q.F16: (3, 256), Q.BF16: (3, 256)}   # others (3, 512)


def main() -> None:
    o, r = Oracle(), Reference()
    out: dict[str, np.ndarray] = {}
    for qt in Q.ALL:
        name = Q.NAMES[qt]
        M, K = SHAPES.get(qt, (3, 512))
        W = synth.weights(qt, M, K, seed=SEED, tensor=qt)
        x = synth.activations(K, seed=SEED)
        rb = Q.row_bytes(qt, K)
        ref_deq = np.stack([r.dequant_row(qt, W[m * rb:(m + 1) * rb], K) for m in range(M)])
        out[f"{name}/W"] = W
        out[f"{name}/x"] = x
        out[f"{name}/ref_deq"] = ref_deq
        out[f"{name}/ref_mv"] = r.dequant_matvec(qt, W, M, K, x)
        out[f"{name}/cuda_deq"] = o.dequant(qt, W, M, K, SEM_CUDA)
        out[f"{name}/cuda_mv64"] = o.matvec_f64(qt, W, M, K, x, SEM_CUDA)
        out[f"{name}/MK"] = np.array([M, K], dtype=np.int64)

    # known-answer blocks of the reference self-test, decoded by the reference
    kat_h = np.array([0x3C00, 0xBC00], dtype=np.uint16)
    out["kat/f16_in"] = kat_h
    out["kat/f16_ref"] = r.dequant_row(Q.F16, kat_h.view(np.uint8), 2)
    kat_b = np.array([0x4000], dtype=np.uint16)
    out["kat/bf16_in"] = kat_b
    out["kat/bf16_ref"] = r.dequant_row(Q.BF16, kat_b.view(np.uint8), 1)
    q8 = np.zeros(34, dtype=np.uint8)
    q8[0:2] = np.array([0x2E66], dtype=np.uint16).view(np.uint8)
    q8[2:] = np.arange(1, 33, dtype=np.uint8)
    out["kat/q8_0_in"] = q8
    out["kat/q8_0_ref"] = r.dequant_row(Q.Q8_0, q8, 32)
    q4 = np.zeros(18, dtype=np.uint8)
    q4[0:2] = np.array([0x3C00], dtype=np.uint16).view(np.uint8)
    q4[2:] = 0x88
    out["kat/q4_0_in88"] = q4.copy()
    out["kat/q4_0_ref88"] = r.dequant_row(Q.Q4_0, q4, 32)
    q4[2] = 0xFF
    out["kat/q4_0_inFF"] = q4.copy()
    out["kat/q4_0_refFF"] = r.dequant_row(Q.Q4_0, q4, 32)
    q4k = np.zeros(144, dtype=np.uint8)
    q4k[0:2] = np.array([0x3C00], dtype=np.uint16).view(np.uint8)
    q4k[4:16] = 0x01
    q4k[16:] = 0x88
    out["kat/q4k_smoke_in"] = q4k
    out["kat/q4k_smoke_ref"] = r.dequant_row(Q.Q4_K, q4k, 256)          # tb_gguf.c: all 8.0
    out["kat/q4k_smoke_cuda"] = o.dequant(Q.Q4_K, q4k, 1, 256, SEM_CUDA).ravel()   # 8.0 / 32.0

    path = os.path.join(HERE, "golden_v1.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
