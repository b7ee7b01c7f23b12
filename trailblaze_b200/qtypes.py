"""GGUF quant types carried by the Trailblaze dequant ABI.

ids are ggml's (layer4/tb_gguf_dequant.cu:447-460); geometry is
(weights per block, bytes per block) as in layer4/tb_gguf.c:380-393.
"""
F32, F16, Q4_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K, IQ3_S, BF16 = 0, 1, 2, 8, 10, 11, 12, 13, 14, 15, 21, 30

NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q8_0: "Q8_0", Q2_K: "Q2_K", Q3_K: "Q3_K",
         Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", Q8_K: "Q8_K", IQ3_S: "IQ3_S", BF16: "BF16"}
BY_NAME = {v: k for k, v in NAMES.items()}

GEOMETRY = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34),
            Q2_K: (256, 84), Q3_K: (256, 110), IQ3_S: (256, 110), Q4_K: (256, 144),
            Q5_K: (256, 176), Q6_K: (256, 210), Q8_K: (256, 292)}

ALL = [F32, F16, BF16, Q4_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K, IQ3_S]


def geometry(qtype: int) -> tuple[int, int]:
    return GEOMETRY[qtype]


def row_bytes(qtype: int, K: int) -> int:
    bw, bb = GEOMETRY[qtype]
    if K % bw:
        raise ValueError(f"K={K} is not a multiple of the {NAMES[qtype]} block size {bw}")
    return (K // bw) * bb


def matrix_bytes(qtype: int, M: int, K: int) -> int:
    return M * row_bytes(qtype, K)


def alg_bytes(qtype: int, M: int, K: int) -> int:
    """Algorithmic bytes of one matvec: weights once, x once, y once."""
    return matrix_bytes(qtype, M, K) + 4 * K + 4 * M
