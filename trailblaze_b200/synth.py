"""Seeded synthetic GGUF tensors and activations (numpy, counter-based).

Distributions follow the benchmark configs: every quant byte uniform, fp16
super-block scales fp16(RNE(|N(0,1)|*0.01)), Q8_K's fp32 d = |N(0,1)|*0.01,
float tensors N(0,1)*0.05, activations fp32 N(0,1).  Values are a pure
function of (seed, tensor id, element index): splitmix64 over a counter, so
any tensor can be regenerated anywhere (here or on a GPU host) bit for bit.
"""
from __future__ import annotations

import numpy as np

from . import qtypes as Q

_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _mix(z: np.ndarray) -> np.ndarray:
    z = z ^ (z >> np.uint64(30))
    z = z * _M1
    z = z ^ (z >> np.uint64(27))
    z = z * _M2
    return z ^ (z >> np.uint64(31))


def _key(seed: int, stream: int) -> np.uint64:
    with np.errstate(over="ignore"):
        k = _mix(np.array([(seed * 0x100000001B3 + stream * 0xD1B54A32D192ED03) & (2**64 - 1)],
                          dtype=np.uint64))
    return k[0]


_CHUNK = 1 << 22


def _u64_into(out: np.ndarray, key: np.uint64, start: int) -> None:
    with np.errstate(over="ignore"):
        ctr = np.arange(start + 1, start + out.size + 1, dtype=np.uint64)
        out[:] = _mix(key + ctr * _GAMMA)


def u64(seed: int, stream: int, n: int, start: int = 0) -> np.ndarray:
    """n 64-bit words of stream `stream`, counter positions start..start+n-1.

    Large requests are filled in independent chunks on a thread pool (numpy
    releases the GIL); the values do not depend on the chunking."""
    key = _key(seed, stream)
    out = np.empty(n, dtype=np.uint64)
    if n <= _CHUNK:
        _u64_into(out, key, start)
        return out
    from concurrent.futures import ThreadPoolExecutor
    import os
    jobs = [(i, min(i + _CHUNK, n)) for i in range(0, n, _CHUNK)]
    with ThreadPoolExecutor(max_workers=min(32, os.cpu_count() or 1)) as ex:
        list(ex.map(lambda ab: _u64_into(out[ab[0]:ab[1]], key, start + ab[0]), jobs))
    return out


def uniform_bytes(seed: int, stream: int, nbytes: int) -> np.ndarray:
    return u64(seed, stream, (nbytes + 7) // 8).view(np.uint8)[:nbytes].copy()


def normals(seed: int, stream: int, n: int) -> np.ndarray:
    """n standard normals (Box-Muller on 53-bit uniforms), float64."""
    m = (n + 1) // 2
    w = u64(seed, stream, 2 * m)
    u1 = ((w[0::2] >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)
    u2 = (w[1::2] >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.empty(2 * m, dtype=np.float64)
    z[0::2] = r * np.cos(2.0 * np.pi * u2)
    z[1::2] = r * np.sin(2.0 * np.pi * u2)
    return z[:n]


def _scales16(seed: int, stream: int, n: int) -> np.ndarray:
    return (np.abs(normals(seed, stream, n)) * 0.01).astype(np.float16).view(np.uint16)


def weights(qtype: int, M: int, K: int, seed: int = 0, tensor: int = 0) -> np.ndarray:
    """Raw GGUF bytes of an M x K tensor (rows contiguous), uint8."""
    bw, bb = Q.geometry(qtype)
    nbytes = Q.matrix_bytes(qtype, M, K)
    s_bytes, s_scale = 2 * tensor, 2 * tensor + 1
    if qtype in (Q.F32, Q.F16, Q.BF16):
        v = normals(seed, s_bytes, M * K) * 0.05
        if qtype == Q.F32:
            return v.astype(np.float32).view(np.uint8).copy()
        if qtype == Q.F16:
            return v.astype(np.float16).view(np.uint8).copy()
        b = (v.astype(np.float32).view(np.uint32) >> np.uint32(16)).astype(np.uint16)
        return b.view(np.uint8).copy()
    raw = uniform_bytes(seed, s_bytes, nbytes)
    nblk = nbytes // bb
    blk = raw.reshape(nblk, bb)
    if qtype == Q.Q8_K:
        d = (np.abs(normals(seed, s_scale, nblk)) * 0.01).astype(np.float32)
        blk[:, 0:4] = d.view(np.uint8).reshape(nblk, 4)
        return raw
    # offsets of the fp16 scale fields per type (tb_gguf_dequant.cu block layouts)
    fields = {Q.Q4_K: (0, 2), Q.Q5_K: (0, 2), Q.Q6_K: (208,), Q.Q3_K: (108,), Q.IQ3_S: (108,),
              Q.Q2_K: (80, 82), Q.Q8_0: (0,), Q.Q4_0: (0,)}[qtype]
    sc = _scales16(seed, s_scale, nblk * len(fields)).reshape(nblk, len(fields))
    for i, off in enumerate(fields):
        blk[:, off:off + 2] = sc[:, i:i + 1].view(np.uint8).reshape(nblk, 2)
    return raw


def activations(K: int, seed: int = 0, stream: int = 1_000_003) -> np.ndarray:
    return normals(seed, stream, K).astype(np.float32)
