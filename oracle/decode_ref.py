"""CPU restatement of the reference's batch-1 decode step (TEST INFRASTRUCTURE ONLY).

numpy, float64, following layer4/tb_infer.c:553-887 (tb_layer_forward) and
:889-1050 (tb_infer_decode) for a dense model with the fused QKV layout
(tb_infer.c:640-649) and explicit positions:

  embedding row       tb_infer.c:936-963 (tb_gguf_dequant_row of the token's row)
  attention RMSNorm   tb_infer.c:609-620, layer1/tb_tensor.c:194-199
  QKV projection      tb_infer.c:640-649 (fused attn_qkv: q | k | v rows)
  RoPE                tb_infer.c:142-155, applied at :665
  QK-norm             tb_infer.c:667-709 (sc = 1/sqrt(sum/HD + eps), x*sc*w)
  KV append, attn     layer1/tb_tensor.c:303-409 (scale 1/sqrt(HD), softmax over 0..pos)
  output + residual   tb_infer.c:719-731
  FFN RMSNorm         tb_infer.c:734-745
  gate/up, SwiGLU     tb_infer.c:862-866, :130-135 (g / (1 + e^-g) * u); the two
                      projections are one tensor here, rows interleaved (gate_i, up_i)
  down + residual     tb_infer.c:866, :876
  final norm, head    tb_infer.c:987-1019
  greedy              layer1/tb_tensor.c:415-420 (first index of the maximum)

Mixture-of-experts layers (n_experts > 0) replace gate/up/down by the routed
FFN of tb_infer.c:753-850: router logits of the FFN-normed x2, softmax, the
reference's top-k scan and renormalisation (tb_infer.c:351-374), each selected
expert's SwiGLU FFN (gate/up rows interleaved as above, down), the outputs
accumulated with their weights in selection order, then the residual
(tb_infer.c:876).  The reference decodes the router tensor with its legacy
4-bit "compat" decoder whatever the tensor's GGUF type (tb_infer.c:757-763);
here it is decoded as the type it is stored in.

quirks=True keeps the reference's order: RoPE before the QK-norm, and K head
j rotated once for every query head h with h % NK == j (tb_infer.c:665).
quirks=False is the Qwen3 order (norm, then a single rotation).

Only tests/ use this module; the shipped library never does.
"""
from __future__ import annotations

import ctypes
import ctypes.util
import functools
from dataclasses import dataclass, field

import numpy as np

from .oracle import SEM_CUDA, Oracle


@dataclass
class DecodeModel:
    """Raw GGUF weight bytes (numpy uint8) plus fp32 norm vectors."""
    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn_dim: int
    vocab: int
    max_ctx: int
    rope_base: float = 1e6
    norm_eps: float = 1e-6
    emb: np.ndarray = None
    emb_qt: int = 12
    out_norm: np.ndarray = None
    lm: np.ndarray = None
    lm_qt: int = 14
    layers: list = field(default_factory=list)   # dicts: wqkv, qkv_qt, wo, o_qt, wgu, gu_qt, wd, d_qt,
                                                # attn_norm, ffn_norm, q_norm, k_norm; routed layers
                                                # instead of wgu / wd: wr, r_qt (router [E][H]),
                                                # wgu_e, gue_qt ([E][2F][H]), wd_e, de_qt ([E][H][F])
    n_experts: int = 0
    top_k: int = 0


def rms_norm(x, w, eps):
    """layer1/tb_tensor.c:194-199: x * (1/sqrt(sum(x^2)/n + eps)) * w."""
    x = np.asarray(x, np.float64)
    return x * (1.0 / np.sqrt(np.dot(x, x) / x.size + eps)) * np.asarray(w, np.float64)


_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.powf.restype = ctypes.c_float
_libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]


@functools.lru_cache(maxsize=4096)
def _rope_theta(pos, base, hd):
    """The reference's fp32 angles (float)pos / powf(base, 2.0f*i/hd), with the
    C library's powf (the one the reference links): at large positions one ulp
    of theta is a visible rotation, so an fp64 angle would not be the reference's."""
    th = np.empty(hd // 2, dtype=np.float32)
    for i in range(hd // 2):
        e = np.float32(np.float32(2.0) * np.float32(i)) / np.float32(hd)
        th[i] = np.float32(pos) / np.float32(_libm.powf(np.float32(base), e))
    return th.astype(np.float64)


def rope(v, pos, base, hd):
    """tb_rope_apply (layer4/tb_infer.c:142-155) on one head: interleaved pairs
    (2i, 2i+1) rotated by theta_i = pos / base^(2i/hd)."""
    theta = _rope_theta(int(pos), float(np.float32(base)), int(hd))
    c, s = np.cos(theta), np.sin(theta)
    v = np.asarray(v, np.float64)
    a, b = v[0::2].copy(), v[1::2].copy()
    out = v.copy()
    out[0::2] = a * c - b * s
    out[1::2] = a * s + b * c
    return out


def swiglu(g, u):
    """layer4/tb_infer.c:130-135: (g / (1 + e^-g)) * u."""
    g, u = np.asarray(g, np.float64), np.asarray(u, np.float64)
    return (g / (1.0 + np.exp(-g))) * u


def route(logits, k):
    """tb_route_experts (layer4/tb_infer.c:351-374) without its optional
    boosts: softmax, then one pass over the experts that replaces the first
    smallest of k slots (initially -1e30) whenever an expert's probability is
    strictly larger, then the k weights divided by their sum.  Returns
    (indices, weights) in slot order."""
    s = np.asarray(logits, np.float64)
    p = np.exp(s - s.max())
    p = p / p.sum()
    idx = [0] * k
    wts = [-1e30] * k
    for e in range(s.size):
        mi = min(range(k), key=lambda i: (wts[i], i))
        if p[e] > wts[mi]:
            wts[mi] = p[e]
            idx[mi] = e
    ws = sum(wts)
    if ws > 0:
        wts = [w / ws for w in wts]
    return idx, wts


def attention(q, kc, vc, n_heads, n_kv_heads):
    """layer1/tb_tensor.c:303-409 for one token: q [NH][HD] against cached
    kc, vc [NK][T][HD] (the new position already appended); query head h uses
    KV head h / (NH/NK); scores * 1/sqrt(HD); softmax over the T positions."""
    NH, NK = n_heads, n_kv_heads
    rep = NH // NK
    HD = q.shape[1]
    out = np.zeros((NH, HD))
    for h in range(NH):
        j = h // rep
        s = (kc[j] @ q[h]) * (1.0 / np.sqrt(HD))
        p = np.exp(s - s.max())
        out[h] = (p @ vc[j]) / p.sum()
    return out


def bf16_round(x):
    """float -> bf16 (round to nearest even) -> float64, as the prefill GEMM's
    operands (fp32 values rounded by __float2bfloat16_rn)."""
    u = np.ascontiguousarray(np.asarray(x, dtype=np.float32)).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    return (r.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


class LazyMat:
    """An M x K GGUF tensor kept as raw bytes: `@ x` dequantises chunks of rows
    (CUDA semantics) to float64 and multiplies them, `[i]` is one dequantised
    row, `.rows(a, b)` the tensor of rows [a, b).  For model widths whose
    float64 matrices would not fit in memory."""

    def __init__(self, o, qt, W, M, K):
        self.o, self.qt, self.W, self.M, self.K = o, qt, W, M, K
        self.rb = o.L.tbo_row_bytes(qt, K)

    def rows(self, a, b):
        return LazyMat(self.o, self.qt, self.W[a * self.rb:b * self.rb], b - a, self.K)

    def __getitem__(self, i):
        return self.o.dequant(self.qt, self.W[i * self.rb:(i + 1) * self.rb], 1, self.K, SEM_CUDA)[0].astype(
            np.float64)

    def __matmul__(self, x):
        x = np.asarray(x, np.float64)
        out = np.empty(self.M)
        step = max(1, (1 << 23) // self.K)
        for r0 in range(0, self.M, step):
            r1 = min(self.M, r0 + step)
            out[r0:r1] = self.rows(r0, r1).dense() @ x
        return out

    def dense(self):
        return self.o.dequant(self.qt, self.W, self.M, self.K, SEM_CUDA).astype(np.float64)


class LazyExperts:
    """E experts of R rows each, stacked in one GGUF tensor: `[e]` is expert e's LazyMat."""

    def __init__(self, o, qt, W, E, R, K):
        self.m = LazyMat(o, qt, W, E * R, K)
        self.R = R

    def __getitem__(self, e):
        return self.m.rows(e * self.R, (e + 1) * self.R)


class DecodeOracle:
    def __init__(self, m: DecodeModel, quirks: bool = True, lazy: bool = False):
        """lazy: keep the tensors as raw bytes and dequantise them chunk by chunk at every
        product (full model widths); otherwise dequantise every tensor once."""
        self.m = m
        self.quirks = quirks
        o = Oracle()
        H, NH, NK, HD, F = m.hidden, m.n_heads, m.n_kv_heads, m.head_dim, m.ffn_dim
        if lazy:
            deq = lambda W, qt, M, K: LazyMat(o, qt, W, M, K)  # noqa: E731
        else:
            deq = lambda W, qt, M, K: o.dequant(qt, W, M, K, SEM_CUDA).astype(np.float64)  # noqa: E731
        self.emb = deq(m.emb, m.emb_qt, m.vocab, H)
        self.lm = deq(m.lm, m.lm_qt, m.vocab, H)
        self.out_norm = m.out_norm.astype(np.float64)
        self.L = []
        E = m.n_experts
        for w in m.layers:
            routed = dict(
                wr=deq(w["wr"], w["r_qt"], E, H),
                wgu_e=(LazyExperts(o, w["gue_qt"], w["wgu_e"], E, 2 * F, H) if lazy else
                       deq(w["wgu_e"], w["gue_qt"], E * 2 * F, H).reshape(E, 2 * F, H)),
                wd_e=(LazyExperts(o, w["de_qt"], w["wd_e"], E, H, F) if lazy else
                      deq(w["wd_e"], w["de_qt"], E * H, F).reshape(E, H, F))) if E else dict(
                wgu=deq(w["wgu"], w["gu_qt"], 2 * F, H),
                wd=deq(w["wd"], w["d_qt"], H, F))
            self.L.append(dict(
                wqkv=deq(w["wqkv"], w["qkv_qt"], (NH + 2 * NK) * HD, H),
                wo=deq(w["wo"], w["o_qt"], H, NH * HD),
                **routed,
                attn_norm=w["attn_norm"].astype(np.float64), ffn_norm=w["ffn_norm"].astype(np.float64),
                q_norm=None if w.get("q_norm") is None else w["q_norm"].astype(np.float64),
                k_norm=None if w.get("k_norm") is None else w["k_norm"].astype(np.float64)))
        # caches [layer][NK][max_ctx][HD]
        self.kc = np.zeros((m.n_layers, NK, m.max_ctx, HD))
        self.vc = np.zeros((m.n_layers, NK, m.max_ctx, HD))

    def prefill(self, tokens, pos0: int):
        """The batched prefill of the library (tb_cuda_dec_prefill) restated one
        token at a time (causal attention makes the two the same): the dense
        layers' projections take bf16-rounded fp32 activations (RMSNorm outputs,
        attention output, SwiGLU activation) against bf16-rounded weights, as the
        tensor-core GEMM does; norms, attention and the residual in float64.
        Fills the caches; returns (last token's logits through the exact output
        matvec, greedy next token)."""
        m = self.m
        H, NH, NK, HD = m.hidden, m.n_heads, m.n_kv_heads, m.head_dim
        rep, eps = NH // NK, m.norm_eps
        if not hasattr(self, "_bf"):
            self._bf = [{k: bf16_round(w[k]) for k in ("wqkv", "wo", "wgu", "wd")} for w in self.L]
        x = None
        for i, token in enumerate(tokens):
            pos = pos0 + i
            x = np.asarray(self.emb[token], np.float64).copy()
            for li, w in enumerate(self.L):
                wb = self._bf[li]
                xn = bf16_round(rms_norm(x, w["attn_norm"], eps))
                qkv = wb["wqkv"] @ xn
                q = qkv[:NH * HD].reshape(NH, HD).copy()
                k = qkv[NH * HD:(NH + NK) * HD].reshape(NK, HD).copy()
                v = qkv[(NH + NK) * HD:].reshape(NK, HD).copy()
                self._rope_norm(w, q, k, pos, rep, eps)
                self.kc[li, :, pos] = k
                self.vc[li, :, pos] = v
                att = attention(q, self.kc[li, :, :pos + 1], self.vc[li, :, :pos + 1], NH, NK)
                x2 = x + wb["wo"] @ bf16_round(att.reshape(-1))
                xn2 = bf16_round(rms_norm(x2, w["ffn_norm"], eps))
                gu = wb["wgu"] @ xn2
                act = bf16_round(swiglu(gu[0::2], gu[1::2]))
                x = x2 + wb["wd"] @ act
        logits = self.lm @ rms_norm(x, self.out_norm, eps)
        return logits, int(np.argmax(logits))

    def _rope_norm(self, w, q, k, pos, rep, eps):
        m = self.m
        NH, NK, HD = m.n_heads, m.n_kv_heads, m.head_dim

        def rope_all():
            for h in range(NH):
                q[h] = rope(q[h], pos, m.rope_base, HD)
            for j in range(NK):
                for _ in range(rep if self.quirks else 1):
                    k[j] = rope(k[j], pos, m.rope_base, HD)

        def norm_all():
            if w["q_norm"] is not None:
                for h in range(NH):
                    q[h] = rms_norm(q[h], w["q_norm"], eps)
            if w["k_norm"] is not None:
                for j in range(NK):
                    k[j] = rms_norm(k[j], w["k_norm"], eps)

        if self.quirks:
            rope_all()
            norm_all()
        else:
            norm_all()
            rope_all()

    def step(self, token: int, pos: int):
        """One token at position pos; returns (logits, next_token).  Updates the caches."""
        m = self.m
        H, NH, NK, HD, F = m.hidden, m.n_heads, m.n_kv_heads, m.head_dim, m.ffn_dim
        rep = NH // NK
        eps = m.norm_eps
        x = self.emb[token].copy()
        for li, w in enumerate(self.L):
            xn = rms_norm(x, w["attn_norm"], eps)
            qkv = w["wqkv"] @ xn
            q = qkv[:NH * HD].reshape(NH, HD).copy()
            k = qkv[NH * HD:(NH + NK) * HD].reshape(NK, HD).copy()
            v = qkv[(NH + NK) * HD:].reshape(NK, HD).copy()

            def rope_all():
                for h in range(NH):
                    q[h] = rope(q[h], pos, m.rope_base, HD)
                for j in range(NK):
                    for _ in range(rep if self.quirks else 1):
                        k[j] = rope(k[j], pos, m.rope_base, HD)

            def norm_all():
                if w["q_norm"] is not None:
                    for h in range(NH):
                        q[h] = rms_norm(q[h], w["q_norm"], eps)
                if w["k_norm"] is not None:
                    for j in range(NK):
                        k[j] = rms_norm(k[j], w["k_norm"], eps)

            if self.quirks:
                rope_all()
                norm_all()
            else:
                norm_all()
                rope_all()
            self.kc[li, :, pos] = k
            self.vc[li, :, pos] = v
            att = attention(q, self.kc[li, :, :pos + 1], self.vc[li, :, :pos + 1], NH, NK)
            x2 = x + w["wo"] @ att.reshape(-1)
            xn2 = rms_norm(x2, w["ffn_norm"], eps)
            if m.n_experts:
                rl = w["wr"] @ xn2
                idx, wts = route(rl, m.top_k)
                ffn = np.zeros(H)
                acts = []
                for e, we in zip(idx, wts):
                    gu = w["wgu_e"][e] @ xn2
                    act = swiglu(gu[0::2], gu[1::2])
                    acts.append(act)
                    ffn += we * (w["wd_e"][e] @ act)
                x = x2 + ffn
                self.last = dict(x2=x2, qkv=qkv, att=att.reshape(-1), router=rl, ids=idx, wts=wts, acts=acts)
                continue
            gu = w["wgu"] @ xn2
            act = swiglu(gu[0::2], gu[1::2])   # (gate, up) rows interleaved
            x = x2 + w["wd"] @ act
            # the last layer's vectors, for tests that read the GPU's
            self.last = dict(x2=x2, qkv=qkv, att=att.reshape(-1), act=act)
        logits = self.lm @ rms_norm(x, self.out_norm, eps)
        return logits, int(np.argmax(logits))
