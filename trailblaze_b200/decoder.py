"""Python handle on the library's decode step (tb_cuda_dec_*, include/tb_gguf_dequant.h part 3).

`Decoder` wraps the C ABI; `synthetic_model` fills one with random-init
weights of a given shape directly in device memory (for benchmarks):

  quant bytes        uniform random bytes
  fp16 d / dmin      |N(0,1)| * 0.01 at the type's header offsets
  norm weights       1 + 0.1 * N(0,1) (fp32)
  KV prefix          N(0,1) (fp32), positions [0, ctx)

Everything is drawn from one seeded torch generator on the device.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import qtypes as Q
from ._lib import DecConfig, DecLayer, lib


@dataclass
class ModelShape:
    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn_dim: int
    vocab: int
    rope_base: float = 1e6
    norm_eps: float = 1e-6
    w_qt: int = Q.Q4_K       # q/k/v/o/gate/up (routed: the experts' gate/up/down) and the token embedding
    down_qt: int = Q.Q6_K    # ffn_down (dense)
    out_qt: int = Q.Q6_K     # output (lm head)
    n_experts: int = 0       # > 0: every layer's FFN is routed (ffn_dim = one expert's width)
    top_k: int = 0
    attn_qt: int = -1        # q/k/v/o when it differs from w_qt
    router_qt: int = Q.F32   # ffn_gate_inp

    @property
    def a_qt(self) -> int:
        return self.w_qt if self.attn_qt < 0 else self.attn_qt

    def bytes_per_token(self, ctx: int) -> int:
        """Algorithmic HBM bytes of one decode step at context ctx (weights once, the
        selected experts only for a routed model, K and V of every layer over ctx
        positions, activations negligible)."""
        H, NH, NK, HD, F = self.hidden, self.n_heads, self.n_kv_heads, self.head_dim, self.ffn_dim
        attn = Q.row_bytes(self.a_qt, H) * (NH + 2 * NK) * HD + Q.row_bytes(self.a_qt, NH * HD) * H
        if self.n_experts:
            ffn = (Q.row_bytes(self.router_qt, H) * self.n_experts +
                   self.top_k * (Q.row_bytes(self.w_qt, H) * 2 * F + Q.row_bytes(self.w_qt, F) * H))
        else:
            ffn = Q.row_bytes(self.w_qt, H) * 2 * F + Q.row_bytes(self.down_qt, F) * H
        per_layer = attn + ffn + 2 * NK * ctx * HD * 4
        return self.n_layers * per_layer + Q.row_bytes(self.out_qt, H) * self.vocab + Q.row_bytes(self.w_qt, H)


# Qwen3-8B shape
QWEN3_8B = ModelShape(36, 4096, 32, 8, 128, 12288, 151936)
# Qwen3-30B-A3B shape: 128 experts of FFN 768, top 8; Q4_K
# experts, Q6_K attention and output
QWEN3_30B_A3B = ModelShape(48, 2048, 32, 4, 128, 768, 151936, w_qt=Q.Q4_K, out_qt=Q.Q6_K, n_experts=128, top_k=8,
                           attn_qt=Q.Q6_K)


class Decoder:
    """rank / world > 1: this process's tensor-parallel share of the model
    (tb_cuda_dec_create_tp; weight shard shapes in include/tb_gguf_dequant.h)."""

    def __init__(self, shape: ModelShape, max_ctx: int, quirks: bool = True, rank: int = 0, world: int = 1):
        self.L = lib()
        self.shape, self.max_ctx, self.rank, self.world = shape, max_ctx, rank, world
        s = shape
        self.cfg = DecConfig(s.n_layers, s.hidden, s.n_heads, s.n_kv_heads, s.head_dim, s.ffn_dim, s.vocab,
                             max_ctx, s.rope_base, s.norm_eps, 1 if quirks else 0)
        if s.n_experts and world > 1:
            self.d = self.L.tb_cuda_dec_create_moe_tp(ctypes.byref(self.cfg), s.n_experts, s.top_k, rank, world)
        elif s.n_experts:
            self.d = self.L.tb_cuda_dec_create_moe(ctypes.byref(self.cfg), s.n_experts, s.top_k)
        elif world > 1:
            self.d = self.L.tb_cuda_dec_create_tp(ctypes.byref(self.cfg), rank, world)
        else:
            self.d = self.L.tb_cuda_dec_create(ctypes.byref(self.cfg))
        if not self.d:
            raise RuntimeError("tb_cuda_dec_create failed")
        self._keep = []

    def tp_handle(self) -> bytes:
        h = (ctypes.c_ubyte * 64)()
        if self.L.tb_cuda_dec_tp_handle(self.d, h) != 1:
            raise RuntimeError("tb_cuda_dec_tp_handle failed")
        return bytes(h)

    def tp_connect(self, handles: list[bytes]) -> None:
        """handles: every rank's tp_handle(), in rank order."""
        buf = (ctypes.c_ubyte * (64 * len(handles))).from_buffer_copy(b"".join(handles))
        if self.L.tb_cuda_dec_tp_connect(self.d, buf) != 1:
            raise RuntimeError("tb_cuda_dec_tp_connect failed")

    def set_layer(self, li: int, wqkv, qkv_qt, wo, o_qt, wgu, gu_qt, wd, d_qt, attn_norm, ffn_norm,
                  q_norm=None, k_norm=None):
        ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        lw = DecLayer(ptr(wqkv), qkv_qt, ptr(wo), o_qt, ptr(wgu), gu_qt, ptr(wd), d_qt, ptr(attn_norm),
                      ptr(ffn_norm), ptr(q_norm), ptr(k_norm))
        self._keep += [wqkv, wo, wgu, wd, attn_norm, ffn_norm, q_norm, k_norm]
        if self.L.tb_cuda_dec_set_layer(self.d, li, ctypes.byref(lw)) != 1:
            raise RuntimeError(f"tb_cuda_dec_set_layer({li}) failed")

    def set_moe_layer(self, li: int, wr, r_qt, wgu_e, gue_qt, wd_e, de_qt):
        """Router [E][H], expert (gate, up) row pairs [E][2F][H], expert down [E][H][F]."""
        self._keep += [wr, wgu_e, wd_e]
        if self.L.tb_cuda_dec_set_moe_layer(self.d, li, wr.data_ptr(), r_qt, wgu_e.data_ptr(), gue_qt,
                                            wd_e.data_ptr(), de_qt) != 1:
            raise RuntimeError(f"tb_cuda_dec_set_moe_layer({li}) failed")

    def set_head(self, emb, emb_qt, out_norm, w_out, out_qt):
        self._keep += [emb, out_norm, w_out]
        if self.L.tb_cuda_dec_set_head(self.d, emb.data_ptr(), emb_qt, out_norm.data_ptr(), w_out.data_ptr(),
                                       out_qt) != 1:
            raise RuntimeError("tb_cuda_dec_set_head failed")

    def load_kv(self, li: int, which: int, t) -> None:
        """t: [n_kv_heads][n][head_dim] fp32 (host or device tensor), loaded at positions [0, n).
        The library copies on its own stream, which does not wait for torch's: a device
        tensor's producer is synchronised first."""
        import torch
        t = t.contiguous()
        if t.is_cuda:
            torch.cuda.current_stream(t.device).synchronize()
        fp = ctypes.cast(ctypes.c_void_p(t.data_ptr()), ctypes.POINTER(ctypes.c_float))
        if self.L.tb_cuda_dec_kv_copy(self.d, li, which, 0, t.shape[1], fp, 1) != 1:
            raise RuntimeError("tb_cuda_dec_kv_copy failed")

    def generate(self, token: int, pos: int, n: int, want_tokens: bool = True, logits=None):
        """n greedy tokens from (token, pos); returns (tokens or None, device milliseconds).
        logits (float32 numpy, this rank's vocabulary rows) receives the last step's logits."""
        toks = (ctypes.c_int * n)() if want_tokens else None
        ms = ctypes.c_float(0.0)
        lp = None
        if logits is not None:
            assert logits.dtype == np.float32 and logits.flags.c_contiguous
            lp = logits.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        if self.L.tb_cuda_dec_generate(self.d, token, pos, n, toks, lp, ctypes.byref(ms)) != 1:
            raise RuntimeError("tb_cuda_dec_generate failed")
        return (list(toks) if want_tokens else None), ms.value

    def set_sampling(self, temperature: float, top_k: int = 0, top_p: float = 0.9) -> None:
        """Greedy below temperature 0.01; else top-k (top_k > 0) or nucleus sampling in the step's graph."""
        if self.L.tb_cuda_dec_set_sampling(self.d, temperature, top_k, top_p) != 1:
            raise RuntimeError("tb_cuda_dec_set_sampling refused the settings")

    def generate_u(self, token: int, pos: int, u, logits=None):
        """len(u) tokens from (token, pos), step i sampled with the variate u[i]; logits (float32 numpy,
        vocab) receives the last step's logits when given.  Returns (tokens, device milliseconds)."""
        u = np.ascontiguousarray(u, dtype=np.float32)
        n = int(u.size)
        toks = (ctypes.c_int * n)()
        ms = ctypes.c_float(0.0)
        fp = ctypes.POINTER(ctypes.c_float)
        lp = None
        if logits is not None:
            assert logits.dtype == np.float32 and logits.flags.c_contiguous
            lp = logits.ctypes.data_as(fp)
        if self.L.tb_cuda_dec_generate_u(self.d, token, pos, n, u.ctypes.data_as(fp), toks, lp,
                                         ctypes.byref(ms)) != 1:
            raise RuntimeError("tb_cuda_dec_generate_u failed")
        return list(toks), ms.value

    def step(self, token: int, pos: int) -> int:
        nxt = ctypes.c_int(-1)
        if self.L.tb_cuda_dec_step(self.d, token, pos, ctypes.byref(nxt), None) != 1:
            raise RuntimeError("tb_cuda_dec_step failed")
        return nxt.value

    def close(self):
        if self.d:
            self.L.tb_cuda_dec_destroy(self.d)
            self.d = None


# header offsets of the fp16 d (and dmin) fields per quant type
_D_OFFSETS = {Q.Q4_K: (0, 2), Q.Q5_K: (0, 2), Q.Q6_K: (208,), Q.Q2_K: (80, 82), Q.Q3_K: (108,),
              Q.Q8_0: (0,), Q.Q4_0: (0,)}


def device_weights(qt: int, M: int, K: int, gen):
    """Random-init raw GGUF bytes of an M x K tensor, drawn on the device."""
    import torch
    bw, bb = Q.geometry(qt)
    nblk = M * (K // bw)
    t = torch.randint(0, 256, (nblk, bb), dtype=torch.uint8, device="cuda", generator=gen)
    for off in _D_OFFSETS.get(qt, ()):
        d = (torch.randn(nblk, device="cuda", generator=gen).abs() * 0.01).to(torch.float16)
        t[:, off:off + 2] = d.view(torch.uint8).view(nblk, 2)
    return t.view(-1)


def synthetic_model(shape: ModelShape, max_ctx: int, ctx: int, seed: int = 20261201, quirks: bool = True,
                    log=None, rank: int = 0, world: int = 1) -> Decoder:
    """A Decoder loaded with random-init weights of `shape` and an N(0,1) KV prefix of ctx positions.

    Every rank draws the whole model from one seeded generator, so the model is
    the same at every world size, and keeps its tensor-parallel share
    (include/tb_gguf_dequant.h part 3): the q, k and v rows of its heads (its kv
    head shared with world / n_kv_heads - 1 other ranks when world exceeds
    n_kv_heads), o's K columns of its q heads, its (gate, up) row pairs and
    down's K columns of those FFN rows (routed: its experts' rows, the router
    whole), its vocabulary rows of the output, the K and V cache of its kv
    heads; the norms and the token embedding whole.  A decode at world N
    therefore computes the same tokens as at world 1."""
    import torch
    from . import shard
    s = shape
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    dec = Decoder(s, max_ctx, quirks, rank, world)
    H, HD, NH, NK, F, V = s.hidden, s.head_dim, s.n_heads, s.n_kv_heads, s.ffn_dim, s.vocab
    nh, f = NH // world, F // world
    # this rank's kv heads [k0, k0 + nk): split, or one head shared by world / NK ranks
    nk, k0 = (NK // world, rank * (NK // world)) if NK % world == 0 else (1, rank // (world // NK))

    def norm(n):
        return 1.0 + 0.1 * torch.randn(n, device="cuda", generator=gen)

    def attn_shard(qkv, qt, wo, oqt):
        if world == 1:
            return qkv, wo
        R = (NH + 2 * NK) * HD
        qkv = torch.cat([shard.row_slice(qkv, qt, R, H, rank * nh * HD, (rank + 1) * nh * HD),
                         shard.row_slice(qkv, qt, R, H, (NH + k0) * HD, (NH + k0 + nk) * HD),
                         shard.row_slice(qkv, qt, R, H, (NH + NK + k0) * HD, (NH + NK + k0 + nk) * HD)])
        wo = shard.k_slice(wo, oqt, H, NH * HD, rank * nh * HD, (rank + 1) * nh * HD).contiguous()
        return qkv, wo

    for li in range(s.n_layers):
        if s.n_experts:
            E, aq = s.n_experts, s.a_qt
            qkv, wo = attn_shard(device_weights(aq, (NH + 2 * NK) * HD, H, gen), aq,
                                 device_weights(aq, H, NH * HD, gen), aq)
            dec.set_layer(li, qkv, aq, wo, aq, None, aq, None, aq, norm(H), norm(H), norm(HD), norm(HD))
            router = (0.05 * torch.randn(E * H, device="cuda", generator=gen)).view(torch.uint8)
            wgu_e = device_weights(s.w_qt, E * 2 * F, H, gen)
            wd_e = device_weights(s.w_qt, E * H, F, gen)
            if world > 1:   # this rank's experts [rank E/w, (rank+1) E/w): whole row ranges
                el = E // world
                wgu_e = shard.row_slice(wgu_e, s.w_qt, E * 2 * F, H, rank * el * 2 * F,
                                        (rank + 1) * el * 2 * F).contiguous()
                wd_e = shard.row_slice(wd_e, s.w_qt, E * H, F, rank * el * H, (rank + 1) * el * H).contiguous()
            dec.set_moe_layer(li, router, Q.F32, wgu_e, s.w_qt, wd_e, s.w_qt)
        else:
            qkv, qt = device_weights(s.w_qt, (NH + 2 * NK) * HD, H, gen), s.w_qt
            wo = device_weights(s.w_qt, H, NH * HD, gen)
            wgu = device_weights(s.w_qt, 2 * F, H, gen)
            wd = device_weights(s.down_qt, H, F, gen)
            qkv, wo = attn_shard(qkv, qt, wo, s.w_qt)
            if world > 1:
                wgu = shard.row_slice(wgu, s.w_qt, 2 * F, H, 2 * rank * f, 2 * (rank + 1) * f).contiguous()
                wd = shard.k_slice(wd, s.down_qt, H, F, rank * f, (rank + 1) * f).contiguous()
            dec.set_layer(li, qkv, qt, wo, s.w_qt, wgu, s.w_qt, wd, s.down_qt, norm(H), norm(H), norm(HD), norm(HD))
        if ctx > 0:
            for which in (0, 1):
                kv = torch.randn(NK, ctx, HD, device="cuda", generator=gen)
                dec.load_kv(li, which, kv[k0:k0 + nk])
    emb = device_weights(s.w_qt, V, H, gen)
    onorm = norm(H)
    w_out = device_weights(s.out_qt, V, H, gen)
    if world > 1:
        w_out = shard.row_slice(w_out, s.out_qt, V, H, rank * (V // world), (rank + 1) * (V // world)).contiguous()
    dec.set_head(emb, s.w_qt, onorm, w_out, s.out_qt)
    torch.cuda.synchronize()
    return dec
