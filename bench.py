"""Benchmark of the B200 GGUF K-quant dequant x fp32 matvec (libtb_cuda_sm100.so).

Metric: K-quant matvec HBM GB/s (algorithmic bytes / time).

Workload — BASELINE config 2, the per-type sweep at Qwen3-4B shapes:
q 4096x2560, k 1024x2560, v 1024x2560, gate 9728x2560, up 9728x2560,
down 2560x9728, lm_head 151936x2560, for each of Q2_K, Q3_K, Q4_K, Q5_K, Q6_K,
Q8_0 (Q4_K added to the config's five types so the headline type is in the
line): 42 matvecs, 1.87 GB of weights resident in HBM, seeded synthetic data
(trailblaze_b200.synth), fp32 activations multiplied in fp32 (the library's
default arithmetic).  Algorithmic bytes per matvec = weights + 4K + 4M.  One
sweep reads every tensor once, so consecutive reads of a tensor are separated
by ~1.9 GB of other traffic (> 126 MB L2): no L2 flush is needed.  A "step"
is R sweeps (--sweeps-per-step, default 100, ~50 ms), so that the K timed
steps span about a second.

`value`      device time of K steps (R replays each of one CUDA graph of the
             sweep), CUDA events on the launching stream, barrier + synchronize
             on both sides, max over ranks; whole-job GB/s.
`e2e`        the same sweep through the blocking reference ABI
             tb_cuda_matvec_device(W_dev, qtype, M, K, x_host, out_host): every
             call copies x host->device and y device->host (wall clock).
`roofline`   the kernel with the largest share of step time, timed per launch
             with CUDA events inside the timed pass; peak = MEASURED_PEAKS.json.
`cpu_baseline` the reference's own CPU path (oracle/_ref, built from its
             sources: tb_dispatch_matvec AVX-512/AVX2 tier for Q4_K/Q3_K/Q8_0,
             tb_gguf_dequant_matvec for Q2_K/Q5_K/Q6_K), all host threads, on a
             bounded row sample of the same tensors.
`reference_gpu` the reference's own CUDA kernels (layer4/tb_gguf_dequant.cu,
             unmodified, built for sm_100a into oracle/_ref) timed per launch on
             the same tensors and B200 at their default geometry, beside this
             library's kernels: the GPU-vs-GPU comparison (no Q2_K kernel there).
`int16`      the same sweep under the opt-in int16 activation arithmetic
             (tb_cuda_set_matvec_arith), labelled as such.

N > 1 (torchrun, one process per GPU, NCCL): weak scaling.  Every matrix is a
row shard of an N-times-taller matrix (rank r owns rows [r*M, (r+1)*M), drawn
from its own seed stream); rows are independent, so there is no collective in
the data path; the only collectives are the timing barriers and the
max-reduction of the elapsed time.

--impl reference: the reference's CPU implementation alone (rank 0; other ranks
exit 0), same config and metric, each step a bounded row sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

from trailblaze_b200 import qtypes as Q  # noqa: E402
from trailblaze_b200 import shard, synth  # noqa: E402

SHAPES = [("q_proj", 4096, 2560), ("k_proj", 1024, 2560), ("v_proj", 1024, 2560),
          ("gate", 9728, 2560), ("up", 9728, 2560), ("down", 2560, 9728), ("lm_head", 151936, 2560)]
TYPES = [Q.Q2_K, Q.Q3_K, Q.Q4_K, Q.Q5_K, Q.Q6_K, Q.Q8_0]
SEED = 20261201
METRIC = "K-quant matvec HBM GB/s (% of 8 TB/s)"
# reference CPU routine per type: 1 = tb_dispatch_matvec AVX-512 tier,
# 2 = AVX2 tier, 0 = tb_gguf_dequant_matvec (the dispatch tiers do no work for these types)
REF_PATH = {Q.Q4_K: 1, Q.Q3_K: 1, Q.Q8_0: 1, Q.Q2_K: 0, Q.Q5_K: 0, Q.Q6_K: 0}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def workload(rank: int, world: int, shape: str | None = None):
    """[(name, qtype, M, K, W bytes (rank's rows), x)] — rank-sharded rows of N*M-row matrices.

    `shape` = "TYPE:M:K" restricts the step to that single matvec (for profiling one launch)."""
    out = []
    types, shapes = TYPES, SHAPES
    if shape:
        tn, m, k = shape.split(":")
        types, shapes = [Q.BY_NAME[tn]], [(f"{m}x{k}", int(m), int(k))]
    for ti, qt in enumerate(types):
        for si, (nm, M, K) in enumerate(shapes):
            tensor = 100 * ti + si
            rb = Q.row_bytes(qt, K)
            full = synth.weights(qt, M, K, seed=SEED + 7919 * rank, tensor=tensor) if world > 1 else \
                synth.weights(qt, M, K, seed=SEED, tensor=tensor)
            assert full.size == M * rb
            out.append((f"{Q.NAMES[qt]}:{nm}", qt, M, K, full))
    xs = {K: synth.activations(K, seed=SEED + K) for _, _, K in shapes}
    return out, xs


class Clocks:
    """nvidia-smi sampling during the timed region (200 ms period)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        try:
            import torch
            u = str(getattr(torch.cuda.get_device_properties(index), "uuid", "") or "")
            if u:
                self.index = u if u.startswith("GPU-") else f"GPU-{u}"
        except Exception:  # noqa: BLE001
            pass
        self.proc = None
        import tempfile
        self.path = os.path.join(tempfile.gettempdir(), f"tb_clocks_{os.getpid()}_{index}.csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.f.close()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for ln in open(self.path):
                p = [v.strip() for v in ln.split(",")]
                if len(p) < 9:
                    continue
                try:
                    sm.append(float(p[1]))
                    mx = float(p[2])
                except ValueError:
                    continue
                for nme, v in zip(names, p[5:9]):
                    if v.lower() == "active":
                        reasons.add(nme)
        except OSError:
            pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        load = [v for v in sm if mx and v >= 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_sample(items, budget_s: float, nthreads: int, repeat: int = 1):
    """Time the reference CPU path on a row sample of every matrix; returns (GB/s, info)."""
    from oracle.oracle import Reference
    ref = Reference()
    # calibrate: 1% of rows of the largest matrix of each type
    xs = {}
    rate = {}
    for name, qt, M, K, W in items:
        if qt in rate:
            continue
        x = synth.activations(K, seed=SEED + K)
        xs[K] = x
        rows = max(nthreads, M // 200)
        rb = Q.row_bytes(qt, K)
        t, _ = ref.time_matvec(REF_PATH[qt], qt, W[:rows * rb], rows, K, rb, x, nthreads, 1)
        rate[qt] = rows * rb / max(t, 1e-9)
    total_bytes = sum(M * Q.row_bytes(qt, K) for _, qt, M, K, _ in items)
    est_full = sum(M * Q.row_bytes(qt, K) / rate[qt] for _, qt, M, K, _ in items)
    frac = min(1.0, budget_s / max(est_full, 1e-9))
    tot_b, tot_t = 0, 0.0
    for name, qt, M, K, W in items:
        rb = Q.row_bytes(qt, K)
        rows = max(min(M, nthreads), int(M * frac))
        x = xs.get(K)
        if x is None:
            x = xs[K] = synth.activations(K, seed=SEED + K)
        t, _ = ref.time_matvec(REF_PATH[qt], qt, W[:rows * rb], rows, K, rb, x, nthreads, repeat)
        tot_b += rows * rb + 4 * K + 4 * rows
        tot_t += t
    info = {"rows_fraction": round(frac, 5), "bytes": tot_b, "seconds": round(tot_t, 3),
            "variant": ref.variant, "of_total_bytes": total_bytes}
    return tot_b / tot_t / 1e9, info


def decode_leg(shape, ctx: int, n: int, e2e_tokens: int = 16, rank: int = 0, world: int = 1, dist=None):
    """Batch-1 greedy decode of a random-init model of `shape` with an N(0,1) fp32 KV
    prefix of ctx positions, through the library's graph-replayed decoder
    (tb_cuda_dec_*).  With world > 1 each rank holds its share of the same model
    (heads, FFN rows or experts, vocabulary), the o / FFN partials and the greedy
    pairs crossing NVLink by the library's own peer stores; times are the slowest
    rank's, and rank 0 also runs the whole model on its GPU to check that the
    tokens and the last logits are those of the single-device decode."""
    from trailblaze_b200.decoder import synthetic_model
    t0 = time.perf_counter()
    dec = synthetic_model(shape, max_ctx=ctx + n + e2e_tokens + 8, ctx=ctx, rank=rank, world=world)
    log(f"[bench] decode model built in {time.perf_counter() - t0:.1f}s")
    try:
        if world > 1:
            hs = [None] * world
            dist.all_gather_object(hs, dec.tp_handle())
            dec.tp_connect(hs)
            dist.barrier()
        dec.generate(1, ctx, 4, want_tokens=False)          # captures the graph, warms up
        if world > 1:
            dist.barrier()
        _, ms = dec.generate(1, ctx, n, want_tokens=False)  # n steps back to back, device time
        ms = shard.max_over_ranks(ms, dist if world > 1 else None, device="cuda")
        tok_s = n / (ms * 1e-3)
        bpt = shape.bytes_per_token(ctx + n // 2)
        # the same n steps again (same positions, so the same cache), tokens and last logits kept
        lg = np.zeros(shape.vocab // world, dtype=np.float32)
        toks, _ = dec.generate(1, ctx, n, want_tokens=True, logits=lg)
        tok = 1
        if world > 1:
            dist.barrier()
        t1 = time.perf_counter()
        for i in range(e2e_tokens):   # blocking step with the token read back each time
            tok = dec.step(tok, ctx + i)
        e2e = e2e_tokens / shard.max_over_ranks(time.perf_counter() - t1, dist if world > 1 else None, device="cuda")
    finally:
        if world > 1:
            dist.barrier()   # no rank unmaps its region while a peer may still store into it
        dec.close()
    check = {}
    if world > 1:
        import torch
        parts = [torch.zeros(shape.vocab // world, device="cuda") for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(lg).cuda())
        if rank == 0:
            lg_tp = torch.cat(parts).cpu().numpy().astype(np.float64)
            one = synthetic_model(shape, max_ctx=ctx + n + e2e_tokens + 8, ctx=ctx)
            try:
                lg1 = np.zeros(shape.vocab, dtype=np.float32)
                toks1, _ = one.generate(1, ctx, n, want_tokens=True, logits=lg1)
            finally:
                one.close()
            check = {"tokens_match_n1": toks == toks1,
                     "tokens_equal": int(sum(a == b for a, b in zip(toks, toks1))), "tokens": n,
                     "last_logits_rel_l2_vs_n1": float(np.linalg.norm(lg_tp - lg1) / np.linalg.norm(lg1))}
        dist.barrier()
    hbm, kind = peaks()
    return {"ctx": ctx, "tokens": n, "tok_per_s": round(tok_s, 2), "ms_per_token": round(ms / n, 4),
            "bytes_per_token": bpt, "GBps": round(bpt * tok_s / 1e9, 1),
            "frac_of_hbm": round(bpt * tok_s / 1e9 / (hbm * world), 4), "hbm_peak_kind": kind,
            "e2e_tok_per_s": round(e2e, 2), "e2e_api": "tb_cuda_dec_step (blocking, token read back)",
            "order": "reference (RoPE before QK-norm, K rotated n_heads/n_kv_heads times)", **check}


def decode_bench(ctx: int, n: int, e2e_tokens: int = 16, rank: int = 0, world: int = 1, dist=None):
    """batch-1 greedy decode of a random-init Qwen3-8B-shape model
    (Q4_K weights, Q6_K ffn_down and output), tensor-parallel at world > 1 (q/k/v by
    heads, o and down by K columns, gate/up by FFN rows, output by vocabulary)."""
    from trailblaze_b200.decoder import QWEN3_8B as shape
    d = decode_leg(shape, ctx, n, e2e_tokens, rank, world, dist)
    return {"model": "qwen3-8b shape: 36 layers, hidden 4096, 32 q / 8 kv heads, head_dim 128, ffn 12288, "
                     "vocab 151936; Q4_K weights, Q6_K ffn_down and output; fp32 KV",
            "parallelism": f"tensor-parallel x{world}" if world > 1 else "one GPU",
            "launches_per_token": 1 + 5 * shape.n_layers + 2, **d}


def moe_bench(ctx: int, n: int, e2e_tokens: int = 16, rank: int = 0, world: int = 1, dist=None):
    """batch-1 greedy decode of a random-init Qwen3-30B-A3B-shape
    routed model (48 layers, hidden 2048, 32 q / 4 kv heads, 128 experts of FFN 768,
    top 8; Q4_K experts, Q6_K attention and output, fp32 router).  Each layer: q/k/v,
    attention, o, router logits, top-k, the selected experts' gate/up and down as two
    expert-group matvecs (expert ids read on the device), combine.  At world > 1 the
    experts are sharded (128 / world per rank), attention is head-sharded (a kv head
    shared by world / 4 ranks at 8), the router replicated, and each rank's weighted
    expert output is summed across ranks over NVLink."""
    from trailblaze_b200.decoder import QWEN3_30B_A3B as shape
    d = decode_leg(shape, ctx, n, e2e_tokens, rank, world, dist)
    return {"model": "qwen3-30b-a3b shape: 48 layers, hidden 2048, 32 q / 4 kv heads, head_dim 128, 128 experts "
                     "(FFN 768) top 8, vocab 151936; Q4_K experts, Q6_K attention and output, fp32 router; fp32 KV",
            "parallelism": (f"expert-parallel x{world} ({shape.n_experts // world} experts per GPU), attention "
                            f"head-sharded" if world > 1 else "one GPU (all 128 experts resident)"),
            "launches_per_token": 1 + 8 * shape.n_layers + 2, **d}


def tensor_peak():
    """Measured dense bf16 TFLOP/s (burst: each GEMM below is timed alone)."""
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def prefill_bench(reps: int = 20):
    """the prefill GEMM C[T][N] = A[T][K] (bf16) x dequant(W)^T on
    the tensor cores (tb_cuda_qgemm_dev), Q4_K and Q6_K weights of 12288 x 4096 and
    4096 x 12288, T in {16, 128, 512}; random-init weights, A ~ N(0,1).  Each shape is
    timed alone over `reps` launches rotating four weight copies (CUDA events on the
    launching stream).  T = 16 is memory-bound (reported in weight GB/s against the
    HBM peak), T = 128 and 512 compute-bound (TFLOP/s against the bf16 peak)."""
    import torch
    from trailblaze_b200 import load
    from trailblaze_b200.decoder import device_weights
    k = load()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(SEED + 5)
    st = torch.cuda.Stream()
    hbm, _ = peaks()
    tpk, tkind = tensor_peak()
    rows = {}
    for qt, qn in ((Q.Q4_K, "Q4_K"), (Q.Q6_K, "Q6_K")):
        for N, K in ((12288, 4096), (4096, 12288)):
            Ws = [device_weights(qt, N, K, gen) for _ in range(4)]
            for T in (16, 128, 512):
                A = torch.randn(T, K, device="cuda", generator=gen).to(torch.bfloat16)
                C = torch.empty(T, N, device="cuda")

                def run(n):
                    for i in range(n):
                        if k.tb_cuda_qgemm_dev(Ws[i % 4].data_ptr(), qt, N, K, A.data_ptr(), T, C.data_ptr(),
                                               st.cuda_stream) != 1:
                            raise RuntimeError("tb_cuda_qgemm_dev refused the shape")
                with torch.cuda.stream(st):
                    run(3)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(st):
                    e0.record(st)
                    run(reps)
                    e1.record(st)
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1) / reps
                tfl = 2.0 * T * N * K / (ms * 1e-3) / 1e12
                wgb = Q.row_bytes(qt, K) * N / (ms * 1e-3) / 1e9
                rows[f"{qn}:{N}x{K}:T{T}"] = {"us": round(ms * 1e3, 1), "TFLOPs": round(tfl, 1),
                                              "frac_bf16_peak": round(tfl / tpk, 4),
                                              "weight_GBps": round(wgb, 1), "frac_hbm": round(wgb / hbm, 4)}
            del Ws
    return {"kernel": "k_qgemm (tcgen05.mma kind::f16, bf16 x bf16 -> fp32 in TMEM; W dequantised to bf16 "
                      "in shared memory; A by TMA)",
            "peak_tflops": tpk, "peak_kind": tkind, "per_shape": rows}


def run_reference(args, rank, world):
    if rank != 0:
        return
    items, _ = workload(0, 1)
    nthreads = os.cpu_count() or 1
    budget = float(os.environ.get("TB_REF_STEP_SECONDS", "4"))
    for _ in range(args.warmup):
        cpu_sample(items, budget / 4, nthreads)
    rates, info = [], {}
    t0 = time.perf_counter()
    for _ in range(args.steps):
        r, info = cpu_sample(items, budget, nthreads)
        rates.append(r)
    wall = time.perf_counter() - t0
    value = statistics.median(rates)
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * wall / max(args.steps, 1), 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": "qwen3-4b-shape per-type matvec sweep (BASELINE config 2 + Q4_K)",
                   "types": [Q.NAMES[t] for t in TYPES], "shapes": SHAPES},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": nthreads, "kind": "reference",
                         "sample": f"{info.get('rows_fraction')} of every matrix's rows per step "
                                   f"({info.get('bytes')} B), tb_dispatch_matvec AVX tier for Q4_K/Q3_K/Q8_0, "
                                   f"tb_gguf_dequant_matvec for Q2_K/Q5_K/Q6_K, "
                                   f"{info.get('variant')} build"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def quiet_init(k) -> int:
    """tb_cuda_init prints its device banner on the C library's stdout, as the
    reference's init does; the bench keeps stdout for its one JSON line, so the
    banner is sent to stderr."""
    import ctypes
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        ok = k.tb_cuda_init()
        ctypes.CDLL(None).fflush(None)
    finally:
        os.dup2(saved, 1)
        os.close(saved)
    return ok


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)   # 20 steps x 100 sweeps: a timed region of about 1.3 s
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--sweeps-per-step", type=int, default=100,
                    help="sweeps of the 42 matvecs per timed step (~0.5 ms each)")
    ap.add_argument("--no-int16", action="store_true", help="skip the opt-in int16-arithmetic sweep")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="skip timing the reference's own CUDA kernels on the same tensors")
    ap.add_argument("--shape", default=None,
                    help="TYPE:M:K — time this single matvec instead of the sweep (profiling aid)")
    ap.add_argument("--no-decode", action="store_true", help="skip the Qwen3-8B-shape decode tok/s leg")
    ap.add_argument("--decode-only", action="store_true",
                    help="only the decode tok/s leg (its line's value is tok/s; profiling aid)")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill GEMM leg (BASELINE config 5)")
    ap.add_argument("--prefill-only", action="store_true", help="only the prefill GEMM leg (profiling aid)")
    ap.add_argument("--no-moe", action="store_true", help="skip the routed (MoE) decode leg (BASELINE config 4)")
    ap.add_argument("--moe-only", action="store_true", help="only the MoE decode leg (profiling aid)")
    ap.add_argument("--moe-ctx", type=int, default=2048)
    ap.add_argument("--decode-ctx", type=int, default=4096)
    ap.add_argument("--decode-tokens", type=int, default=64)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))

    from trailblaze_b200 import load
    k = load()
    assert quiet_init(k) == 1

    if args.prefill_only:
        with Clocks(local) as clk:
            pf = prefill_bench()
        if rank == 0:
            best = max(v["TFLOPs"] for v in pf["per_shape"].values())
            print(json.dumps({"metric": "prefill GEMM TFLOP/s (best shape)", "value": best, "unit": "TFLOP/s",
                              "n_gpus": world, "higher_is_better": True, "dtype": "bf16",
                              "data": "synthetic (seeded torch generator on the device)",
                              "config": {"workload": "prefill only (profiling aid)"}, "prefill": pf,
                              "clocks": clk.summary()}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    if args.moe_only:
        with Clocks(local) as clk:
            d = moe_bench(args.moe_ctx, args.decode_tokens, rank=rank, world=world, dist=dist if world > 1 else None)
        if world > 1:
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"metric": "Qwen3-30B-A3B-shape MoE decode tok/s", "value": d["tok_per_s"],
                              "unit": "tok/s", "n_gpus": world, "higher_is_better": True,
                              "dtype": "fp32", "data": "synthetic (seeded torch generator on the device)",
                              "config": {"workload": "MoE decode only (profiling aid)"}, "moe": d,
                              "clocks": clk.summary()}), flush=True)
        return

    if args.decode_only:
        with Clocks(local) as clk:
            d = decode_bench(args.decode_ctx, args.decode_tokens, rank=rank, world=world,
                             dist=dist if world > 1 else None)
        if world > 1:
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"metric": "Qwen3-8B-shape Q4_K decode tok/s", "value": d["tok_per_s"],
                              "unit": "tok/s", "n_gpus": world, "higher_is_better": True,
                              "dtype": "fp32", "data": "synthetic (seeded torch generator on the device)",
                              "config": {"workload": "decode only (profiling aid)"}, "decode": d,
                              "clocks": clk.summary()}), flush=True)
        return

    t_gen = time.perf_counter()
    items, xs_host = workload(rank, world, args.shape)
    log(f"[bench] rank {rank}: generated {sum(w.nbytes for *_, w in items) / 1e9:.2f} GB in "
        f"{time.perf_counter() - t_gen:.1f}s")
    stream = torch.cuda.Stream()
    dW = [torch.from_numpy(w).cuda() for *_, w in items]
    dx = {K: torch.from_numpy(x).cuda() for K, x in xs_host.items()}
    dy = [torch.empty(M, dtype=torch.float32, device="cuda") for _, _, M, _, _ in items]
    torch.cuda.synchronize()
    alg = [Q.alg_bytes(qt, M, K) for _, qt, M, K, _ in items]
    sweep_bytes = sum(alg)
    R = max(1, args.sweeps_per_step)
    sh = stream.cuda_stream
    assert k.tb_cuda_get_matvec_arith() == 0   # fp32 activations, fp32 products and sums

    def ours(i, s):
        _, qt, M, K, _ = items[i]
        return k.tb_cuda_matvec_dev(dW[i].data_ptr(), qt, M, K, dx[K].data_ptr(), dy[i].data_ptr(), s)

    def sweep(s):
        for i in range(len(items)):
            assert ours(i, s) == 1

    def capture():
        with torch.cuda.stream(stream):
            sweep(sh)   # sets kernel attributes and plans before capture
        torch.cuda.synchronize()
        assert k.tb_cuda_last_error() == 0
        n0 = k.tb_cuda_launch_count()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            sweep(stream.cuda_stream)
        torch.cuda.synchronize()
        return gr, k.tb_cuda_launch_count() - n0

    g, launches_per_sweep = capture()
    for _ in range(args.warmup):
        for _ in range(R):
            g.replay()
    torch.cuda.synchronize()
    assert k.tb_cuda_last_error() == 0

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        time.sleep(0.3)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(args.steps):
                for _ in range(R):
                    g.replay()
            ev1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = ev0.elapsed_time(ev1)
    assert k.tb_cuda_last_error() == 0
    ms = shard.max_over_ranks(ms, dist if world > 1 else None, device="cuda")
    ms_step = ms / args.steps
    value = shard.whole_job_rate(sweep_bytes * R, world, ms_step * 1e-3) / 1e9

    # ---- per-launch timing: one sweep captured with a timing event between
    # consecutive launches, replayed; the events run on the launching stream
    # inside the graph, so no host launch gap enters the figures ----
    def per_launch(launch, idx, reps):
        """Average device ms of launch(i, stream) for i in idx, from a graph with an event
        between launches (or single launches between events if graphs refuse events)."""
        per = np.zeros(len(idx))
        try:
            evs = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(len(idx) + 1)]
            g2 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g2, stream=stream):
                evs[0].record(stream)
                for j, i in enumerate(idx):
                    assert launch(i, stream.cuda_stream) == 1
                    evs[j + 1].record(stream)
            for _ in range(reps):
                g2.replay()
                torch.cuda.synchronize()
                for j in range(len(idx)):
                    per[j] += evs[j].elapsed_time(evs[j + 1])
            del g2
            how = "CUDA graph of one sweep with an event between launches"
        except RuntimeError as e:   # no timing events inside graphs: time single launches
            log(f"[bench] in-graph timing unavailable ({e}); timing single launches")
            per[:] = 0
            how = "single launches between CUDA events (includes the host launch gap)"
            ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in idx]
            with torch.cuda.stream(stream):
                for _ in range(reps):
                    for j, i in enumerate(idx):
                        ev2[j][0].record(stream)
                        assert launch(i, sh) == 1
                        ev2[j][1].record(stream)
                    torch.cuda.synchronize()
                    for j in range(len(idx)):
                        per[j] += ev2[j][0].elapsed_time(ev2[j][1])
        return per / reps, how

    all_idx = list(range(len(items)))
    reps = max(3, min(args.steps, 10))
    per, per_how = per_launch(ours, all_idx, reps)
    assert k.tb_cuda_last_error() == 0
    # dominant kernel: a (type) instantiation, ranked by its share of the step
    by_type = {}
    for i, (name, qt, M, K, _) in enumerate(items):
        by_type.setdefault(qt, []).append(i)
    top_qt = max(by_type, key=lambda q: sum(per[i] for i in by_type[q]))
    top_i = max(by_type[top_qt], key=lambda i: per[i])
    hbm, hbm_kind = peaks()
    ach = alg[top_i] / (per[top_i] * 1e-3) / 1e9
    traffic = None
    tf = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tf):
        try:
            traffic = json.load(open(tf)).get(items[top_i][0])
        except ValueError:
            traffic = None

    def per_table(p):
        return {items[i][0]: {"us": round(p[j] * 1e3, 2), "GBps": round(alg[i] / (p[j] * 1e-3) / 1e9, 1),
                              "frac_hbm": round(alg[i] / (p[j] * 1e-3) / 1e9 / hbm, 3)}
                for j, i in enumerate(all_idx)}

    def per_type(p, idx):
        out = {}
        for qt in TYPES:
            js = [j for j, i in enumerate(idx) if items[i][1] == qt]
            if js:
                b = sum(alg[idx[j]] for j in js)
                t = sum(p[j] for j in js) * 1e-3
                out[Q.NAMES[qt]] = {"GBps": round(b / t / 1e9, 1), "frac_hbm": round(b / t / 1e9 / hbm, 3),
                                    "us": round(t * 1e6, 1)}
        return out

    per_mv = per_table(per)

    # ---- the opt-in int16 activation arithmetic on the same sweep (labelled) ----
    int16 = None
    if world == 1 and not args.shape and not args.no_int16:
        try:
            assert k.tb_cuda_set_matvec_arith(1) == 0
            g16, _ = capture()
            for _ in range(3):
                g16.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n16 = max(20, R)
            with torch.cuda.stream(stream):
                e0.record(stream)
                for _ in range(n16):
                    g16.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            ms16 = e0.elapsed_time(e1) / n16
            p16, _ = per_launch(ours, all_idx, reps)
            assert k.tb_cuda_last_error() == 0
            int16 = {"x_arith": "int16 block-scaled (x rounded to 2^-15 of each 128-activation slot's "
                                "largest |x|; exact dp4a products and sums); opt-in, narrower than fp32",
                     "value": round(sweep_bytes / (ms16 * 1e-3) / 1e9, 3), "unit": "GB/s",
                     "ms_per_sweep": round(ms16, 4), "per_type": per_type(p16, all_idx)}
            del g16
        except Exception as e:  # noqa: BLE001 - the int16 leg must not sink the fp32 line
            int16 = {"unavailable": f"{type(e).__name__}: {e}"}
        finally:
            k.tb_cuda_set_matvec_arith(0)

    # ---- the reference's own CUDA kernels on the same tensors (GPU vs GPU) ----
    ref_gpu = None
    if world == 1 and not args.no_ref_gpu:
        try:
            from oracle.oracle import ReferenceCuda
            rc = ReferenceCuda()
            if not hasattr(rc.L, "tbr_cuda_launch"):
                raise RuntimeError("oracle/_ref/libtbref_cuda.so predates tbr_cuda_launch")
            ridx = [i for i in all_idx if items[i][1] != Q.Q2_K]   # the reference has no Q2_K kernel

            def theirs(i, s):
                _, qt, M, K, _ = items[i]
                return rc.L.tbr_cuda_launch(dW[i].data_ptr(), qt, M, K, dx[K].data_ptr(), dy[i].data_ptr(), s)

            for i in ridx:   # warm-up
                assert theirs(i, sh) == 1
            torch.cuda.synchronize()
            pr, _ = per_launch(theirs, ridx, 3)
            b = sum(alg[i] for i in ridx)
            t_ref = float(sum(pr)) * 1e-3
            t_ours = float(sum(per[all_idx.index(i)] for i in ridx)) * 1e-3
            po = np.array([per[all_idx.index(i)] for i in ridx])
            ref_gpu = {"kernels": "k_*_matvec of layer4/tb_gguf_dequant.cu, unmodified, sm_100a, 128 threads x M "
                                  "CTAs (the reference's default geometry)",
                       "types": [Q.NAMES[t] for t in TYPES if t != Q.Q2_K],
                       "value": round(b / t_ref / 1e9, 3), "unit": "GB/s",
                       "ours_same_subset_GBps": round(b / t_ours / 1e9, 1),
                       "speedup_ours_over_reference": round(t_ref / t_ours, 2),
                       "per_type_reference": per_type(pr, ridx),
                       "per_type_speedup": {n: round(v["us"] / per_type(po, ridx)[n]["us"], 2)
                                            for n, v in per_type(pr, ridx).items()}}
        except Exception as e:  # noqa: BLE001 - the comparison leg must not sink the line
            ref_gpu = {"unavailable": f"{type(e).__name__}: {e}"}

    # ---- end to end through the blocking reference ABI (about a second of sweeps) ----
    e2e = None
    if not args.no_e2e:
        outs = [np.empty(M, dtype=np.float32) for _, _, M, _, _ in items]
        xh = {K: np.ascontiguousarray(x) for K, x in xs_host.items()}

        def blocking_sweep():
            ok = 0
            for i, (_, qt, M, K, _) in enumerate(items):
                ok += k.tb_cuda_matvec_device(dW[i].data_ptr(), qt, M, K, xh[K], outs[i]) == 1
            return ok

        t0 = time.perf_counter()
        for _ in range(2):
            assert blocking_sweep() == len(items)
        est = (time.perf_counter() - t0) / 2
        e_sweeps = int(min(400, max(3, round(1.0 / max(est, 1e-6)))))
        if world > 1:
            e_sweeps = int(shard.max_over_ranks(float(e_sweeps), dist, device="cuda"))
            dist.barrier()
        torch.cuda.synchronize()
        ok = 0
        t0 = time.perf_counter()
        for _ in range(e_sweeps):
            ok += blocking_sweep()
        torch.cuda.synchronize()
        dt = shard.max_over_ranks(time.perf_counter() - t0, dist if world > 1 else None, device="cuda")
        assert ok == e_sweeps * len(items), f"{e_sweeps * len(items) - ok} blocking matvecs failed"
        e2e = {"value": round(world * sweep_bytes * e_sweeps / dt / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": R * sum(4 * K for _, _, _, K, _ in items),
               "d2h_bytes_per_step": R * sum(4 * M for _, _, M, _, _ in items),
               "sweeps_timed": e_sweeps,
               "api": "tb_cuda_matvec_device (blocking, host x in / host y out), every call's return checked"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            hosts = [(n, qt, M, K, w) for n, qt, M, K, w in items]
            rate, info = cpu_sample(hosts, float(os.environ.get("TB_CPU_SECONDS", "12")), os.cpu_count() or 1)
            cpu = {"value": round(rate, 3), "unit": "GB/s", "cores": os.cpu_count(), "kind": "reference",
                   "sample": f"first {info['rows_fraction']} of every matrix's rows ({info['bytes']} B, "
                             f"{info['seconds']} s), tb_dispatch_matvec AVX tier for Q4_K/Q3_K/Q8_0, "
                             f"tb_gguf_dequant_matvec for Q2_K/Q5_K/Q6_K, {info['variant']} build"}
        except Exception as e:  # noqa: BLE001 - the baseline must not sink the GPU line
            cpu = {"value": None, "unit": "GB/s", "cores": os.cpu_count(), "kind": "reference",
                   "sample": f"unavailable: {type(e).__name__}: {e}"}

    clocks = clk.summary()
    decode = None
    if not args.no_decode and not args.shape:
        try:
            decode = decode_bench(args.decode_ctx, args.decode_tokens, rank=rank, world=world,
                                  dist=dist if world > 1 else None)
        except Exception as e:  # noqa: BLE001 - the decode leg must not sink the sweep line
            decode = {"unavailable": f"{type(e).__name__}: {e}"}
    moe = None
    if not args.no_moe and not args.shape:
        try:
            moe = moe_bench(args.moe_ctx, args.decode_tokens, rank=rank, world=world,
                            dist=dist if world > 1 else None)
        except Exception as e:  # noqa: BLE001 - the MoE leg must not sink the sweep line
            moe = {"unavailable": f"{type(e).__name__}: {e}"}
    prefill = None
    if world == 1 and not args.no_prefill and not args.shape:
        try:
            prefill = prefill_bench()
        except Exception as e:  # noqa: BLE001 - the prefill leg must not sink the sweep line
            prefill = {"unavailable": f"{type(e).__name__}: {e}"}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "x_arith": "fp32 (fp32 activations, fp32 products and fp32 sums, as the reference's kernels)",
        "data": "synthetic (seeded; trailblaze_b200.synth)",
        "config": {"workload": (f"single matvec {args.shape} (profiling aid, not the headline)" if args.shape
                                else "qwen3-4b-shape per-type matvec sweep (BASELINE config 2 + Q4_K)"),
                   "types": [Q.NAMES[t] for t in TYPES], "shapes": SHAPES,
                   "sweeps_per_step": R, "bytes_per_sweep_per_gpu": sweep_bytes,
                   "timed_region_s": round(ms * 1e-3, 3),
                   "l2": (f"no flush: each sweep streams {sweep_bytes / 1e9:.2f} GB > 126 MB L2 before a tensor "
                          "is re-read" if sweep_bytes > 2 * 126e6
                          else "inputs partly L2-resident between sweeps (profiling aid)"),
                   "parallelism": f"row-sharded x{world}, no data-path collective",
                   "timing": "R replays per step of a CUDA graph of one sweep, CUDA events, max over ranks"},
        "frac_of_8TBps": round(value / world / 8000.0, 4),
        "gpu_launches": launches_per_sweep * R * args.steps,
        "roofline": {"bound": "hbm", "kernel": f"k_matvec<{Q.NAMES[top_qt]}> on {items[top_i][0]}",
                     "achieved": round(ach, 1), "peak": hbm, "peak_kind": hbm_kind, "unit": "GB/s",
                     "frac": round(ach / hbm, 4), "traffic": traffic,
                     "alg_bytes_per_launch": alg[top_i], "timing": per_how},
        "per_matvec": per_mv,
        "per_type": per_type(per, all_idx),
        "clocks": clocks,
    }
    if int16:
        line["int16"] = int16
    if ref_gpu:
        line["reference_gpu"] = ref_gpu
    if e2e:
        line["e2e"] = e2e
    if decode:
        line["decode"] = decode
    if moe:
        line["moe"] = moe
    if prefill:
        line["prefill"] = prefill
    if cpu:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
