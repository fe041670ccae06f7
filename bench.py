#!/usr/bin/env python
"""OABF decode dequant-GEMV benchmark on B200 (1..8 GPUs, one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--m 1] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Workload (12B-class decoder, random init, seeded): every linear of 48 decoder layers —
q 4096x3840, k/v 2048x3840, o 3840x4096, gate/up 15360x3840, down 3840x15360 — compressed
to OABF (block 16; weights N(0, 0.02) bf16 with 1.5% StudentT(3)*20*0.02 outliers). q|k|v and
gate|up are fused launches, so one step = one decode token (M activations of bf16) through
192 fused dequant-GEMV launches reading ~7.4 GB of packed weights (inputs far larger than
L2, so no flush is needed). Tensor parallelism over N ranks: q/k/v/gate/up split their output
rows, o/down split their input in whole 256-column stages and sum their partial outputs across
ranks, by default inside the GEMV itself (``--exchange fused``: peer-memory push and ordered sum
over NVLink in the epilogue; ``allreduce``: a separate NVLink all-reduce kernel; ``nccl``).

``value`` = algorithmic bytes per step over all ranks (11 B per 16-weight block + 10 B per
outlier + bf16 X and Y) / step time, max over ranks. The headline step is one CUDA graph of the
192 launches in model order, timed with CUDA events; per-kind graphs give the per-kind rates and
the roofline kernel. ``e2e`` runs the same step through the public ``OABFLinear`` modules with
the activations copied from pinned host memory each step and the outputs copied back. At N = 1
the line also carries ``model_decode`` (whole tokens of a random-init 12B-class Gemma-3 around
these linears: embedding, norms, RoPE, KV cache, attention, GeGLU, bf16 lm_head and the greedy
pick in one CUDA graph per token), ``prefill`` (the gate|up linear at M = 2048 on the path
packed_linear takes there, the two-pass expansion + cuBLASLt GEMM, beside the fused tcgen05
prefill GEMM), ``bf16_cublas_decode`` and ``compress``.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "OABF dequant-GEMV HBM GB/s and decode tokens/s at 1/2/4/8 B200"
N_LAYERS = 48
KINDS = ("qkv", "o", "gate_up", "down")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--m", type=int, default=1, help="decode batch (tokens per step, <= 16)")
    ap.add_argument("--layers", type=int, default=N_LAYERS)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", choices=("fused", "allreduce", "nccl"), default="fused",
                    help="row-parallel exchange (tensor parallelism): fused into the GEMV epilogue "
                         "over NVLink peer memory, a separate NVLink all-reduce kernel, or NCCL")
    ap.add_argument("--no-model", action="store_true",
                    help="skip the full-model decode token step (N = 1 only)")
    ap.add_argument("--no-70b", action="store_true", help="skip the 70B-class stress section")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the prefill GEMM and the bf16 cuBLAS decode baseline")
    return ap.parse_args()


# --------------------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# --------------------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.n0 = 0

    def __enter__(self):
        # the sampler is running (its first sample read) before the timed region starts, and only
        # samples read after that count: a short region (a few steps on many GPUs) still gets some
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t_end = time.monotonic() + 5.0
            while not self.lines and time.monotonic() < t_end and self.proc.poll() is None:
                time.sleep(0.005)
        except Exception:
            self.proc = None
        self.n0 = len(self.lines)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            # at least one sample read after the region began (taken during it or as it ends)
            t_end = time.monotonic() + 0.5
            while len(self.lines) <= self.n0 and time.monotonic() < t_end and self.proc.poll() is None:
                time.sleep(0.005)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[self.n0:]:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------------------
# weights
# --------------------------------------------------------------------------------------
def _progress(rank, msg):
    """One line to stderr per phase in multi-rank runs (shows where a stuck rank is)."""
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        print(f"[rank {rank}] {time.strftime('%H:%M:%S')} {msg}", file=sys.stderr, flush=True)


GEMMA12B = dict(n_heads=16, n_kv_heads=8, head_dim=256, inter=15360, vocab=262144, hidden=3840)


def build_layers(n_layers, rank, world, device, shapes=None, plan_args=None, frac=0.015, seed0=1000,
                 records=True):
    """Every linear of n_layers decoder layers, this rank's part as the whole-model tensor-parallel
    plan splits it (whole heads; the MLP in 256-column stages), compressed on the GPU; with
    ``records`` also the stage records that one-token launches read (about the packed size again
    in device memory)."""
    from flashbfp_b200 import OABFCompressor, packed, tp, workloads
    comp = OABFCompressor(16, 64)
    shapes = shapes or workloads.GEMMA12B_LAYER
    pa = plan_args or GEMMA12B
    plan = tp.DecoderPlan(pa["n_heads"], pa["n_kv_heads"], pa["head_dim"], pa["inter"], pa["vocab"],
                          rank, world)
    layers = []
    shard_bytes = {k: 0 for k in KINDS}
    for li in range(n_layers):
        parts = {}
        for j, (name, (n, k)) in enumerate(shapes.items()):
            W = workloads.decode_weight(n, k, seed=seed0 + 16 * li + j, frac=frac, device=device)
            # this rank's part, compressed with the whole matrix's threshold
            dp, sp = plan.compress(W, name, comp)
            parts[name] = packed.from_compressed(dp, sp, device, build_tiles=False)
            del W, dp, sp
        L = {
            "qkv": packed.concat_rows([parts["q_proj"], parts["k_proj"], parts["v_proj"]]),
            "o": parts["o_proj"].build_tiles(),
            "gate_up": packed.concat_rows([parts["gate_proj"], parts["up_proj"]]),
            "down": parts["down_proj"].build_tiles(),
        }
        for kk in KINDS:
            shard_bytes[kk] += L[kk].packed_bytes()
            if records:
                L[kk].build_records()
        layers.append(L)
        if li % 8 == 7:
            torch.cuda.empty_cache()
    return layers, shard_bytes


def step_io(layers, m, device, fp32_kinds):
    """Activation inputs per kind and output buffers per (layer, kind) (fp32 for the row-parallel
    kinds whose partial outputs a separate all-reduce sums)."""
    from flashbfp_b200 import workloads
    L0 = layers[0]
    xs = {kk: workloads.activations(m, L0[kk].k_in, seed=7 + i, device=device)
          for i, kk in enumerate(KINDS)}
    outs = []
    for L in layers:
        o = {}
        for kk in KINDS:
            rowpar = kk in fp32_kinds
            o[kk] = torch.empty(m, L[kk].n_out, dtype=torch.float32 if rowpar else torch.bfloat16,
                                device=device)
        outs.append(o)
    return xs, outs


def algorithmic_bytes(layers, m, kind):
    tot = 0
    for L in layers:
        pw = L[kind]
        tot += pw.packed_bytes() + 2 * m * pw.k_in + 2 * m * pw.n_out
    return tot


# --------------------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------------------
def run_ours(args):
    import torch.distributed as dist
    from flashbfp_b200 import build as _build
    from flashbfp_b200.linear import packed_linear, OABFLinear

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    if rank == 0:
        _build.build()
    if world > 1:
        dist.barrier()
    m = args.m
    _progress(rank, "building layers")
    layers, shard_bytes = build_layers(args.layers, rank, world, device)
    _progress(rank, "layers built")
    # row-parallel kinds: exchange fused into the GEMV where the tensor-core kernel takes the
    # shard, else the GEMV's fp32 partials and a separate all-reduce
    from flashbfp_b200.linear import fused_shard_eligible
    rowpar = [kk for kk in ("o", "down") if world > 1]
    ar_elems = 16 * max(layers[0][kk].n_out for kk in ("o", "down"))
    fused = {kk for kk in rowpar if args.exchange == "fused" and
             all(fused_shard_eligible(Ly[kk], ar_elems) for Ly in layers)}
    if world > 1:                               # every rank takes the same path
        got = [None] * world
        dist.all_gather_object(got, sorted(fused))
        fused = set.intersection(*(set(g) for g in got))
    xs, outs = step_io(layers, m, device, set(rowpar) - fused)
    from flashbfp_b200 import _lib
    L = _lib.lib()
    ws = {kk: torch.zeros(L.fbfp_gemv_workspace_bytes(16, layers[0][kk].npad), dtype=torch.uint8,
                          device=device) for kk in KINDS}
    reducer = None
    if world > 1 and args.exchange != "nccl":
        from flashbfp_b200.tp import NVLinkAllReduce
        reducer = NVLinkAllReduce(ar_elems)

    def exchange(y):
        if reducer is not None:
            reducer(y)
        else:
            dist.all_reduce(y)

    def launch_one(kk, pw, y):
        if kk in ("o", "down") and world > 1:
            if kk in fused:
                _gemv_fused(L, _lib, xs[kk], pw, y, ws[kk], reducer)
            else:
                _gemv(L, _lib, xs[kk], pw, y, ws[kk])
                exchange(y)
        else:
            _gemv(L, _lib, xs[kk], pw, y, ws[kk])

    def launch_kind(kk):
        for li, Ly in enumerate(layers):
            launch_one(kk, Ly[kk], outs[li][kk])

    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for kk in KINDS:                        # eager warm-up (sets kernel attributes)
            launch_kind(kk)
    torch.cuda.synchronize(device)
    for kk in KINDS:                            # a kernel that gave up a bounded wait fails here
        _lib.check(L.fbfp_gemv_check(_lib.ptr(ws[kk]), _lib.stream_ptr(device)), "fbfp_gemv_check")
    _progress(rank, "eager warm-up done")
    def launch_step():
        # one decode token in model order: per layer q|k|v, o, gate|up, down (row-parallel
        # kinds all-reduce their partial outputs); consecutive launches overlap through
        # programmatic dependent launch
        for li, Ly in enumerate(layers):
            for kk in KINDS:
                launch_one(kk, Ly[kk], outs[li][kk])

    graphs = {}
    for kk in KINDS:                            # per kind: rates and the roofline kernel
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            launch_kind(kk)
        graphs[kk] = g
    g_step = torch.cuda.CUDAGraph()             # the whole step: the headline number
    with torch.cuda.graph(g_step, stream=stream):
        launch_step()
    graphs["step"] = g_step
    torch.cuda.synchronize(device)
    _progress(rank, "graphs captured")

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            g_step.replay()
            for kk in KINDS:
                graphs[kk].replay()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()

    K = args.steps
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk, torch.cuda.stream(stream):
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
        start.record(stream)
        for _ in range(K):
            g_step.replay()
        stop.record(stream)
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
    _progress(rank, "timed steps done")
    elapsed_ms = start.elapsed_time(stop)
    # per-kind rates (all 48 launches of one kind back to back), outside the headline timing;
    # each kind's timed replays follow one untimed replay, which (for the kinds that exchange
    # with the other ranks) lines the ranks up, so no rank's timing absorbs another's late start
    Kk = max(1, K // 4)
    kind_ms = {}
    with torch.cuda.stream(stream):
        for kk in KINDS:
            graphs[kk].replay()
            a_ev, b_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a_ev.record(stream)
            for _ in range(Kk):
                graphs[kk].replay()
            b_ev.record(stream)
            b_ev.synchronize()
            kind_ms[kk] = a_ev.elapsed_time(b_ev) / Kk
    t = torch.tensor([elapsed_ms] + [kind_ms[kk] for kk in KINDS], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t[0])
    kind_ms = {kk: float(t[1 + i]) for i, kk in enumerate(KINDS)}
    ms_per_step = elapsed_ms / K

    # whole-job algorithmic bytes per step (sum of the shards over the ranks)
    b = torch.tensor([algorithmic_bytes(layers, m, kk) for kk in KINDS], dtype=torch.float64,
                     device=device)
    if world > 1:
        dist.all_reduce(b)
    kind_bytes = {kk: float(b[i]) for i, kk in enumerate(KINDS)}
    _progress(rank, "step timings reduced")
    step_bytes = sum(kind_bytes.values())
    value = step_bytes / (ms_per_step * 1e-3) / 1e9

    # ---------------- e2e through the public module API ----------------
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, layers, xs, stream, device, world, rank, step_bytes, exchange, reducer, fused)

    model = None
    if m == 1 and not args.no_model:
        _progress(rank, "model decode")
        model = run_models(layers, device, rank, world)

    stress = None
    if not args.no_70b:
        _progress(rank, "70B-class stress")
        stress = run_stress70b(device, rank, world)

    prefill = bf16 = compress = sweep = None
    if world == 1 and not args.no_prefill:
        sweep = run_decode_sweep(layers, device)
        prefill = run_prefill(layers, device)
        bf16 = run_bf16_decode(device, m=m)
        compress = run_compress(device)

    result = None
    if rank == 0:
        peaks = _peaks()
        per_rank_kind = {kk: kind_bytes[kk] / world / (kind_ms[kk] * 1e-3) / 1e9 for kk in KINDS}
        dom = "gate_up"
        achieved = per_rank_kind[dom]
        peak = peaks["hbm_gbs"]
        result = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": K,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded random 12B-class weights, OABF-compressed on the GPU)",
            "config": {
                "workload": (f"decode step: M={m} bf16 token(s) through the linears of {args.layers} "
                             "12B-class layers (q|k|v 8192x3840, o 3840x4096, gate|up 30720x3840, "
                             "down 3840x15360; OABF block 16, 1.5% StudentT(3)x20 outliers)"),
                "m": m, "layers": args.layers, "parallelism": f"tp{world}",
                "exchange": (None if world == 1 else
                             "NCCL all-reduce" if args.exchange == "nccl" else
                             "one-shot all-reduce kernel over NVLink peer memory (csrc/allreduce.cu)"
                             if args.exchange == "allreduce" else
                             "fused into the GEMV epilogue: peer-memory push and ordered sum over "
                             "NVLink (fbfp_gemv_allreduce) for %s" % (sorted(fused) or "none")),
                "launches_per_step": 4 * args.layers,
                "l2": "inputs larger than L2 (%.2f GB packed per step per rank)" % (step_bytes / world / 1e9),
                "graphs": ("one CUDA graph per step (192 launches in model order, programmatic "
                           "dependent launch between them); per-kind rates from per-kind graphs"),
            },
            "decode_tokens_per_s": round(m * 1000.0 / ms_per_step, 1),
            "decode_tokens_per_s_note": "linear layers only (no attention/norm/lm_head)",
            "layers_gbs_per_rank": {kk: round(v, 1) for kk, v in per_rank_kind.items()},
            "roofline": {
                "bound": "hbm", "kernel": "gemv_cc_kernel (stage records, gate|up 30720x3840 launches)",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": peaks["source"],
                "traffic": _traffic(m),
            },
            "gpu_launches": 4 * args.layers * K,
            "e2e": e2e,
            "model_decode": model,
            "decode_sweep": sweep,
            "stress_70b": stress,
            "prefill": prefill,
            "bf16_cublas_decode": bf16,
            "compress": compress,
        }
    clocks = clk.summary()
    if rank == 0:
        result["clocks"] = clocks
        if not args.no_cpu_baseline and world == 1:
            result["cpu_baseline"] = cpu_baseline_sample(10.0)
        print(json.dumps(result), flush=True)
    # CUDA graphs that captured NCCL collectives go before the process group does
    for g in graphs.values():
        g.reset()
    del graphs
    torch.cuda.synchronize(device)
    if world > 1:
        # Every collective of this run has completed (the step timings were all-reduced above).
        # Tearing NCCL down after graph-captured collectives can block indefinitely, so the
        # ranks leave without it.
        _progress(rank, "done")
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)


def _gemv(L, _lib, X, pw, Y, ws):
    from flashbfp_b200.linear import gemv_records, records_eligible
    if X.shape[0] == 1 and records_eligible(X, pw):     # one token: the stage-record kernel
        gemv_records(X, pw, Y, ws)
        return
    gemv = L.fbfp_gemv_resident if pw.resident else L.fbfp_gemv
    _lib.check(gemv(_lib.ptr(X), _lib.DTYPE_CODE[X.dtype], X.shape[0], X.stride(0),
                           _lib.ptr(pw.exps), _lib.ptr(pw.signs), _lib.ptr(pw.payload), pw.n_out,
                           pw.k_in, pw.kpad, pw.npad, _lib.ptr(pw.entries if pw.nnz else None),
                           _lib.ptr(pw.seg_ptr if pw.nnz else None), None, 0, _lib.ptr(Y),
                           _lib.DTYPE_CODE[Y.dtype], Y.stride(0), _lib.ptr(ws),
                           _lib.stream_ptr(X.device)), "fbfp_gemv")


def _gemv_fused(L, _lib, X, pw, Y, ws, reducer):
    from flashbfp_b200.linear import gemv_records, records_eligible
    if X.shape[0] == 1 and records_eligible(X, pw):
        gemv_records(X, pw, Y, ws, reducer=reducer)
        return
    _lib.check(L.fbfp_gemv_allreduce(_lib.ptr(X), _lib.DTYPE_CODE[X.dtype], X.shape[0], X.stride(0),
                                     _lib.ptr(pw.exps), _lib.ptr(pw.signs), _lib.ptr(pw.payload), pw.n_out,
                                     pw.k_in, pw.kpad, pw.npad, _lib.ptr(pw.entries if pw.nnz else None),
                                     _lib.ptr(pw.seg_ptr if pw.nnz else None), None, 0, _lib.ptr(Y),
                                     _lib.DTYPE_CODE[Y.dtype], Y.stride(0), _lib.ptr(ws), reducer.handle,
                                     1 if pw.resident else 0, _lib.stream_ptr(X.device)),
               "fbfp_gemv_allreduce")


def run_e2e(args, layers, xs, stream, device, world, rank, step_bytes, exchange, reducer, fused):
    """Public-API step: OABFLinear modules in a CUDA graph; host activations in, outputs out."""
    import torch.distributed as dist
    from flashbfp_b200.linear import OABFLinear, packed_linear_allreduce
    mods = []
    for Ly in layers:
        mm = {}
        for kk in KINDS:
            pw = Ly[kk]
            lin = OABFLinear(pw.k_in, pw.n_out, bias=False)
            lin._pw = pw
            lin.compressed = True
            mm[kk] = lin
        mods.append(mm)
    host_x = {kk: xs[kk].cpu().pin_memory() for kk in KINDS}
    dev_x = {kk: torch.empty_like(xs[kk]) for kk in KINDS}
    last = {}

    def body():
        for mm in mods:
            for kk in KINDS:
                if kk in fused:
                    y = packed_linear_allreduce(dev_x[kk], mm[kk]._pw, reducer)
                else:
                    y = mm[kk](dev_x[kk])
                    if kk in ("o", "down") and world > 1:
                        y = y.float()
                        exchange(y)
                last[kk] = y

    with torch.cuda.stream(stream):
        for kk in KINDS:
            dev_x[kk].copy_(host_x[kk])
        body()
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        body()
    host_y = {kk: torch.empty(last[kk].shape, dtype=last[kk].dtype).pin_memory() for kk in KINDS}
    h2d = sum(t.numel() * t.element_size() for t in host_x.values())
    d2h = sum(t.numel() * t.element_size() for t in host_y.values())

    def step():
        for kk in KINDS:
            dev_x[kk].copy_(host_x[kk], non_blocking=True)
        g.replay()
        for kk in KINDS:
            host_y[kk].copy_(last[kk], non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    K = max(1, args.steps // 2)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record(stream)
        for _ in range(K):
            step()
        b.record(stream)
    torch.cuda.synchronize(device)
    ms = a.elapsed_time(b) / K
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    g.reset()
    del g
    return {"value": round(step_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 5),
            "steps": K, "api": "OABFLinear.forward in a CUDA graph"}


def run_prefill(layers, device, ms=(512, 2048, 8192), iters=5):
    """Prefill (tensor-bound): the gate|up (30720x3840) and down (3840x15360) linears of layer 0
    at M bf16 tokens through packed_linear, on both paths: the fused tcgen05 kernel
    (fbfp_gemm_prefill) and the two-pass one (fbfp_gemm_expanded: expansion of the packed matrix
    into a bf16 scratch, then a cuBLASLt bf16 GEMM), which packed_linear takes where
    ``expanded_preferred`` says so (512 tokens, or 32 when the fused kernel would have fewer tiles
    than SMs); beside cuBLAS bf16 on a dense bf16 weight of the same shape. CUDA events on the
    launching stream; 3 warm-up launches."""
    from flashbfp_b200 import workloads
    from flashbfp_b200.linear import EXPANDED_MIN_M, expanded_preferred, packed_linear, check_device_errors
    peaks = _peaks()

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) / iters

    rows = []
    for kk in ("gate_up", "down"):
        pw = layers[0][kk]
        Wb = (torch.randn(pw.n_out, pw.k_in, device=device) * 0.02).to(torch.bfloat16)
        for m in ms:
            X = workloads.activations(m, pw.k_in, seed=11, device=device)
            Y = torch.empty(m, pw.n_out, dtype=torch.bfloat16, device=device)
            flops = 2.0 * m * pw.n_out * pw.k_in
            ms_f = timed(lambda: packed_linear(X, pw, out=Y, prefill="fused"))
            ms_e = timed(lambda: packed_linear(X, pw, out=Y, prefill="expanded"))
            check_device_errors(device)
            ms_b = timed(lambda: torch.matmul(X, Wb.t()))
            path = "expanded" if expanded_preferred(m, pw, device) else "fused"
            ms_ = ms_e if path == "expanded" else ms_f
            tf = flops / (ms_ * 1e-3) / 1e12
            rows.append({"linear": f"{kk} {pw.n_out}x{pw.k_in}", "m": m, "path": path, "ms": round(ms_, 4),
                         "tflops": round(tf, 1), "frac": round(tf / peaks["bf16_tflops"], 4),
                         "fused_tflops": round(flops / (ms_f * 1e-3) / 1e12, 1),
                         "expanded_tflops": round(flops / (ms_e * 1e-3) / 1e12, 1),
                         "cublas_bf16_tflops": round(flops / (ms_b * 1e-3) / 1e12, 1)})
            del X, Y
        del Wb
    head = next(r for r in rows if r["m"] == 2048 and r["linear"].startswith("gate_up"))
    fused_frac = round(head["fused_tflops"] / peaks["bf16_tflops"], 4)
    return {"workload": "prefill: OABF gate|up and down linears at M = 512, 2048, 8192 bf16 tokens",
            "m": 2048, "path": head["path"], "ms": head["ms"], "tflops": head["tflops"],
            "roofline": {"bound": "tensor", "achieved": head["tflops"], "peak": peaks["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": head["frac"], "peak_source": peaks["source"],
                         "kernel": f"{head['path']} path, gate|up at M=2048 (expanded: expand_x15_kernel "
                                   "+ cuBLASLt bf16 GEMM; fused: prefill_tc_kernel)"},
            "fused": {"kernel": "prefill_tc_kernel", "tflops": head["fused_tflops"], "frac": fused_frac},
            "expanded_min_m": EXPANDED_MIN_M,
            "cublas_bf16_tflops": head["cublas_bf16_tflops"],
            "cublas_bf16_note": "torch.matmul on a dense bf16 weight of the same shape (uncompressed)",
            "sizes": rows}


def run_compress(device, iters=5):
    """GPU compressor (threshold, pack, outlier list) on a gate|up-sized bf16 matrix; HBM-bound,
    reported as input bytes/s and as algorithmic bytes/s (input + 11 B/block + 10 B/outlier)."""
    from flashbfp_b200 import OABFCompressor, workloads
    n, k = 30720, 3840
    W = workloads.decode_weight(n, k, seed=21, device=device)
    comp = OABFCompressor()
    for _ in range(2):
        dp, sp = comp.compress_matrix_device(W)
    torch.cuda.synchronize(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        dp, sp = comp.compress_matrix_device(W)
    b.record()
    torch.cuda.synchronize(device)
    ms = a.elapsed_time(b) / iters
    nb = dp["exponents"].numel()
    inp = 2.0 * n * k
    alg = inp + 11.0 * nb + 10.0 * int(sp["count"])
    return {"workload": f"compress_matrix_device on a {n}x{k} bf16 weight (1.5% StudentT(3) outliers)",
            "ms": round(ms, 4), "input_gbs": round(inp / (ms * 1e-3) / 1e9, 1),
            "algorithmic_gbs": round(alg / (ms * 1e-3) / 1e9, 1), "outliers": int(sp["count"])}


def _decoder(layers, device, reducer, rank, world, batch, prompt, gen):
    """The random-init 12B-class Gemma-3 around the given layers (this rank's parts): 5
    sliding-window layers of 1024 per global one, 16 query / 8 key-value heads of 256, bf16
    embedding and lm_head of 262144 x 3840 (this rank's vocabulary rows). The layers hold
    PackedWeights, or bf16 tensors for the uncompressed baseline."""
    from flashbfp_b200 import tp
    from flashbfp_b200.decode import DecodeLayer, DecoderShape, GemmaDecoder
    H, I, NH, NKV, HD, V = 3840, 15360, 16, 8, 256, 262144
    n = len(layers)
    types = ["full_attention" if (i + 1) % 6 == 0 else "sliding_attention" for i in range(n)]
    shape = DecoderShape(hidden=H, inter=I, n_heads=NH, n_kv_heads=NKV, head_dim=HD, vocab=V,
                         layer_types=types, sliding_window=1024, query_pre_attn_scalar=256.0)
    g = torch.Generator(device=device).manual_seed(11)

    def rnd(*sz, scale):
        return (scale * torch.randn(*sz, generator=g, device=device)).to(torch.bfloat16)

    dls = [DecodeLayer(qkv=Ly["qkv"], o=Ly["o"], gate_up=Ly["gate_up"], down=Ly["down"],
                       input_ln=rnd(H, scale=0.1), post_attn_ln=rnd(H, scale=0.1),
                       pre_ffn_ln=rnd(H, scale=0.1), post_ffn_ln=rnd(H, scale=0.1),
                       q_norm=rnd(HD, scale=0.1), k_norm=rnd(HD, scale=0.1)) for Ly in layers]
    embed, final = rnd(V, H, scale=0.02), rnd(H, scale=0.1)
    v0, v1 = tp.DecoderPlan(NH, NKV, HD, I, V, rank, world).vocab
    lm_head = rnd(V, H, scale=0.02)[v0:v1].clone()
    return GemmaDecoder(shape, dls, embed, final, lm_head, max_ctx=prompt + gen + 1, device=device,
                        max_prefill=prompt, reducer=reducer, vocab_offset=v0, batch=batch)


def run_model_decode(layers, device, reducer=None, rank=0, world=1, batch=1, prompt=128, gen=256,
                     dense=False):
    """Whole decode tokens of the random-init 12B-class Gemma-3: every sequence's ``prompt``
    tokens as one prefill chunk (timed on its own), then ``gen`` greedy tokens for all ``batch``
    sequences together, timed as back-to-back replays of the one-step CUDA graph (max over
    ranks)."""
    import torch.distributed as dist
    dec = _decoder(layers, device, reducer, rank, world, batch, prompt, gen)
    dec.capture()
    gids = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 262144, (prompt,), generator=gids).tolist() for _ in range(batch)]
    dec.reset(0)
    dec.prefill(prompts[0])                     # warm-up of the prompt path, then timed
    dec.reset(0)
    dec.stream.synchronize()
    if world > 1:
        dist.barrier()
    pa, pb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pa.record(dec.stream)
    for b, p in enumerate(prompts):
        dec.prefill(p, seq=b)
    pb.record(dec.stream)
    dec.stream.synchronize()
    prefill_ms = pa.elapsed_time(pb)
    a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(dec.stream)
    for _ in range(gen):
        dec.step()
    b_.record(dec.stream)
    dec.check()
    ms = a.elapsed_time(b_) / gen
    t = torch.tensor([ms, prefill_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, prefill_ms = float(t[0]), float(t[1])
    if dense:
        lin = sum(2 * Ly[kk].numel() for Ly in layers for kk in KINDS)      # bf16 tensors
    else:
        lin = sum(Ly[kk].packed_bytes() for Ly in layers for kk in KINDS)
    H = 3840
    per_rank = lin + 2 * dec.vocab_l * H + 2 * batch * H      # linears, lm_head rows, embedding rows
    dec.release()
    del dec
    torch.cuda.empty_cache()
    return {"workload": (f"random-init 12B-class Gemma-3 decode: {len(layers)} layers (5 sliding-window "
                         "layers of 1024 per global one), 16 q / 8 kv heads x 256, vocab 262144, "
                         f"{prompt} prompt tokens then {gen} greedy tokens, batch {batch}, "
                         f"{'tp%d' % world if world > 1 else '1 GPU'}"
                         + (", uncompressed bf16 linears (cuBLAS)" if dense else ", OABF linears")),
            "batch": batch, "ms_per_step": round(ms, 4),
            "tokens_per_s": round(batch * 1000.0 / ms, 1),
            "prefill_ms": round(prefill_ms, 3),
            "prefill_tokens_per_s": round(batch * prompt * 1000.0 / prefill_ms, 1),
            "weight_gbs_per_rank": round(per_rank / (ms * 1e-3) / 1e9, 1),
            "weight_bytes_per_rank": per_rank,
            "graph": "one CUDA graph per step: linears, decode.cu kernels, bf16 lm_head, greedy pick",
            "lm_head": "uncompressed bf16 through cuBLAS (left alone by the model surgery)"}


def run_models(layers, device, rank, world):
    """Whole-model decode at batch 1 and 8 (tensor-parallel over the ranks), and at one GPU the
    same decoder on uncompressed bf16 linears, with the speed-up over it."""
    out = {}
    dred = None
    if world > 1:
        from flashbfp_b200.tp import NVLinkAllReduce
        dred = NVLinkAllReduce(128 * 3840)          # a 128-token prompt chunk of the residual stream
    for key, batch in (("batch1", 1), ("batch8", 8)):
        if world == 1:
            try:
                out[key] = run_model_decode(layers, device, batch=batch)
            except Exception as e:                  # reported on the line; the headline stands
                out[key] = {"error": f"{type(e).__name__}: {e}"[:300]}
        else:                                       # every rank takes the same collective steps
            out[key] = run_model_decode(layers, device, dred, rank, world, batch)
    if world == 1:
        try:
            dl = dense_layers(len(layers), device)
            out["bf16_batch1"] = run_model_decode(dl, device, dense=True)
            del dl
            torch.cuda.empty_cache()
            if "tokens_per_s" in out.get("batch1", {}):
                r = out["batch1"]["tokens_per_s"] / out["bf16_batch1"]["tokens_per_s"]
                out["speedup_vs_bf16"] = round(r, 3)
                out["speedup_note"] = ("whole-token tokens/s of the OABF decoder over the same decoder on "
                                       "uncompressed bf16 linears (cuBLAS), both one CUDA graph per token; "
                                       "target 3x, weight-byte ceiling of the linears 2.55x")
        except Exception as e:
            out["bf16_batch1"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if dred is not None:
        torch.cuda.synchronize(device)
        dred.close()
    return out


def run_decode_sweep(layers, device, ms=(4, 16), steps=20):
    """The 48-layer linear step at M = 4 and 16 bf16 tokens (one CUDA graph per step, as the
    headline), with per-kind rates from per-kind graphs."""
    res = {}
    for m in ms:
        ms_step, kms, _ = time_linear_step(layers, m, device, 1, None, steps)
        tot = sum(algorithmic_bytes(layers, m, kk) for kk in KINDS)
        res[f"m{m}"] = {"ms_per_step": round(ms_step, 4), "gbs": round(tot / (ms_step * 1e-3) / 1e9, 1),
                        "tokens_per_s_linears": round(m * 1000.0 / ms_step, 1),
                        "layers_gbs": {kk: round(algorithmic_bytes(layers, m, kk) / (kms[kk] * 1e-3) / 1e9, 1)
                                       for kk in KINDS}}
    return res


def dense_layers(n_layers, device):
    """bf16 weights of the 12B-class layer shapes (random, N(0, 0.02)) for the uncompressed
    baseline decoder: q|k|v, o, gate|up, down per layer."""
    shapes = {"qkv": (8192, 3840), "o": (3840, 4096), "gate_up": (30720, 3840), "down": (3840, 15360)}
    g = torch.Generator(device=device).manual_seed(77)
    return [{kk: (0.02 * torch.randn(n, k, generator=g, device=device)).to(torch.bfloat16)
             for kk, (n, k) in shapes.items()} for _ in range(n_layers)]


LLAMA70B = dict(n_heads=64, n_kv_heads=8, head_dim=128, inter=28672, vocab=128256, hidden=8192)


def time_linear_step(layers, m, device, world, reducer, steps):
    """One decode step over `layers` (q|k|v, o, gate|up, down per layer in model order; the
    row-parallel o and down summed over the ranks, fused into the GEMV where every shard takes
    it) as one CUDA graph: (ms per step max over ranks, per-kind ms, kinds fused)."""
    import torch.distributed as dist
    from flashbfp_b200 import _lib
    from flashbfp_b200.linear import fused_shard_eligible
    L = _lib.lib()
    fused = set()
    if world > 1:
        fused = {kk for kk in ("o", "down")
                 if all(fused_shard_eligible(Ly[kk], reducer.max_elems) for Ly in layers)}
        got = [None] * world
        dist.all_gather_object(got, sorted(fused))
        fused = set.intersection(*(set(g) for g in got))
    rowpar = {"o", "down"} if world > 1 else set()
    xs, outs = step_io(layers, m, device, rowpar - fused)
    ws = {kk: torch.zeros(L.fbfp_gemv_workspace_bytes(16, layers[0][kk].npad), dtype=torch.uint8,
                          device=device) for kk in KINDS}

    def one(kk, li):
        Ly = layers[li]
        if kk in fused:
            _gemv_fused(L, _lib, xs[kk], Ly[kk], outs[li][kk], ws[kk], reducer)
        else:
            _gemv(L, _lib, xs[kk], Ly[kk], outs[li][kk], ws[kk])
            if kk in rowpar:
                reducer(outs[li][kk])

    st = torch.cuda.Stream(device)
    st.wait_stream(torch.cuda.current_stream(device))
    graphs = {}
    with torch.cuda.stream(st):
        for li in range(len(layers)):
            for kk in KINDS:
                one(kk, li)
    torch.cuda.synchronize(device)
    for kk in KINDS:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for li in range(len(layers)):
                one(kk, li)
        graphs[kk] = g
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for li in range(len(layers)):
            for kk in KINDS:
                one(kk, li)
    graphs["step"] = g
    with torch.cuda.stream(st):
        for _ in range(3):
            g.replay()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    kreps = max(1, steps // 4)
    t = []
    with torch.cuda.stream(st):
        for gg, reps in [(g, steps)] + [(graphs[kk], kreps) for kk in KINDS]:
            gg.replay()                         # untimed: lines the ranks up
            a_ev, b_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a_ev.record(st)
            for _ in range(reps):
                gg.replay()
            b_ev.record(st)
            b_ev.synchronize()
            t.append(a_ev.elapsed_time(b_ev) / reps)
    torch.cuda.synchronize(device)
    for kk in KINDS:
        _lib.check(L.fbfp_gemv_check(_lib.ptr(ws[kk]), _lib.stream_ptr(device)), "fbfp_gemv_check")
    tt = torch.tensor(t, dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    for gg in graphs.values():
        gg.reset()
    return float(tt[0]), {kk: float(tt[1 + i]) for i, kk in enumerate(KINDS)}, fused


def run_stress70b(device, rank, world, steps=10):
    """70B-class stress (hidden 8192, 64 q / 8 kv heads of 128, MLP 28672): decode M=1 over 80
    layers at 1.5% outliers, tensor-parallel over the ranks; at one GPU also the outlier
    fractions 0.5 / 1.5 / 5% on 8 layers, the prefill GEMM at M = 4096 and the GPU compressor on
    the gate|up matrix. Weights drawn on the GPU shard by shard, never whole on the host."""
    import torch.distributed as dist
    from flashbfp_b200 import OABFCompressor, workloads
    from flashbfp_b200.linear import packed_linear, check_device_errors
    out = {"shape": "hidden 8192, q 8192x8192, k/v 1024x8192, o 8192x8192, gate/up 28672x8192, "
                    "down 8192x28672 per layer"}
    reducer = None
    if world > 1:
        from flashbfp_b200.tp import NVLinkAllReduce
        reducer = NVLinkAllReduce(16 * 8192)
    layers, _ = build_layers(80, rank, world, device, workloads.LLAMA70B_LAYER, LLAMA70B, 0.015, 50000)
    ms, kms, fused = time_linear_step(layers, 1, device, world, reducer, steps)
    b = torch.tensor([algorithmic_bytes(layers, 1, kk) for kk in KINDS], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(b)
    tot = float(b.sum())
    out["decode_m1_80_layers"] = {
        "parallelism": f"tp{world}", "ms_per_step": round(ms, 4),
        "gbs": round(tot / (ms * 1e-3) / 1e9, 1),
        "frac_of_hbm_per_gpu": round(tot / world / (ms * 1e-3) / 1e9 / _peaks()["hbm_gbs"], 4),
        "tokens_per_s_linears": round(1000.0 / ms, 1),
        "layers_gbs_per_rank": {kk: round(float(b[i]) / world / (kms[kk] * 1e-3) / 1e9, 1)
                                for i, kk in enumerate(KINDS)},
        "exchange_fused": sorted(fused), "packed_gb_total": round(tot / 1e9, 2)}
    if world == 1:
        pf = []
        for kk in ("gate_up", "down"):
            pw = layers[0][kk]
            X = workloads.activations(4096, pw.k_in, seed=3, device=device)
            Y = torch.empty(4096, pw.n_out, dtype=torch.bfloat16, device=device)
            for _ in range(2):
                packed_linear(X, pw, out=Y)
            torch.cuda.synchronize(device)
            a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(3):
                packed_linear(X, pw, out=Y)
            c.record()
            torch.cuda.synchronize(device)
            check_device_errors(device)
            t = a.elapsed_time(c) / 3
            tf = 2.0 * 4096 * pw.n_out * pw.k_in / (t * 1e-3) / 1e12
            pf.append({"linear": f"{kk} {pw.n_out}x{pw.k_in}", "m": 4096, "path": "expanded", "ms": round(t, 3),
                       "tflops": round(tf, 1), "frac": round(tf / _peaks()["bf16_tflops"], 4)})
            del X, Y
        out["prefill_m4096"] = pf
        del layers
        torch.cuda.empty_cache()
        W = workloads.decode_weight(57344, 8192, seed=9, device=device)
        comp = OABFCompressor()
        for _ in range(2):
            dp, sp = comp.compress_matrix_device(W)
        torch.cuda.synchronize(device)
        a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(3):
            dp, sp = comp.compress_matrix_device(W)
        c.record()
        torch.cuda.synchronize(device)
        t = a.elapsed_time(c) / 3
        out["compress_gate_up"] = {"matrix": "57344x8192 bf16", "ms": round(t, 3),
                                   "input_gbs": round(2.0 * W.numel() / (t * 1e-3) / 1e9, 1),
                                   "algorithmic_gbs": round((2.0 * W.numel() + 11.0 * dp["exponents"].numel()
                                                             + 10.0 * int(sp["count"])) / (t * 1e-3) / 1e9, 1)}
        del W, dp, sp
        torch.cuda.empty_cache()
        sweep = {}
        for frac in (0.005, 0.015, 0.05):
            ly, _ = build_layers(8, 0, 1, device, workloads.LLAMA70B_LAYER, LLAMA70B, frac, 60000)
            ms8, kms8, _ = time_linear_step(ly, 1, device, 1, None, steps)
            tot8 = sum(algorithmic_bytes(ly, 1, kk) for kk in KINDS)
            sweep[f"{frac * 100:g}%"] = {"ms_per_step_8_layers": round(ms8, 4),
                                         "gbs": round(tot8 / (ms8 * 1e-3) / 1e9, 1),
                                         "outliers_per_layer": int(sum(ly[0][kk].nnz for kk in KINDS)),
                                         "layers_gbs": {kk: round(algorithmic_bytes(ly, 1, kk) / (kms8[kk] * 1e-3) / 1e9, 1)
                                                        for kk in KINDS}}
            del ly
            torch.cuda.empty_cache()
        out["outlier_sweep_m1_8_layers"] = sweep
    else:
        del layers
        torch.cuda.empty_cache()
    if reducer is not None:
        torch.cuda.synchronize(device)
        reducer.close()
    return out


def run_bf16_decode(device, m=1, n_layers=8, iters=50):
    """The same decode step with uncompressed bf16 weights through cuBLAS (F.linear), timed on
    n_layers layers (inputs larger than L2) and scaled to 48 layers; the bf16 baseline that the
    compressed format is meant to beat."""
    from flashbfp_b200 import workloads
    shapes = {"qkv": (8192, 3840), "o": (3840, 4096), "gate_up": (30720, 3840), "down": (3840, 15360)}
    Ws = [{kk: (torch.randn(n, k, device=device) * 0.02).to(torch.bfloat16) for kk, (n, k) in shapes.items()}
          for _ in range(n_layers)]
    xs = {kk: workloads.activations(m, k, seed=3, device=device) for kk, (n, k) in shapes.items()}

    def step():
        for Ly in Ws:
            for kk in shapes:
                torch.nn.functional.linear(xs[kk], Ly[kk])

    for _ in range(3):
        step()
    torch.cuda.synchronize(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        step()
    b.record()
    torch.cuda.synchronize(device)
    ms48 = a.elapsed_time(b) / iters * N_LAYERS / n_layers
    byts = sum(2 * n * k for n, k in shapes.values()) * N_LAYERS
    del Ws
    torch.cuda.empty_cache()
    return {"layers_timed": n_layers, "ms_per_step_48_layers": round(ms48, 4),
            "decode_tokens_per_s": round(m * 1000.0 / ms48, 1),
            "weight_gbs": round(byts / (ms48 * 1e-3) / 1e9, 1),
            "note": "uncompressed bf16 weights, torch F.linear (cuBLAS), eager launches"}


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "source": "measured (MEASURED_PEAKS.json)"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def _traffic(m):
    """DRAM bytes per gate|up launch from the committed ncu summary (None until captured)."""
    p = os.path.join(ROOT, "profiles", "gemv_gate_up_traffic.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d.get(f"m{m}")
    except Exception:
        return None


# --------------------------------------------------------------------------------------
# CPU baseline and reference arm: the torch restatement of the reference's CPU path
# (oracle/cpu_torch.py; same torch operations and dtypes, bit-identical outputs, cost within a
# few percent of the reference's own code where both were timed: oracle/port_calibration.json)
# --------------------------------------------------------------------------------------
def _calibration():
    try:
        with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "oracle",
                               "port_calibration.json")) as f:
            c = json.load(f)
        run = max(c["runs"], key=lambda r: r["threads"])
        return {"forward": run["forward"]["reference_over_port"],
                "compress": run["compress"]["reference_over_port"],
                "measured": f"reference / port time on {c['shape'][0]}x{c['shape'][1]} bf16, "
                            f"{run['threads']} threads, {c['cpus']}-CPU host"}
    except Exception:
        return None


def _timed(fn, seconds, max_iters=1000):
    fn()
    t0 = time.perf_counter()
    it = 0
    while True:
        fn()
        it += 1
        el = time.perf_counter() - t0
        if (el >= seconds and it >= 3) or it >= max_iters:
            return it, el


def cpu_baseline_sample(seconds):
    """The reference's CPU forward (unpack + matmul + outliers) on the full o_proj at M=1 and
    its compressor on the same matrix, on all host threads torch uses."""
    import torch
    from flashbfp_b200 import workloads
    from oracle import cpu_torch
    n, k = 3840, 4096
    W = workloads.decode_weight(n, k, seed=4242)
    X = workloads.activations(1, k, seed=0)
    dp, sp = cpu_torch.compress_matrix(W)
    rcv = cpu_torch.outlier_rcv(sp, dp["padded_shape"], n, k)
    fb = cpu_torch.algorithmic_bytes_forward(dp, sp["count"], 1, 2)
    it, el = _timed(lambda: cpu_torch.fallback_forward(X, dp, rcv), seconds / 2)
    cb = cpu_torch.algorithmic_bytes_compress(W, dp, sp["count"])
    itc, elc = _timed(lambda: cpu_torch.compress_matrix(W), seconds / 2)
    return {"value": round(fb * it / el / 1e9, 4), "unit": "GB/s", "cores": cpu_torch.threads(),
            "kind": "port", "host_cpus": os.cpu_count(),
            "sample": f"o_proj 3840x4096 bf16 OABF at M=1: {it} CPU forwards in {el:.1f} s "
                      "(torch restatement of _cpu_fallback_gemm + outlier index_add_)",
            "compress_gbs": round(cb * itc / elc / 1e9, 4),
            "compress_sample": f"compress_matrix of the same bf16 matrix: {itc} runs in {elc:.1f} s",
            "reference_over_port": _calibration()}


def run_reference(args):
    """Reference arm: the reference's CPU path (torch restatement) on the host cores, same metric;
    one step = the four linears of one 12B-class decoder layer at full size, M tokens."""
    import torch
    from oracle import cpu_torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from flashbfp_b200 import workloads
    layers = []
    for i, (n, k) in enumerate([(8192, 3840), (3840, 4096), (30720, 3840), (3840, 15360)]):
        W = workloads.decode_weight(n, k, seed=9000 + i)
        dp, sp = cpu_torch.compress_matrix(W)
        del W
        rcv = cpu_torch.outlier_rcv(sp, dp["padded_shape"], n, k)
        X = workloads.activations(args.m, k, seed=i)
        layers.append((X, dp, rcv, cpu_torch.algorithmic_bytes_forward(dp, sp["count"], args.m, 2)))
    step_bytes = sum(L[3] for L in layers)

    def step():
        for X, dp, rcv, _ in layers:
            cpu_torch.fallback_forward(X, dp, rcv)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    val = step_bytes * args.steps / el / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(val, 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el * 1000 / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"reference CPU path on one 12B-class decoder layer per step (q|k|v 8192x3840, "
                               f"o 3840x4096, gate|up 30720x3840, down 3840x15360), M={args.m}",
                   "m": args.m, "parallelism": "host cores"},
        "cpu_baseline": {"value": round(val, 4), "unit": "GB/s", "cores": cpu_torch.threads(), "kind": "port",
                         "sample": "the four linears of one decoder layer per step, full size",
                         "reference_over_port": _calibration()},
        "e2e": {"value": round(val, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)
