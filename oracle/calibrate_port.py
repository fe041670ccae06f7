"""Calibrate the torch restatement of the reference's CPU path against the reference itself.

TEST/BENCH INFRASTRUCTURE ONLY. Run where a checkout of the reference is available:

    python oracle/calibrate_port.py --reference /path/to/FlashBFP

It imports the reference package from that checkout (unmodified, through its public API:
``OABFCompressor.compress_matrix`` and ``OABFLinear.load_from_weight`` + ``forward`` on CPU
tensors, which take ``_cpu_fallback_gemm``), times it and ``oracle/cpu_torch.py`` on the same
inputs with the same number of torch threads, checks that both give the same bytes / outputs,
and writes the times and their ratio to ``oracle/port_calibration.json``. bench.py reports that
ratio beside the port's CPU timing, so the reference's own cost on the GPU box's host cores can
be read off as port time x ratio.
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def _best(fn, reps):
    fn()
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        best = min(best, time.perf_counter() - t0)
    return best


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of the reference project (the directory holding flash_bfp/)")
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from flash_bfp import OABFCompressor, OABFLinear

    from flashbfp_b200 import workloads
    from oracle import cpu_torch

    n, k = 3840, 4096                                     # o_proj of the 12B-class layer
    W = workloads.decode_weight(n, k, seed=4242)          # bf16
    X = workloads.activations(1, k, seed=1)               # bf16, one token
    out = {"shape": [n, k], "w_dtype": "bf16", "x_dtype": "bf16", "m": 1,
           "host": platform.processor() or platform.machine(), "cpus": os.cpu_count(),
           "torch": torch.__version__, "runs": []}
    for threads in sorted({1, os.cpu_count() or 1}):
        torch.set_num_threads(threads)
        comp = OABFCompressor()
        ref_dp, ref_sp = comp.compress_matrix(W)
        dp, sp = cpu_torch.compress_matrix(W)
        assert torch.equal(ref_dp["payload"], dp["payload"]) and torch.equal(ref_dp["signs"], dp["signs"])
        assert torch.equal(ref_dp["exponents"], dp["exponents"]) and ref_sp["count"] == sp["count"]
        t_ref_c = _best(lambda: comp.compress_matrix(W), args.reps)
        t_port_c = _best(lambda: cpu_torch.compress_matrix(W), args.reps)

        lin = OABFLinear(k, n, bias=False)
        lin.load_from_weight(W, comp, torch.device("cpu"))
        rcv = cpu_torch.outlier_rcv(sp, dp["padded_shape"], n, k)
        with torch.no_grad():
            y_ref = lin(X)
        y_port = cpu_torch.fallback_forward(X, dp, rcv)
        assert torch.equal(y_ref, y_port), "port and reference forward differ"
        with torch.no_grad():
            t_ref_f = _best(lambda: lin(X), args.reps)
        t_port_f = _best(lambda: cpu_torch.fallback_forward(X, dp, rcv), args.reps)
        run = {"threads": threads,
               "compress": {"reference_s": round(t_ref_c, 4), "port_s": round(t_port_c, 4),
                            "reference_over_port": round(t_ref_c / t_port_c, 3)},
               "forward": {"reference_s": round(t_ref_f, 4), "port_s": round(t_port_f, 4),
                           "reference_over_port": round(t_ref_f / t_port_f, 3)}}
        out["runs"].append(run)
        print(json.dumps(run))
    with open(os.path.join(HERE, "port_calibration.json"), "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()
