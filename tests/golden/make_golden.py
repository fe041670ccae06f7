"""Generate the golden OABF fixtures by running the reference implementation.

Run in a container where the reference package (Ragu-123/FlashBFP,
``flash_bfp``) is importable::

    python tests/golden/make_golden.py --reference /path/to/FlashBFP

Every fixture is produced by the reference's own code, unmodified:
``OABFCompressor.compute_dynamic_threshold`` / ``compress_matrix``
(compressor.py:11-117), ``_cpu_fallback_gemm`` (triton_kernel.py:89-127, whose
dequantised weight matrix is captured by wrapping ``torch.matmul`` for the one
call) and ``OABFLinear.load_from_weight`` / ``forward`` / ``state_dict``
(triton_kernel.py:218-379). The reference runs on the CPU here, so
``oabf_gemm`` takes its CPU fallback path.

Outputs ``tests/golden/<case>.npz`` (small matrices) and
``tests/golden/fullsize.json`` (digests of the packed bytes for the full-size
4096x4096 workload, regenerated from its seed by the tests).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # repo root
from flashbfp_b200 import workloads  # noqa: E402


def _bits_bf16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _capture_fallback_weights(fallback, X, dense_payload):
    """Run the reference ``_cpu_fallback_gemm`` and capture the W it builds."""
    captured = {}
    real = torch.matmul

    def spy(a, b, *args, **kw):
        captured["Wt"] = b.detach().clone()
        return real(a, b, *args, **kw)

    torch.matmul = spy
    try:
        Y = fallback(X, dense_payload)
    finally:
        torch.matmul = real
    return Y, captured["Wt"].t().contiguous()


def run_case(ref, name, W: torch.Tensor, xs, bias_seed=None):
    comp = ref.OABFCompressor(block_size=16, tile_size=64)
    dt = "bf16" if W.dtype == torch.bfloat16 else "fp32"
    thr = comp.compute_dynamic_threshold(W)
    dp, sp = comp.compress_matrix(W)
    n, k = W.shape
    rec = {
        "dtype": np.array(dt),
        "W": W.float().numpy(),
        "threshold": np.array(thr, dtype=np.float64),
        "exponents": dp["exponents"].numpy(),
        "signs": dp["signs"].numpy(),
        "payload": dp["payload"].numpy(),
        "orig_shape": np.array(tuple(dp["orig_shape"]), dtype=np.int64),
        "padded_shape": np.array(tuple(dp["padded_shape"]), dtype=np.int64),
        "block_idx": sp["block_idx"].numpy(),
        "offset": sp["offset"].numpy(),
        "value_bits": sp["value"].numpy().view(np.uint16),
        "count": np.array(sp["count"], dtype=np.int64),
    }
    # dequantised dense weights exactly as the reference fallback builds them
    for xdt, key in ((torch.float32, "Wdeq_f32"), (torch.bfloat16, "Wdeq_bf16fb")):
        X0 = torch.zeros(1, k, dtype=xdt)
        _, Wd = _capture_fallback_weights(ref.tk._cpu_fallback_gemm, X0, dp)
        rec[key] = Wd.float().numpy()
    # OABFLinear: outlier (r, c, v) cache, forward outputs and state_dict
    has_bias = bias_seed is not None
    lin = ref.OABFLinear(k, n, bias=has_bias)
    if has_bias:
        g = torch.Generator().manual_seed(bias_seed)
        with torch.no_grad():
            lin.bias.copy_(torch.randn(n, generator=g) * 0.1)
        rec["bias"] = lin.bias.detach().numpy().copy()
    lin.load_from_weight(W, comp, torch.device("cpu"))
    if lin._sp_r_idx is not None:
        rec["r_idx"] = lin._sp_r_idx.numpy()
        rec["c_idx"] = lin._sp_c_idx.numpy()
        rec["v_val"] = lin._sp_v_val.numpy()
    for i, X in enumerate(xs):
        with torch.no_grad():
            Y = lin(X)
        rec[f"X{i}"] = X.float().numpy()
        rec[f"X{i}_dtype"] = np.array("bf16" if X.dtype == torch.bfloat16 else "fp32")
        rec[f"Y{i}"] = Y.float().numpy()
    sd = lin.state_dict()
    rec["state_dict_keys"] = np.array(sorted(sd.keys()))
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **rec)
    return thr, sp["count"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of the reference project (the directory holding flash_bfp/)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import flash_bfp  # noqa: F401
    import flash_bfp.triton_kernel as tk
    from flash_bfp import OABFCompressor, OABFLinear

    class Ref:
        pass
    ref = Ref()
    ref.OABFCompressor, ref.OABFLinear, ref.tk = OABFCompressor, OABFLinear, tk
    torch.set_num_threads(1)

    summary = {}
    for name, (W, xs, bias_seed) in workloads.golden_cases().items():
        thr, cnt = run_case(ref, name, W, xs, bias_seed)
        summary[name] = (thr, cnt)
        print(f"{name:24s} {tuple(W.shape)} {str(W.dtype):15s} thr={thr!r} outliers={cnt}")

    # full-size config: digests only (the tests regenerate W from its seed)
    full = {}
    for name, W in workloads.fullsize_cases().items():
        comp = OABFCompressor(16, 64)
        torch.set_num_threads(os.cpu_count() or 1)
        dp, sp = comp.compress_matrix(W)
        thr = comp.compute_dynamic_threshold(W)
        ex = dp["exponents"].numpy()
        full[name] = {
            "shape": list(W.shape),
            "dtype": "bf16" if W.dtype == torch.bfloat16 else "fp32",
            "threshold": thr,
            "count": int(sp["count"]),
            "exp_min": int(ex.min()), "exp_max": int(ex.max()),
            "sha256_exponents": hashlib.sha256(ex.tobytes()).hexdigest(),
            "sha256_signs": hashlib.sha256(dp["signs"].numpy().tobytes()).hexdigest(),
            "sha256_payload": hashlib.sha256(dp["payload"].numpy().tobytes()).hexdigest(),
            "sha256_block_idx": hashlib.sha256(sp["block_idx"].numpy().tobytes()).hexdigest(),
            "sha256_offset": hashlib.sha256(sp["offset"].numpy().tobytes()).hexdigest(),
            "sha256_value": hashlib.sha256(sp["value"].numpy().tobytes()).hexdigest(),
        }
        print(name, {k: v for k, v in full[name].items() if not k.startswith("sha")})
    with open(os.path.join(HERE, "fullsize.json"), "w") as f:
        json.dump(full, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
