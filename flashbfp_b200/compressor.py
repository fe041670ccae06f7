"""OABFCompressor on the GPU, with the reference's API and output bytes.

Mirrors ``flash_bfp.compressor.OABFCompressor`` (flash_bfp/compressor.py:5-117):
same constructor, ``compute_dynamic_threshold(W) -> float`` and
``compress_matrix(W) -> (dense_payload, sparse_outliers)`` with identical keys, dtypes and
bytes. The work runs in CUDA kernels (libflashbfp.so: fbfp_compress_*); CPU inputs are
copied to the current CUDA device first, and the public ``compress_matrix`` returns CPU
tensors like the reference. ``compress_matrix_device`` keeps the results on the device.
"""
from __future__ import annotations

from typing import Dict, Tuple

import torch

from . import _lib


def padded_dims(n_out: int, k_in: int, block_size: int, tile_size: int) -> Tuple[int, int]:
    """(Kpad, Npad): K padded to a multiple of block_size, N to a multiple of tile_size
    (compressor.py:49-53)."""
    r = k_in % block_size
    kpad = k_in if r == 0 else k_in + (block_size - r)
    c = n_out % tile_size
    npad = n_out if c == 0 else n_out + (tile_size - c)
    return kpad, npad


def _device_input(W: torch.Tensor) -> torch.Tensor:
    if W.device.type == "meta":
        W = torch.zeros(W.shape, dtype=W.dtype)
    if not W.is_cuda:
        if not torch.cuda.is_available():
            raise RuntimeError("OABFCompressor runs on the GPU: no CUDA device is available "
                               "(FlashBFP-B200 has no CPU fallback)")
        W = W.to(torch.cuda.current_device())
    if W.dtype not in (torch.float32, torch.bfloat16):
        raise NotImplementedError(f"OABFCompressor: weights of dtype {W.dtype} are not supported "
                                  "(float32 and bfloat16 are)")
    if W.dim() != 2:
        raise ValueError(f"OABFCompressor expects a 2-D weight matrix, got shape {tuple(W.shape)}")
    if W.stride(1) != 1:
        W = W.contiguous()
    return W.detach()


class OABFCompressor:
    def __init__(self, block_size: int = 16, tile_size: int = 64, variance_threshold: float = 1e-5):
        self.block_size = block_size
        self.tile_size = tile_size
        self.variance_threshold = variance_threshold   # unused, as in the reference

    def _check_sizes(self):
        if self.block_size != 16:
            raise ValueError(f"OABF packing is defined for block_size=16 (got {self.block_size})")
        if self.tile_size < 1:
            raise ValueError(f"tile_size must be positive (got {self.tile_size})")

    # -- compressor.py:11-32 ------------------------------------------------------------
    def _threshold_device(self, W: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        L = _lib.lib()
        n, k = W.shape
        kpad, npad = padded_dims(n, k, 16, max(self.tile_size, 1))
        scratch = torch.empty(L.fbfp_compress_scratch_bytes(n, k, kpad, npad), dtype=torch.uint8,
                              device=W.device)
        thr = torch.empty(1, dtype=torch.float32, device=W.device)
        _lib.check(L.fbfp_compress_threshold(_lib.ptr(W), _lib.DTYPE_CODE[W.dtype], n, k, W.stride(0),
                                             _lib.ptr(thr), _lib.ptr(scratch),
                                             _lib.stream_ptr(W.device)), "fbfp_compress_threshold")
        return thr, scratch

    def compute_dynamic_threshold(self, W: torch.Tensor) -> float:
        if W.numel() == 0:
            return 0.05
        W = _device_input(W)
        thr, _ = self._threshold_device(W)
        return float(thr.item())

    # -- compressor.py:34-117 -----------------------------------------------------------
    def compress_matrix_device(self, W: torch.Tensor, threshold: float | None = None):
        """Like ``compress_matrix`` but every tensor stays on the CUDA device.

        ``threshold`` (optional) replaces the computed threshold, e.g. to compress shards
        of a matrix with the statistics of the whole matrix."""
        if W.numel() == 0:
            raise ValueError("Weight matrix cannot be empty.")
        self._check_sizes()
        W = _device_input(W)
        L = _lib.lib()
        dev = W.device
        n, k = W.shape
        kpad, npad = padded_dims(n, k, 16, self.tile_size)
        nb = npad * kpad // 16
        st = _lib.stream_ptr(dev)
        if threshold is None:
            thr, scratch = self._threshold_device(W)
        else:
            thr = torch.tensor([threshold], dtype=torch.float32, device=dev)
            scratch = None
        need = L.fbfp_compress_scratch_bytes(n, k, kpad, npad)
        if scratch is None or scratch.numel() < need:
            scratch = torch.empty(need, dtype=torch.uint8, device=dev)
        exps = torch.empty(nb, dtype=torch.int8, device=dev)
        signs = torch.empty(nb, dtype=torch.int16, device=dev)
        payload = torch.empty(nb, 2, dtype=torch.int32, device=dev)
        row_off = torch.empty(npad + 1, dtype=torch.int32, device=dev)
        dt = _lib.DTYPE_CODE[W.dtype]
        _lib.check(L.fbfp_compress_pack(_lib.ptr(W), dt, n, k, W.stride(0), kpad, npad, _lib.ptr(thr),
                                        _lib.ptr(exps), _lib.ptr(signs), _lib.ptr(payload),
                                        _lib.ptr(row_off), _lib.ptr(scratch), st), "fbfp_compress_pack")
        count = int(row_off[npad].item())
        bidx = torch.empty(count, dtype=torch.int32, device=dev)
        off = torch.empty(count, dtype=torch.int32, device=dev)
        val = torch.empty(count, dtype=torch.float16, device=dev)
        if count:
            _lib.check(L.fbfp_compress_outliers(_lib.ptr(W), dt, n, k, W.stride(0), kpad, npad,
                                                _lib.ptr(row_off), _lib.ptr(bidx), _lib.ptr(off),
                                                _lib.ptr(val), _lib.ptr(scratch), st),
                       "fbfp_compress_outliers")
        dense_payload = {
            "exponents": exps,
            "signs": signs,
            "payload": payload,
            "orig_shape": torch.Size((n, k)),
            "padded_shape": (kpad, npad),
        }
        sparse_outliers = {"block_idx": bidx, "offset": off, "value": val, "count": count}
        return dense_payload, sparse_outliers

    def compress_matrix(self, W: torch.Tensor) -> Tuple[Dict, Dict]:
        """Reference-compatible result: CPU tensors with the reference's dtypes and bytes."""
        dp, sp = self.compress_matrix_device(W)
        dense_payload = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in dp.items()}
        sparse_outliers = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in sp.items()}
        return dense_payload, sparse_outliers


def _main(argv=None) -> None:
    """``python -m flashbfp_b200.compressor [N K [reps]]``: time ``compress_matrix_device`` on a
    seeded N x K bf16 weight (N(0, 0.02) with 1.5% heavy-tailed outliers) on the current GPU,
    after two warm-up calls; prints the time per call and the bytes moved per second."""
    import json
    import sys
    from . import workloads
    args = [int(a) for a in (sys.argv[1:] if argv is None else argv)]
    n, k = (args[0], args[1]) if len(args) >= 2 else (30720, 3840)
    reps = args[2] if len(args) >= 3 else 5
    dev = torch.device("cuda", torch.cuda.current_device())
    W = workloads.decode_weight(n, k, seed=21, device=dev)
    comp = OABFCompressor()
    for _ in range(2):
        dp, sp = comp.compress_matrix_device(W)
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        dp, sp = comp.compress_matrix_device(W)
    b.record()
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / reps
    alg = 2.0 * n * k + 11.0 * dp["exponents"].numel() + 10.0 * int(sp["count"])
    print(json.dumps({"shape": [n, k], "ms": round(ms, 4), "input_gbs": round(2.0 * n * k / ms / 1e6, 1),
                      "algorithmic_gbs": round(alg / ms / 1e6, 1), "outliers": int(sp["count"])}))


if __name__ == "__main__":
    _main()
