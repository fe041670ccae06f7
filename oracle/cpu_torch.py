"""Torch restatement of the reference's CPU path, for the timed CPU baseline.

TEST/BENCH INFRASTRUCTURE ONLY: imported by bench.py's CPU-baseline leg and reference arm, by
tests, and by the calibration recipe beside this file. Nothing in the product imports it.

The reference (Ragu-123/FlashBFP, pure Python on torch) is not compiled code, so it cannot be
built into a library that travels with the repository; this module restates the two CPU
routines the reference runs on the host, step by step, with the same torch operations in the
same dtypes, so that it costs what the reference costs on the same host threads:

* ``compress_matrix`` — ``OABFCompressor.compute_dynamic_threshold`` and ``compress_matrix``
  (flash_bfp/compressor.py:11-33 and :34-117): pad, flatten, threshold from mean / variance /
  fourth moment in W's dtype, outlier mask and COO list, per-block shared exponent, 4-bit
  mantissas, sign and nibble packing.
* ``fallback_forward`` — ``OABFLinear.forward`` without a GPU: ``_cpu_fallback_gemm``
  (flash_bfp/triton_kernel.py:89-127: 16 passes that unpack one nibble position each, in the
  activation dtype, then ``X @ W^T``), the outlier product added with ``index_add_``
  (:339-356) and the bias (:358-362).

Both run on torch's intra-op threads (``torch.get_num_threads()``). Their outputs are checked
against the reference-generated fixtures by tests/test_cpu_torch_port.py.
"""
from __future__ import annotations

from typing import Dict, Tuple

import torch


def dynamic_threshold(W: torch.Tensor) -> float:
    """compressor.py:11-33, in W's own dtype (bf16 moments for bf16 weights)."""
    if W.numel() == 0:
        return 0.05
    mu = W.mean()
    var = W.var()
    k4 = ((W - mu) ** 4).mean() / (var ** 2 + 1e-8)
    scale = 2.43 * (1.0 + 0.1 * torch.log(torch.clamp(k4 / 3.0, min=0.5)))
    return float(torch.clamp(var.sqrt() * scale, 0.01, 0.20))


def _padded(n: int, k: int, block: int, tile: int) -> Tuple[int, int]:
    return k + (-k) % block, n + (-n) % tile


def compress_matrix(W: torch.Tensor, block: int = 16, tile: int = 64) -> Tuple[Dict, Dict]:
    """compressor.py:34-117 on the host: the reference's dicts (int8 exponents, int16 signs,
    int32 payload pairs; int32 block index and offset, fp16 values)."""
    if W.numel() == 0:
        raise ValueError("Weight matrix cannot be empty.")
    W = W.detach().cpu()
    n, k = W.shape
    kpad, npad = _padded(n, k, block, tile)
    flat = torch.nn.functional.pad(W, (0, kpad - k, 0, npad - n)).reshape(-1)
    thr = dynamic_threshold(W)
    mask = flat.abs() > thr
    where = torch.nonzero(mask).reshape(-1)
    sparse = {"block_idx": (where // block).to(torch.int32), "offset": (where % block).to(torch.int32),
              "value": flat[where].to(torch.float16), "count": int(where.numel())}
    blocks = torch.where(mask, 0.0, flat).reshape(-1, block)
    amax = blocks.abs().max(dim=1).values
    e = torch.floor(torch.log2(torch.clamp(amax, min=1e-8)))
    denom = torch.where(amax < 1e-7, 1.0, torch.pow(2.0, e))
    mant = torch.clamp(torch.round(blocks.abs() / denom[:, None] * 15.0), 0, 15).to(torch.int32)
    sbits = (blocks < 0).to(torch.int32) << torch.arange(block, dtype=torch.int32)
    nib = mant << (4 * torch.arange(8, dtype=torch.int32)).repeat(2)
    words = torch.stack([nib[:, :8].sum(dim=1), nib[:, 8:].sum(dim=1)], dim=1).to(torch.int32)
    dense = {"exponents": e.to(torch.int8), "signs": sbits.sum(dim=1).to(torch.int16),
             "payload": words, "orig_shape": W.shape, "padded_shape": (kpad, npad)}
    return dense, sparse


def outlier_rcv(sparse: Dict, padded_shape, n: int, k: int):
    """OABFLinear.load_from_weight's cached outlier indices (triton_kernel.py:254-291): input
    row = flat index mod kpad, output column = flat index div kpad, kept inside the layer."""
    if sparse["count"] == 0:
        return None
    kpad = padded_shape[0]
    g = sparse["block_idx"].long() * 16 + sparse["offset"].long()
    r, c = g % kpad, g // kpad
    keep = (r < k) & (c < n)
    return r[keep], c[keep], sparse["value"][keep].to(torch.float32)


def fallback_forward(X: torch.Tensor, dense: Dict, rcv=None, bias: torch.Tensor | None = None) -> torch.Tensor:
    """OABFLinear.forward on the host: triton_kernel.py:89-127, :339-356, :358-362."""
    kpad, npad = dense["padded_shape"]
    n, k = dense["orig_shape"]
    e = dense["exponents"].to(torch.float32)
    s = dense["signs"].to(torch.int32)
    p = dense["payload"].to(torch.int32).reshape(-1, 2)
    Wb = torch.zeros((p.shape[0], 16), dtype=X.dtype)
    for j in range(16):                                   # one nibble position per pass
        m = (p[:, j // 8] >> (4 * (j % 8))) & 0xF
        sign = torch.where(((s >> j) & 1) == 1, -1.0, 1.0)
        Wb[:, j] = sign * (m.to(X.dtype) / 15.0) * torch.pow(2.0, e)
    W = Wb.reshape(npad, kpad)[:n, :k]
    X2 = X.reshape(-1, k)
    Y = torch.matmul(X2, W.t())
    if rcv is not None and rcv[1].numel():
        r, c, v = rcv
        v = v.to(X.dtype)
        if Y.shape[0] == 1:                               # the one-token form: a 1-D index_add_
            Y[0].index_add_(0, c, X2[0, r] * v)
        else:
            Y.index_add_(1, c, X2[:, r] * v[None, :])
    if bias is not None:
        Y = Y + bias                                      # an fp32 bias promotes the output
    return Y.reshape(*X.shape[:-1], n)


def algorithmic_bytes_forward(dense: Dict, count: int, m: int, x_bytes: int) -> int:
    """Bytes a forward must move at least: 11 per 16-weight block, 10 per outlier (int32 index
    pair at the reference's widths would be more), the activations in and the outputs out."""
    n, k = dense["orig_shape"]
    return 11 * int(dense["exponents"].numel()) + 10 * count + x_bytes * m * (k + n)


def algorithmic_bytes_compress(W: torch.Tensor, dense: Dict, count: int) -> int:
    """Bytes the compressor must move at least: W read once, the packed arrays and the COO
    list written once."""
    return W.numel() * W.element_size() + 11 * int(dense["exponents"].numel()) + 10 * count


def threads() -> int:
    return int(torch.get_num_threads())


__all__ = ["dynamic_threshold", "compress_matrix", "outlier_rcv", "fallback_forward",
           "algorithmic_bytes_forward", "algorithmic_bytes_compress", "threads"]
