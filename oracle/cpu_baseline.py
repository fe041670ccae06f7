"""CPU port of the reference's OABFLinear forward path, for the timed CPU baseline.

TEST/BENCH INFRASTRUCTURE ONLY (imported by bench.py's CPU-baseline leg and by tests).

Restates, with vectorised numpy on the host cores, what the reference runs when it has no
usable GPU: ``_cpu_fallback_gemm`` (flash_bfp/triton_kernel.py:89-127 — unpack the 16
nibbles of every block with 16 vectorised passes, scale by 2^e, crop, then ``X @ W^T``)
followed by the outlier ``index_add_`` (:339-356) and the bias add (:358-362). Arithmetic
is fp32 (numpy has no bf16); BLAS threads are whatever numpy's BLAS uses on the host.
"""
from __future__ import annotations

import numpy as np


def unpack_dense(exps: np.ndarray, signs: np.ndarray, payload: np.ndarray, padded_shape, orig_shape):
    kpad, npad = padded_shape
    nb = exps.shape[0]
    pay = payload.reshape(nb, 2).view(np.uint32)
    s = signs.view(np.uint16).astype(np.uint32)
    scale = np.exp2(exps.astype(np.float32))
    out = np.empty((nb, 16), dtype=np.float32)
    for i in range(8):                                          # triton_kernel.py:112-116
        m = ((pay[:, 0] >> (4 * i)) & 0xF).astype(np.float32)
        sg = np.where((s >> i) & 1, np.float32(-1.0), np.float32(1.0))
        out[:, i] = sg * (m / np.float32(15.0)) * scale
    for i in range(8):                                          # :118-122
        m = ((pay[:, 1] >> (4 * i)) & 0xF).astype(np.float32)
        sg = np.where((s >> (i + 8)) & 1, np.float32(-1.0), np.float32(1.0))
        out[:, i + 8] = sg * (m / np.float32(15.0)) * scale
    n, k = orig_shape
    return out.reshape(npad, kpad)[:n, :k]                      # :124-125


def fallback_forward(X: np.ndarray, exps, signs, payload, padded_shape, orig_shape,
                     r_idx=None, c_idx=None, v_val=None, bias=None) -> np.ndarray:
    W = unpack_dense(exps, signs, payload, padded_shape, orig_shape)
    Y = X.astype(np.float32) @ W.T                              # :127
    if r_idx is not None and len(r_idx):
        prod = X[:, r_idx].astype(np.float32) * v_val[None, :]  # :352-356
        np.add.at(Y, (slice(None), c_idx), prod)
    if bias is not None:
        Y = Y + bias[None, :]
    return Y
