"""CPU restatement of the FlashBFP OABF algorithm (numpy).

TEST INFRASTRUCTURE ONLY. This module is the checker for the CUDA path: it is
imported by ``tests/``, by ``__graft_entry__.smoke()`` and by the CPU-baseline
leg of ``bench.py``. The product (``flashbfp_b200``) never imports it and has no
CPU fallback.

Every function restates one piece of the reference (Ragu-123/FlashBFP) and cites
the file:line it follows. The reference computes in torch on the CPU with all
arithmetic in the dtype of W; the restatement reproduces those roundings
explicitly:

* element-wise ops and 0-dim ops on bf16 compute in fp32 and round once to
  bf16 (round-to-nearest-even); Python scalars enter arithmetic as fp32;
* comparisons and ``clamp`` round their Python-scalar operand to the tensor
  dtype first (so ``x < 1e-7`` on bf16 compares against bf16(1e-7));
* ``torch.log2`` on the CPU is the correctly rounded fp32 log2 (checked
  exhaustively over every fp32 code in [2^-30, 2^3) and every bf16 code), which
  makes ``floor(log2(x))`` one larger than the exact exponent for the top few
  mantissa codes of each binade;
* ``torch.var`` is an fp64-accumulated unbiased variance rounded once,
  ``torch.mean`` on bf16 is the exact mean rounded once.

Parity pin: the restatement is checked against golden vectors produced by
running the reference itself (``tests/golden/make_golden.py``) and against the
reference live on random inputs in the CPU test-suite. The one known gap is
``torch.mean`` on fp32, which the reference accumulates with torch's float
cascade sum: the restatement uses the exact mean, which moves the fp32
threshold by at most one ulp in rare cases (it never changes a threshold that
is clamped to 0.20, the case for every weight distribution with >=0.5% large
outliers).
"""
from __future__ import annotations

import numpy as np

BLOCK = 16

# --------------------------------------------------------------------------
# rounding helpers
# --------------------------------------------------------------------------

def round_bf16(x) -> np.ndarray:
    """Round fp32 values to bf16 (RNE), returned as fp32 values."""
    a = np.asarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    r = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32)
    out = r.view(np.float32).copy()
    if np.any(nan):
        out = np.where(nan, np.float32(np.nan), out)
    return out


def rnd(x, dt: str):
    """Round a value computed in fp32/fp64 to dtype ``dt`` (via fp32, like torch)."""
    f = np.asarray(x, dtype=np.float32)
    if dt == "fp32":
        return f
    if dt == "bf16":
        return round_bf16(f)
    raise ValueError(f"unsupported dtype {dt}")


def _f32(x):
    return np.float32(x)


def bf16_bits(a) -> np.ndarray:
    """bf16 bit patterns (uint16) of fp32 values that are exactly bf16."""
    return (np.asarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def floor_log2_torch(x: np.ndarray, dt: str) -> np.ndarray:
    """``torch.floor(torch.log2(x))`` in dtype ``dt`` (compressor.py:87).

    torch's CPU log2 is the correctly rounded fp32 log2; for bf16 that fp32
    result is rounded once more to bf16 before ``floor``.
    """
    lg = np.log2(np.asarray(x, dtype=np.float64)).astype(np.float32)
    return np.floor(rnd(lg, dt)).astype(np.float32)


# --------------------------------------------------------------------------
# compressor.py:11-32  compute_dynamic_threshold
# --------------------------------------------------------------------------

def compute_dynamic_threshold(W: np.ndarray, dt: str) -> float:
    """Kurtosis-adaptive outlier threshold (compressor.py:11-32).

    ``W`` holds fp32 values exactly representable in ``dt``. Every step is
    rounded to ``dt`` as the reference's dtype-following torch ops do.
    """
    w = np.asarray(W, dtype=np.float32).reshape(-1)
    n = w.size
    if n == 0:                                   # compressor.py:16-17
        return 0.05
    w64 = w.astype(np.float64)
    with np.errstate(all="ignore"):
        mean = rnd(w64.sum() / n, dt)                                 # :19
        var = rnd(w64.var(ddof=1) if n > 1 else np.nan, dt)           # :20
        std = rnd(np.sqrt(np.float32(var)), dt)                       # :21
        d = rnd(w - np.float32(mean), dt)                             # :24 (W - mean)
        p = rnd(d.astype(np.float64) ** 4, dt)                        # :24 (** 4)
        fourth = rnd(p.astype(np.float64).sum() / n, dt)              # :24 mean
        var2 = rnd(_f32(var) * _f32(var), dt)                         # :25 variance ** 2
        den = rnd(_f32(var2) + _f32(1e-8), dt)                        # :25 + 1e-8
        kurt = rnd(_f32(fourth) / _f32(den), dt)                      # :25
        k3 = rnd(_f32(kurt) / _f32(3.0), dt)                          # :29 kurtosis / 3.0
        half = rnd(0.5, dt)
        k3c = k3 if (np.isnan(k3) or k3 >= half) else half            # clamp(min=0.5)
        lg = rnd(np.float32(np.log(np.float64(k3c))), dt)             # torch.log
        t1 = rnd(_f32(0.1) * _f32(lg), dt)                            # 0.1 * log(.)
        t2 = rnd(_f32(1.0) + _f32(t1), dt)                            # 1.0 + .
        scale = rnd(_f32(2.43) * _f32(t2), dt)                        # base_factor * (.)
        thr = rnd(_f32(std) * _f32(scale), dt)                        # :30
    lo, hi = rnd(0.01, dt), rnd(0.20, dt)                             # :32 clamp (NaN stays)
    if not np.isnan(thr):
        thr = min(max(thr, lo), hi)
    return float(thr)


# --------------------------------------------------------------------------
# compressor.py:34-117  compress_matrix
# --------------------------------------------------------------------------

def padded_dims(n_out: int, k_in: int, block_size: int = 16, tile_size: int = 64):
    """(Kpad, Npad) exactly as compressor.py:49-53 pads them."""
    kpad = k_in if k_in % block_size == 0 else k_in + (block_size - k_in % block_size)
    npad = n_out if n_out % tile_size == 0 else n_out + (tile_size - n_out % tile_size)
    return kpad, npad


def compress_matrix(W: np.ndarray, dt: str, block_size: int = 16, tile_size: int = 64,
                    threshold: float | None = None):
    """OABF compression of W[N_out, K_in] (compressor.py:34-117).

    Returns ``(dense_payload, sparse_outliers)`` with the reference's keys and
    dtypes as numpy arrays: exponents int8[nb], signs int16[nb],
    payload int32[nb, 2]; block_idx int32, offset int32, value float16, count.
    ``threshold`` overrides the computed threshold (used to test packing in
    isolation); ``None`` computes it as the reference does.
    """
    W = np.asarray(W, dtype=np.float32)
    if W.size == 0:
        raise ValueError("Weight matrix cannot be empty.")          # :40-41
    if block_size != BLOCK:
        raise ValueError("only block_size=16 is supported")
    n_out, k_in = W.shape
    kpad, npad = padded_dims(n_out, k_in, block_size, tile_size)
    Wp = np.zeros((npad, kpad), dtype=np.float32)                    # :57 zero pad
    Wp[:n_out, :k_in] = W
    flat = Wp.reshape(-1)                                            # :60 row-major flatten
    thr = compute_dynamic_threshold(W, dt) if threshold is None else threshold  # :64 unpadded W
    thr_dt = rnd(thr, dt)                                            # scalar -> dtype for compare
    with np.errstate(invalid="ignore"):
        mask = np.abs(flat) > thr_dt                                 # :65
    idx = np.nonzero(mask)[0]                                        # :66 ascending
    vals = flat[idx].astype(np.float16)                              # :67,78 -> fp16 (RNE)
    dense = np.where(mask, np.float32(0.0), flat)                    # :69
    nb = flat.size // BLOCK
    blocks = dense.reshape(nb, BLOCK)                                # :83
    bmax = np.abs(blocks).max(axis=1)                                # :86
    e = floor_log2_torch(np.maximum(bmax, rnd(1e-8, dt)), dt)        # :87
    scale = np.where(bmax < rnd(1e-7, dt), np.float32(1.0),
                     np.exp2(e).astype(np.float32))                  # :90
    aligned = np.abs(blocks) / scale[:, None]                        # :91 exact (power of 2)
    q = rnd(aligned * np.float32(15.0), dt)                          # :94 * 15.0 in dtype
    mant = np.clip(np.rint(q), 0, 15).astype(np.int64)               # round half-even, clamp
    sgn = (blocks < 0).astype(np.int64)                              # :97
    sh = np.arange(16, dtype=np.int64)
    signs = ((sgn << sh).sum(axis=1) & 0xFFFF).astype(np.uint16).view(np.int16)      # :100-101
    nib = np.arange(8, dtype=np.int64) * 4
    p0 = ((mant[:, :8] << nib).sum(axis=1) & 0xFFFFFFFF).astype(np.uint32).view(np.int32)
    p1 = ((mant[:, 8:] << nib).sum(axis=1) & 0xFFFFFFFF).astype(np.uint32).view(np.int32)
    payload = np.stack([p0, p1], axis=-1)                            # :104-107
    dense_payload = {
        "exponents": e.astype(np.int8),
        "signs": signs,
        "payload": payload,
        "orig_shape": (n_out, k_in),
        "padded_shape": (kpad, npad),                                # :114 (in-dim first)
    }
    sparse = {
        "block_idx": (idx // BLOCK).astype(np.int32),                # :72,76
        "offset": (idx % BLOCK).astype(np.int32),                    # :73,77
        "value": vals,
        "count": int(idx.size),
    }
    return dense_payload, sparse


# --------------------------------------------------------------------------
# dequantisation: triton_kernel.py:73-80 (fp32 formula), :112-122 (fallback),
# main.py:83-113 (outlier re-insertion)
# --------------------------------------------------------------------------

M_OVER_15_F32 = (np.arange(16, dtype=np.float32) / np.float32(15.0)).astype(np.float32)


def unpack_fields(exps, signs, payload):
    """Per-element (sign, mantissa) and per-block exponent arrays."""
    pay = np.asarray(payload).reshape(-1, 2).view(np.uint32) if np.asarray(payload).dtype == np.int32 \
        else np.asarray(payload).reshape(-1, 2).astype(np.uint32)
    nb = pay.shape[0]
    s = np.asarray(signs).astype(np.int64) & 0xFFFF
    i = np.arange(16)
    sgn = (s[:, None] >> i[None, :]) & 1
    w0 = pay[:, 0].astype(np.int64)
    w1 = pay[:, 1].astype(np.int64)
    mant = np.empty((nb, 16), dtype=np.int64)
    mant[:, :8] = (w0[:, None] >> (4 * i[None, :8])) & 0xF
    mant[:, 8:] = (w1[:, None] >> (4 * i[None, :8])) & 0xF
    e = np.asarray(exps).astype(np.int64)
    return sgn, mant, e


def dequantize_dense(exps, signs, payload, padded_shape, orig_shape, crop=True) -> np.ndarray:
    """fp32 dense weights ``sign * fl(m/15) * 2^e`` (triton_kernel.py:80).

    sign=1 with m=0 yields -0.0, as the reference formula does. Returns
    [Npad, Kpad] or, with ``crop``, [N, K] (triton_kernel.py:124-125).
    """
    kpad, npad = padded_shape
    sgn, mant, e = unpack_fields(exps, signs, payload)
    mag = M_OVER_15_F32[mant] * np.exp2(e).astype(np.float32)[:, None]
    w = np.where(sgn == 1, -mag, mag).astype(np.float32)
    W = w.reshape(npad, kpad)
    if crop:
        n, k = orig_shape
        W = W[:n, :k]
    return W


def dequantize_dense_bf16_fallback(exps, signs, payload, padded_shape, orig_shape) -> np.ndarray:
    """Weights as ``_cpu_fallback_gemm`` builds them for bf16 X (triton_kernel.py:115):
    ``m/15`` is rounded to bf16 before the power-of-two scale."""
    kpad, npad = padded_shape
    sgn, mant, e = unpack_fields(exps, signs, payload)
    m15 = round_bf16(M_OVER_15_F32)
    mag = m15[mant] * np.exp2(e).astype(np.float32)[:, None]
    w = np.where(sgn == 1, -mag, mag).astype(np.float32)
    n, k = orig_shape
    return w.reshape(npad, kpad)[:n, :k]


def outlier_rcv(sparse, padded_shape, in_features: int, out_features: int):
    """Outlier (row r = in-dim, col c = out-dim, value fp32) as OABFLinear.load_from_weight
    derives them (triton_kernel.py:255-287): global index = block_idx*16 + offset,
    r = g % Kpad, c = g // Kpad, kept when r < in_features and c < out_features."""
    kpad, npad = padded_shape
    if sparse["count"] == 0:
        z = np.zeros(0, dtype=np.int64)
        return z, z, np.zeros(0, dtype=np.float32)
    g = sparse["block_idx"].astype(np.int64) * 16 + sparse["offset"].astype(np.int64)
    r = g % kpad
    c = g // kpad
    if (r < 0).any() or (r >= kpad).any():
        raise IndexError("outlier row index out of padded bounds")
    if (c < 0).any() or (c >= npad).any():
        raise IndexError("outlier column index out of padded bounds")
    keep = (r < in_features) & (c < out_features)
    return r[keep], c[keep], sparse["value"][keep].astype(np.float32)


def dequantize_full(dense_payload, sparse) -> np.ndarray:
    """W_full[N, K] fp32 = dense part with outliers written back (main.py:100-113)."""
    n, k = dense_payload["orig_shape"]
    W = dequantize_dense(dense_payload["exponents"], dense_payload["signs"],
                         dense_payload["payload"], dense_payload["padded_shape"],
                         dense_payload["orig_shape"]).copy()
    r, c, v = outlier_rcv(sparse, dense_payload["padded_shape"], k, n)
    W[c, r] = v
    return W


def linear_reference(X: np.ndarray, dense_payload, sparse, bias=None) -> np.ndarray:
    """Exact-math OABFLinear forward: ``X @ W_full^T + bias`` in fp64
    (dequantize-then-matmul, triton_kernel.py:89-127 plus the outlier
    correction :339-356 and bias :358-362)."""
    W = dequantize_full(dense_payload, sparse).astype(np.float64)
    Y = np.asarray(X, dtype=np.float64) @ W.T
    if bias is not None:
        Y = Y + np.asarray(bias, dtype=np.float64)[None, :]
    return Y


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


# --------------------------------------------------------------------------
# torch CPU log2 exception tables (used to check the CUDA constants)
# --------------------------------------------------------------------------

def log2_bump_counts(dt: str, e_lo: int = -30, e_hi: int = 3) -> dict:
    """For each binade e: how many of its top mantissa codes have
    ``floor(log2(x)) == e + 1`` under the restated torch semantics."""
    out = {}
    if dt == "fp32":
        top = np.arange((1 << 23) - 64, 1 << 23, dtype=np.uint32)
        for e in range(e_lo, e_hi + 1):
            x = (top + np.uint32((e + 127) << 23)).view(np.float32)
            out[e] = int((floor_log2_torch(x, dt) != e).sum())
    else:
        top = np.arange(0, 128, dtype=np.uint32)
        for e in range(e_lo, e_hi + 1):
            x = ((top + np.uint32((e + 127) << 7)) << 16).view(np.float32)
            out[e] = int((floor_log2_torch(x, dt) != e).sum())
    return out
