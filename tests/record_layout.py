"""CPU model of the decode GEMV's stage-record layout (csrc/gemv_rec.cu), for tests.

``outlier_tiles`` restates the outlier layout of csrc/outliers.cu (entries grouped by 128-row
group and 256-column stage, per-row starts); ``build_records`` restates fbfp_records_build (offset
table, 5-bit fields, biased exponents, each record's outliers); ``decode_records`` restates the
kernel's dequantisation (the bf16 pair (K | f) - C with K = eb * 0x00800080, C = K + 0x00100010).
The layout and the bit arithmetic are checked against the oracle without a GPU, and the
GPU-built records are compared byte for byte with this model.
"""
from __future__ import annotations

import numpy as np

FIELDS = 20480
EXP_OFF = 20480
ROFF_OFF = 22528
ENT_OFF = 22816
SUB = 5120


def n_units(npad: int, kpad: int) -> int:
    return ((npad + 127) // 128) * (kpad // 256)


def table_bytes(units: int) -> int:
    return ((units + 1) * 8 + 255) // 256 * 256


def outlier_tiles(block_idx, offset, value_bits, npad: int, kpad: int, n_out: int, k_in: int):
    """(entries uint32[], seg_ptr int32[units + 1], roff uint16[units, 136]) of the COO list."""
    n_stages = kpad // 256
    units = n_units(npad, kpad)
    g = np.asarray(block_idx).astype(np.int64) * 16 + np.asarray(offset).astype(np.int64)
    n, k = g // kpad, g % kpad
    keep = (k < k_in) & (n < n_out)
    n, k = n[keep], k[keep]
    v = np.asarray(value_bits).astype(np.uint32)[keep] & 0xFFFF
    u = (n // 128) * n_stages + k // 256
    r = n % 128
    order = np.lexsort((k, r, u))                     # by unit, then row, then column
    u, r, k, v = u[order], r[order], k[order], v[order]
    entries = (v | ((k % 256).astype(np.uint32) << 16) | (r.astype(np.uint32) << 24)).astype(np.uint32)
    counts = np.bincount(u, minlength=units)
    seg_ptr = np.zeros(units + 1, dtype=np.int64)
    seg_ptr[1:] = np.cumsum(counts)
    roff = np.zeros((units, 136), dtype=np.uint16)
    for uu in range(units):
        rows = r[seg_ptr[uu]:seg_ptr[uu + 1]]
        rc = np.bincount(rows, minlength=128)
        roff[uu, 1:129] = np.cumsum(rc)
    return entries, seg_ptr.astype(np.int32), roff


def _fields(exps, signs, payload):
    pay = np.asarray(payload).reshape(-1, 2).view(np.uint32).astype(np.int64)
    s = np.asarray(signs).astype(np.int64) & 0xFFFF
    i = np.arange(16)
    sgn = (s[:, None] >> i[None, :]) & 1
    mant = np.empty((pay.shape[0], 16), dtype=np.int64)
    mant[:, :8] = (pay[:, :1] >> (4 * i[None, :8])) & 0xF
    mant[:, 8:] = (pay[:, 1:] >> (4 * i[None, :8])) & 0xF
    f = np.where(sgn == 1, 16 - mant, 16 + mant)
    eb = (np.asarray(exps).astype(np.int64) + 134) & 0xFF
    return eb, f


def build_records(exps, signs, payload, npad: int, kpad: int, tiles=None) -> np.ndarray:
    """The records buffer as fbfp_records_build writes it (only the bytes it defines; the build
    zero-fills the allocation first, and the buffer here ends at the table's end offset)."""
    assert kpad % 256 == 0
    kb = kpad // 16
    n_stages = kpad // 256
    units = n_units(npad, kpad)
    if tiles is None:
        seg_ptr = np.zeros(units + 1, dtype=np.int64)
        entries = np.zeros(0, dtype=np.uint32)
        roff = np.zeros((units, 136), dtype=np.uint16)
    else:
        entries, seg_ptr, roff = tiles
        seg_ptr = np.asarray(seg_ptr).astype(np.int64)
    groups = (seg_ptr[1:] - seg_ptr[:-1] + 3) // 4
    pre = np.zeros(units + 1, dtype=np.int64)
    pre[1:] = np.cumsum(groups)
    table = table_bytes(units) + np.arange(units + 1, dtype=np.int64) * ENT_OFF + 16 * pre
    out = np.zeros(int(table[-1]), dtype=np.uint8)
    out[:8 * (units + 1)] = np.frombuffer(table.astype(np.int64).tobytes(), dtype=np.uint8)
    eb, f = _fields(exps, signs, payload)
    eb = eb.reshape(npad, kb)
    f = f.reshape(npad, kb // 2, 2, 16)                 # [row][block pair][block][element]
    w = np.zeros((npad, kb // 2, 5), dtype=np.int64)
    for b in range(2):
        for el in range(16):
            P = 8 * b + el // 2
            hi = 16 * (el & 1)
            fv = f[:, :, b, el]
            if P < 15:
                w[:, :, P // 3] |= fv << (5 * (P % 3) + hi)
            else:
                for k in range(5):
                    w[:, :, k] |= ((fv >> k) & 1) << (15 + hi)
    w32 = (w & 0xFFFFFFFF).astype(np.uint32)
    for n in range(npad):
        g, row = n >> 7, n & 127
        for bp in range(kb // 2):
            st, pp = bp >> 3, bp & 7
            c, h = pp >> 1, pp & 1
            base = int(table[g * n_stages + st])
            sb = base + c * SUB
            for j in range(5):
                wi = 5 * h + j
                chunk, within = wi >> 2, wi & 3
                off = sb + chunk * 2048 + row * (16 if chunk < 2 else 8) + within * 4
                out[off:off + 4] = np.frombuffer(w32[n, bp, j].tobytes(), dtype=np.uint8)
            for b in range(2):
                out[base + EXP_OFF + c * 512 + row * 4 + 2 * h + b] = eb[n, 2 * bp + b]
    for u in range(units):
        base = int(table[u])
        out[base + ROFF_OFF:base + ROFF_OFF + 272] = np.frombuffer(roff[u].astype(np.uint16).tobytes(), dtype=np.uint8)
        e = np.asarray(entries[seg_ptr[u]:seg_ptr[u + 1]], dtype=np.uint32)
        out[base + ENT_OFF:base + ENT_OFF + 4 * e.size] = np.frombuffer(e.tobytes(), dtype=np.uint8)
    return out


def _bf16(bits):
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


def decode_records(rec: np.ndarray, npad: int, kpad: int) -> np.ndarray:
    """float32 [npad, kpad] of s*m*2^e as the kernel's A operands hold them (the 1/15 excluded)."""
    kb = kpad // 16
    n_stages = kpad // 256
    units = n_units(npad, kpad)
    table = rec[:8 * (units + 1)].view(np.int64)
    out = np.zeros((npad, kpad), dtype=np.float32)
    words = rec[: (rec.size // 4) * 4].view(np.uint32)
    for n in range(npad):
        g, row = n >> 7, n & 127
        for bp in range(kb // 2):
            st, pp = bp >> 3, bp & 7
            c, h = pp >> 1, pp & 1
            base = int(table[g * n_stages + st])
            sb = base + c * SUB
            w = []
            for j in range(5):
                wi = 5 * h + j
                chunk, within = wi >> 2, wi & 3
                off = sb + chunk * 2048 + row * (16 if chunk < 2 else 8) + within * 4
                w.append(int(words[off // 4]))
            ebs = [int(rec[base + EXP_OFF + c * 512 + row * 4 + 2 * h + b]) for b in range(2)]
            spare = (((w[0] >> 15) & 0x00010001) | ((w[1] >> 14) & 0x00020002) | ((w[2] >> 13) & 0x00040004)
                     | ((w[3] >> 12) & 0x00080008) | ((w[4] >> 11) & 0x00100010))
            for b in range(2):
                K = (ebs[b] * 0x00800080) & 0xFFFFFFFF
                C = K + 0x00100010
                for j in range(8):
                    P = 8 * b + j
                    fl = ((w[P // 3] >> (5 * (P % 3))) & 0x001F001F) if P < 15 else spare
                    v = fl | K
                    lo = _bf16(v & 0xFFFF) - _bf16(C & 0xFFFF)       # exact in bf16
                    hi = _bf16(v >> 16) - _bf16(C >> 16)
                    k0 = 16 * (2 * bp + b) + 2 * j
                    out[n, k0] = lo
                    out[n, k0 + 1] = hi
    return out


def decode_outliers(rec: np.ndarray, npad: int, kpad: int):
    """The outliers the records hold, as (row n, column k, fp16 bits) sorted by flat index."""
    n_stages = kpad // 256
    units = n_units(npad, kpad)
    table = rec[:8 * (units + 1)].view(np.int64)
    rows, cols, vals = [], [], []
    for u in range(units):
        base = int(table[u])
        ro = rec[base + ROFF_OFF:base + ROFF_OFF + 272].view(np.uint16)
        cnt = int(ro[128])
        e = rec[base + ENT_OFF:base + ENT_OFF + 4 * cnt].view(np.uint32)
        g, st = u // n_stages, u % n_stages
        for r in range(128):
            for x in e[ro[r]:ro[r + 1]]:
                assert (int(x) >> 24) == r
                rows.append(g * 128 + r)
                cols.append(st * 256 + ((int(x) >> 16) & 0xFF))
                vals.append(int(x) & 0xFFFF)
    rows, cols, vals = np.array(rows, dtype=np.int64), np.array(cols, dtype=np.int64), np.array(vals)
    o = np.argsort(rows * kpad + cols, kind="stable")
    return rows[o], cols[o], vals[o]
