"""Device-resident OABF matrices: container, fused-row concatenation and TP shards.

A ``PackedWeight`` holds the reference's packed arrays on the device — exponents
int8[npad*kb], signs int16[npad*kb], payload int32[npad*kb, 2], block b = n*kb + j — plus
the outlier list in COO form (block index, offset, fp16 bits; ascending flat order) and in
the (128-row group, 256-column stage) form the fused kernels read, and, on request
(``build_records``), the stage records of ``fbfp_gemv_records`` (one contiguous record per
128-row group and 256-column stage with its weights, 11 bytes per 16, and its outliers).

Row concatenation serves fused launches (q|k|v, gate|up share their input); row and
block-column slices serve tensor parallelism. Because the outlier threshold is a
whole-matrix statistic, shards are always cut from (or compressed with the threshold of)
the whole matrix, so a shard's bytes equal the corresponding bytes of the full compression.
"""
from __future__ import annotations

from typing import List, Optional

import torch

from . import _lib


class PackedWeight:
    def __init__(self, exps, signs, payload, n_out: int, k_in: int, kpad: int, npad: int,
                 coo=None, entries=None, seg_ptr=None):
        self.exps, self.signs, self.payload = exps, signs, payload
        self.n_out, self.k_in, self.kpad, self.npad = int(n_out), int(k_in), int(kpad), int(npad)
        self.coo = coo                  # (block_idx int32, offset int32, value bits int16)
        self.entries, self.seg_ptr = entries, seg_ptr
        self.records = None             # stage records of fbfp_gemv_records (build_records)
        # True once a fence kernel follows the last kernel that wrote these arrays on the current
        # stream: GEMVs may then use fbfp_gemv_resident (weight fetch overlapping the previous
        # kernel's tail)
        self.resident = False

    @property
    def device(self):
        return self.exps.device

    @property
    def kb_row(self) -> int:
        return self.kpad // 16

    @property
    def nnz(self) -> int:
        return 0 if self.coo is None else int(self.coo[0].numel())

    def packed_bytes(self) -> int:
        """Algorithmic bytes of the reference format: 11 per block + 10 per COO outlier."""
        return 11 * self.npad * self.kb_row + 10 * self.nnz

    def apply(self, fn):
        self.resident = False
        self.exps, self.signs, self.payload = fn(self.exps), fn(self.signs), fn(self.payload)
        if self.coo is not None:
            self.coo = tuple(fn(t) for t in self.coo)
        if self.entries is not None:
            self.entries, self.seg_ptr = fn(self.entries), fn(self.seg_ptr)
        if self.records is not None:
            self.records = fn(self.records)
        return self

    def build_tiles(self) -> "PackedWeight":
        """(Re)build the tile-grouped outlier entries from the COO list (and drop stage records
        built from the previous ones)."""
        L = _lib.lib()
        dev = self.device
        count = self.nnz
        entries = torch.zeros((count + 3) // 4 * 4 + 4, dtype=torch.int32, device=dev)
        seg_ptr = torch.empty(L.fbfp_outlier_tiles_index_words(self.npad, self.kpad), dtype=torch.int32,
                              device=dev)
        scratch = torch.empty(L.fbfp_outlier_tiles_scratch_bytes(self.npad, self.kpad),
                              dtype=torch.uint8, device=dev)
        b, o, v = self.coo if count else (None, None, None)
        with torch.cuda.device(dev):
            _lib.check(L.fbfp_outlier_tiles_build(_lib.ptr(b), _lib.ptr(o), _lib.ptr(v), count,
                                                  self.kpad, self.npad, self.n_out, self.k_in,
                                                  _lib.ptr(entries), _lib.ptr(seg_ptr),
                                                  _lib.ptr(scratch), _lib.stream_ptr(dev)),
                       "fbfp_outlier_tiles_build")
            self.entries, self.seg_ptr, self.records = entries, seg_ptr, None
            _lib.check(L.fbfp_stream_fence(_lib.stream_ptr(dev)), "fbfp_stream_fence")
        self.resident = True
        return self

    def build_records(self) -> "PackedWeight":
        """Build the stage records ``fbfp_gemv_records`` reads (kpad a multiple of 256; about the
        packed size again in HBM). Raises ValueError for exponents above 120, which the
        compressor never emits."""
        L = _lib.lib()
        if self.entries is None:
            self.build_tiles()
        count = self.nnz
        nbytes = L.fbfp_records_bytes(self.npad, self.kpad, count)
        if nbytes < 0 or self.payload.data_ptr() % 8 != 0:
            raise ValueError(f"no stage records for kpad={self.kpad} (a multiple of 256 is needed)")
        dev = self.device
        records = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        scratch = torch.empty(L.fbfp_records_scratch_bytes(self.npad, self.kpad), dtype=torch.uint8, device=dev)
        bad = torch.zeros(1, dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(L.fbfp_records_build(_lib.ptr(self.exps), _lib.ptr(self.signs), _lib.ptr(self.payload),
                                            self.npad, self.kpad, _lib.ptr(self.entries if count else None),
                                            _lib.ptr(self.seg_ptr if count else None), count,
                                            _lib.ptr(records), _lib.ptr(bad), _lib.ptr(scratch),
                                            _lib.stream_ptr(dev)), "fbfp_records_build")
            if int(bad.item()):
                raise ValueError(f"{int(bad.item())} blocks have exponents above 120, which the "
                                 "compressor never emits (dense values are at most 0.2)")
            self.records = records
            _lib.check(L.fbfp_stream_fence(_lib.stream_ptr(dev)), "fbfp_stream_fence")
        return self


def from_compressed(dense_payload, sparse_outliers, device, build_tiles: bool = True) -> PackedWeight:
    """PackedWeight from the compressor's dicts (any device; reference or widened dtypes)."""
    kpad, npad = dense_payload["padded_shape"]
    n_out, k_in = dense_payload["orig_shape"]
    exps = dense_payload["exponents"].to(device=device)
    exps = exps.round().to(torch.int8) if exps.is_floating_point() else exps.to(torch.int8)
    signs = dense_payload["signs"].to(device=device).to(torch.int16)
    payload = dense_payload["payload"].to(device=device, dtype=torch.int32).reshape(-1, 2).contiguous()
    coo = None
    if sparse_outliers is not None:
        coo = (sparse_outliers["block_idx"].to(device=device, dtype=torch.int32).contiguous(),
               sparse_outliers["offset"].to(device=device, dtype=torch.int32).contiguous(),
               sparse_outliers["value"].to(device=device, dtype=torch.float16).view(torch.int16).contiguous())
    pw = PackedWeight(exps.contiguous(), signs.contiguous(), payload, n_out, k_in, kpad, npad, coo)
    if build_tiles and coo is not None:
        pw.build_tiles()
    return pw


def concat_rows(parts: List[PackedWeight]) -> PackedWeight:
    """Stack matrices with the same K along the output dimension (fused launch).
    Output row offsets are the running sums of the parts' padded row counts."""
    kpad = parts[0].kpad
    k_in = parts[0].k_in
    assert all(p.kpad == kpad and p.k_in == k_in for p in parts), "parts must share K"
    kb = kpad // 16
    exps = torch.cat([p.exps for p in parts])
    signs = torch.cat([p.signs for p in parts])
    payload = torch.cat([p.payload for p in parts])
    bl, ol, vl = [], [], []
    row0 = 0
    for p in parts:
        if p.nnz:
            bl.append(p.coo[0] + row0 * kb)
            ol.append(p.coo[1])
            vl.append(p.coo[2])
        row0 += p.npad
    dev = parts[0].device
    if bl:
        coo = (torch.cat(bl), torch.cat(ol), torch.cat(vl))
    else:
        z = torch.zeros(0, dtype=torch.int32, device=dev)
        coo = (z, z.clone(), torch.zeros(0, dtype=torch.int16, device=dev))
    pw = PackedWeight(exps, signs, payload, row0, k_in, kpad, row0, coo)
    return pw.build_tiles()


def shard_rows(pw: PackedWeight, r0: int, r1: int, tiles: bool = True) -> PackedWeight:
    """Output rows [r0, r1) (column-parallel shard); r0, r1 multiples of 16. ``tiles=False``
    keeps only the COO outliers (no kernel layout; works on CPU tensors)."""
    assert r0 % 16 == 0 and (r1 % 16 == 0 or r1 == pw.npad) and 0 <= r0 < r1 <= pw.npad
    kb = pw.kb_row
    exps = pw.exps[r0 * kb:r1 * kb].contiguous()
    signs = pw.signs[r0 * kb:r1 * kb].contiguous()
    payload = pw.payload[r0 * kb:r1 * kb].contiguous()
    coo = None
    if pw.coo is not None:
        b, o, v = pw.coo
        keep = (b >= r0 * kb) & (b < r1 * kb)
        coo = ((b[keep] - r0 * kb).contiguous(), o[keep].contiguous(), v[keep].contiguous())
    n_out = max(0, min(pw.n_out, r1) - r0)
    out = PackedWeight(exps, signs, payload, n_out, pw.k_in, pw.kpad, r1 - r0, coo)
    return out.build_tiles() if tiles else out


def shard_cols(pw: PackedWeight, kb0: int, kb1: int, tiles: bool = True) -> PackedWeight:
    """Input block-columns [kb0, kb1) (row-parallel shard): K range [16*kb0, 16*kb1).
    ``tiles=False`` keeps only the COO outliers (works on CPU tensors)."""
    kb = pw.kb_row
    assert 0 <= kb0 < kb1 <= kb
    nkb = kb1 - kb0
    v2 = lambda t: t.view(pw.npad, kb, *t.shape[1:])[:, kb0:kb1].reshape(pw.npad * nkb, *t.shape[1:]).contiguous()
    exps, signs, payload = v2(pw.exps), v2(pw.signs), v2(pw.payload)
    coo = None
    if pw.coo is not None:
        b, o, v = pw.coo
        n = b // kb
        j = b % kb
        keep = (j >= kb0) & (j < kb1)
        coo = ((n[keep] * nkb + (j[keep] - kb0)).to(torch.int32).contiguous(), o[keep].contiguous(),
               v[keep].contiguous())
    k_in = max(0, min(pw.k_in, 16 * kb1) - 16 * kb0)
    out = PackedWeight(exps, signs, payload, pw.n_out, k_in, 16 * nkb, pw.npad, coo)
    return out.build_tiles() if tiles else out
