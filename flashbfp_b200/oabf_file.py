"""Compact on-disk OABF format: compressed layers stored as the compressor's dicts, as they are.

The compressor's output (flash_bfp/compressor.py:109-117) is written without conversion:
exponents int8[nb], signs int16[nb], payload int32[nb, 2] (11 bytes per 16-weight block) and
the outlier list block_idx int32, offset int32, value fp16 (10 bytes per outlier), plus an
optional bias in its own dtype. Loading therefore needs no recompression, and it reads the file
once into pinned host memory and copies every array to the GPU asynchronously.

Layout of a ``.oabf`` file (little-endian):

    bytes 0-7    magic b"OABF\\x00\\x01\\x00\\x00" (format version 1)
    bytes 8-15   uint64: length H of the JSON index that follows
    bytes 16..   the JSON index (UTF-8), then zero padding up to the data start, a multiple of 4096
    data         the arrays, each starting on a 256-byte boundary (offsets in the index are
                 relative to the data start)

The index is ``{"format": "oabf", "version": 1, "block_size": 16, "tile_size": 64,
"data_offset": D, "layers": [...]}``. Each layer holds ``name``, ``orig_shape`` [N, K],
``padded_shape`` [Kpad, Npad] (the compressor's order: in-dim first), ``count`` and ``arrays``.
``arrays`` maps exponents, signs, payload, block_idx, offset, value and bias (when the layer
has one) to ``{"dtype", "shape", "offset", "nbytes", "crc32"}``.
"""
from __future__ import annotations

import json
import os
import zlib
from typing import Dict, Optional, Tuple

import numpy as np
import torch

MAGIC = b"OABF\x00\x01\x00\x00"
VERSION = 1
_ALIGN = 256
_DATA_ALIGN = 4096

_DTYPES = {
    "int8": torch.int8, "int16": torch.int16, "int32": torch.int32, "int64": torch.int64,
    "float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32,
}
_NAMES = {v: k for k, v in _DTYPES.items()}

# (field, dtype the compressor emits)
_DENSE = (("exponents", torch.int8), ("signs", torch.int16), ("payload", torch.int32))
_SPARSE = (("block_idx", torch.int32), ("offset", torch.int32), ("value", torch.float16))

Layer = Tuple[Dict, Dict, Optional[torch.Tensor]]


class OABFFileError(ValueError):
    """A file that is not a readable OABF file (bad magic, version, index or checksum)."""


def _as_bytes(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    return t.view(torch.uint8).reshape(-1).numpy() if t.numel() else np.zeros(0, np.uint8)


def _native(t, dtype: torch.dtype, field: str) -> torch.Tensor:
    """The field in the compressor's own dtype. Widened reference dtypes (fp32 exponents, int32
    signs) must hold exact values of the narrow type."""
    t = torch.as_tensor(t)
    if t.dtype == dtype:
        return t
    if dtype.is_floating_point:
        return t.to(dtype)
    if t.is_floating_point():
        if not bool(torch.equal(t, t.round())):
            raise ValueError(f"{field}: non-integer values")
        t = t.round()
    info = torch.iinfo(dtype)
    if t.numel() and (int(t.min()) < info.min or int(t.max()) > info.max):
        raise ValueError(f"{field}: values outside {dtype}")
    return t.to(dtype)


def save_layers(path: str, layers: Dict[str, Layer], block_size: int = 16, tile_size: int = 64) -> None:
    """Write ``{name: (dense_payload, sparse_outliers, bias or None)}`` to ``path``."""
    entries, blobs = [], []
    offset = 0
    for name, (dp, sp, bias) in layers.items():
        kpad, npad = (int(v) for v in dp["padded_shape"])
        n, k = (int(v) for v in dp["orig_shape"])
        nb = npad * kpad // block_size
        arrays = {}
        fields = [(f, _native(dp[f], dt, f)) for f, dt in _DENSE]
        fields[2] = ("payload", fields[2][1].reshape(nb, 2))
        count = int(sp["count"]) if sp is not None else 0
        for f, dt in _SPARSE:
            src = sp[f] if (sp is not None and count) else torch.zeros(0, dtype=dt)
            fields.append((f, _native(src, dt, f)))
        if bias is not None:
            fields.append(("bias", torch.as_tensor(bias).detach()))
        if fields[0][1].numel() != nb or fields[1][1].numel() != nb:
            raise ValueError(f"{name}: {nb} blocks expected from padded_shape {(kpad, npad)}")
        for f, t in fields:
            raw = _as_bytes(t)
            offset = (offset + _ALIGN - 1) // _ALIGN * _ALIGN
            arrays[f] = {"dtype": _NAMES[t.dtype], "shape": list(t.shape), "offset": offset,
                         "nbytes": int(raw.size), "crc32": zlib.crc32(raw) & 0xFFFFFFFF}
            blobs.append((offset, raw))
            offset += raw.size
        entries.append({"name": name, "orig_shape": [n, k], "padded_shape": [kpad, npad],
                        "count": count, "arrays": arrays})
    index = {"format": "oabf", "version": VERSION, "block_size": block_size, "tile_size": tile_size,
             "data_offset": 0, "layers": entries}
    head = json.dumps(index).encode()
    data_offset = (16 + len(head) + 64 + _DATA_ALIGN - 1) // _DATA_ALIGN * _DATA_ALIGN
    index["data_offset"] = data_offset
    head = json.dumps(index).encode()
    if 16 + len(head) > data_offset:                     # the offset's digits grew the index
        data_offset += _DATA_ALIGN
        index["data_offset"] = data_offset
        head = json.dumps(index).encode()
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(np.uint64(len(head)).tobytes())
        f.write(head)
        f.write(b"\x00" * (data_offset - 16 - len(head)))
        pos = 0
        for off, raw in blobs:
            if off > pos:
                f.write(b"\x00" * (off - pos))
            f.write(raw.tobytes())
            pos = off + raw.size
    os.replace(tmp, path)


def read_index(path: str) -> Dict:
    """The JSON index of an OABF file (checks the magic and version)."""
    with open(path, "rb") as f:
        head = f.read(16)
        if len(head) < 16 or head[:8] != MAGIC:
            if len(head) >= 8 and head[:4] == MAGIC[:4]:
                raise OABFFileError(f"{path}: unsupported OABF format version {head[4:8]!r}")
            raise OABFFileError(f"{path}: not an OABF file")
        n = int(np.frombuffer(head[8:16], dtype=np.uint64)[0])
        raw = f.read(n)
    if len(raw) != n:
        raise OABFFileError(f"{path}: truncated index")
    try:
        index = json.loads(raw.decode())
    except ValueError as e:
        raise OABFFileError(f"{path}: unreadable index ({e})") from None
    if index.get("format") != "oabf" or index.get("version") != VERSION:
        raise OABFFileError(f"{path}: unsupported index {index.get('format')!r} v{index.get('version')!r}")
    return index


def load_layers(path: str, device=None, verify: bool = False) -> Dict[str, Layer]:
    """``{name: (dense_payload, sparse_outliers, bias or None)}`` from ``path``, the arrays in the
    compressor's dtypes, on ``device`` (default: CPU). The file is read once; with a CUDA device
    it goes through pinned memory and every array is copied asynchronously on the current
    stream. ``verify`` checks each array's CRC-32."""
    index = read_index(path)
    base = int(index["data_offset"])
    size = os.path.getsize(path) - base
    need = 0
    for e in index["layers"]:
        for a in e["arrays"].values():
            need = max(need, int(a["offset"]) + int(a["nbytes"]))
    if size < need:
        raise OABFFileError(f"{path}: truncated data ({size} of {need} bytes)")
    dev = torch.device(device) if device is not None else torch.device("cpu")
    pin = dev.type == "cuda"
    buf = torch.empty(need, dtype=torch.uint8, pin_memory=pin)
    with open(path, "rb") as f:
        f.seek(base)
        got = f.readinto(memoryview(buf.numpy()))
    if got != need:
        raise OABFFileError(f"{path}: short read ({got} of {need} bytes)")
    out: Dict[str, Layer] = {}
    for e in index["layers"]:
        arrs = {}
        for field, a in e["arrays"].items():
            lo, nbytes = int(a["offset"]), int(a["nbytes"])
            chunk = buf[lo:lo + nbytes]
            if verify and (zlib.crc32(chunk.numpy()) & 0xFFFFFFFF) != int(a["crc32"]):
                raise OABFFileError(f"{path}: checksum mismatch in {e['name']}.{field}")
            dt = _DTYPES[a["dtype"]]
            t = chunk.view(dt).reshape(a["shape"]) if nbytes else torch.zeros(a["shape"], dtype=dt)
            arrs[field] = t.to(dev, non_blocking=True) if pin else t.clone()
        dp = {"exponents": arrs["exponents"], "signs": arrs["signs"], "payload": arrs["payload"],
              "padded_shape": tuple(e["padded_shape"]), "orig_shape": torch.Size(e["orig_shape"])}
        sp = {"block_idx": arrs["block_idx"], "offset": arrs["offset"], "value": arrs["value"],
              "count": int(e["count"])}
        out[e["name"]] = (dp, sp, arrs.get("bias"))
    if pin:
        torch.cuda.current_stream(dev).synchronize()      # the pinned buffer may be released now
    return out


def save_compressed_model(model: torch.nn.Module, path: str) -> int:
    """Write every compressed OABFLinear of ``model`` (names as in ``find_linear_layers``:
    ``model.<dotted path>``); returns the number of layers written."""
    from .linear import OABFLinear
    layers = {}
    for name, mod in model.named_modules():
        if isinstance(mod, OABFLinear) and mod.compressed:
            pw = mod.packed
            dp = {"exponents": pw.exps, "signs": pw.signs, "payload": pw.payload,
                  "padded_shape": (pw.kpad, pw.npad), "orig_shape": (mod.out_features, mod.in_features)}
            if pw.nnz:
                b, o, v = pw.coo
                sp = {"block_idx": b, "offset": o, "value": v.view(torch.float16), "count": pw.nnz}
            else:
                sp = {"count": 0}
            layers["model." + name if name else "model"] = (dp, sp, mod.bias)
    save_layers(path, layers)
    return len(layers)


def load_compressed_model(model: torch.nn.Module, path: str, device=None) -> torch.nn.Module:
    """Replace the targeted linears of ``model`` (the ``compress_gemma_model`` name filter) with
    OABFLinear layers loaded from ``path`` without recompressing; every targeted layer must be in
    the file with matching shapes."""
    from .linear import OABFLinear
    from .model import find_linear_layers
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    stored = load_layers(path, dev)
    for parent, sub_name, lin, full in find_linear_layers(model):
        if full not in stored:
            raise KeyError(f"{path} has no layer {full}")
        dp, sp, bias = stored[full]
        if tuple(dp["orig_shape"]) != (lin.out_features, lin.in_features):
            raise ValueError(f"{full}: stored shape {tuple(dp['orig_shape'])} vs layer "
                             f"{(lin.out_features, lin.in_features)}")
        layer = OABFLinear(lin.in_features, lin.out_features, bias=lin.bias is not None).to(dev)
        if lin.bias is not None:
            if bias is None:
                raise ValueError(f"{full}: the layer has a bias, the file does not")
            layer.bias.data.copy_(bias)
        layer.load_compressed(dp, sp, dev)
        setattr(parent, sub_name, layer)
    return model
