"""The compact on-disk OABF format (flashbfp_b200/oabf_file.py).

CPU: the compressor's dicts (made by the oracle's restatement of compress_matrix) survive a
save/load round trip bit for bit, reference-widened dtypes are stored in the native ones, the
file costs 11 bytes per block and 10 per outlier plus a small index, and damaged files (magic,
version, truncation, checksum) are refused. GPU: a compressed model written with
save_compressed_model and read into a fresh model with load_compressed_model holds the same
packed bytes and gives the same logits, without recompression.
"""
import json
import os

import numpy as np
import pytest
import torch

from flashbfp_b200 import oabf_file
from oracle import oabf


def _layer(n, k, seed, outliers=True, bias_dtype=None):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    if not outliers:                    # every value under the threshold's 0.01 floor
        W = rng.uniform(-0.005, 0.005, size=(n, k)).astype(np.float32)
    if outliers:
        idx = rng.choice(n * k, size=max(1, n * k // 100), replace=False)
        W.reshape(-1)[idx] = rng.uniform(0.3, 0.9, size=idx.size).astype(np.float32)
    dp, sp = oabf.compress_matrix(W, "fp32")
    dpt = {kk: (torch.from_numpy(v) if isinstance(v, np.ndarray) else v) for kk, v in dp.items()}
    spt = {kk: (torch.from_numpy(v) if isinstance(v, np.ndarray) else v) for kk, v in sp.items()}
    bias = None
    if bias_dtype is not None:
        bias = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(bias_dtype)
    return dpt, spt, bias


def _same(a, b):
    return a.dtype == b.dtype and a.shape == b.shape and torch.equal(a, b)


def test_round_trip_is_bit_exact(tmp_path):
    layers = {
        "model.layers.0.self_attn.q_proj": _layer(100, 300, 1, True, torch.bfloat16),
        "model.layers.0.mlp.down_proj": _layer(64, 512, 2, True, None),
        "model.layers.1.mlp.up_proj": _layer(70, 48, 3, False, torch.float32),
    }
    assert layers["model.layers.1.mlp.up_proj"][1]["count"] == 0
    path = str(tmp_path / "m.oabf")
    oabf_file.save_layers(path, layers)
    got = oabf_file.load_layers(path, verify=True)
    assert list(got) == list(layers)
    for name, (dp, sp, bias) in layers.items():
        gdp, gsp, gbias = got[name]
        for f in ("exponents", "signs", "payload"):
            assert _same(gdp[f], dp[f]), (name, f)
        assert tuple(gdp["padded_shape"]) == tuple(dp["padded_shape"])
        assert tuple(gdp["orig_shape"]) == tuple(dp["orig_shape"])
        assert gsp["count"] == sp["count"]
        for f in ("block_idx", "offset", "value"):
            assert _same(gsp[f], sp[f]), (name, f)
        assert (gbias is None) == (bias is None)
        if bias is not None:
            assert _same(gbias, bias)


def test_layout_is_compact_and_aligned(tmp_path):
    dp, sp, _ = _layer(256, 1024, 4)
    path = str(tmp_path / "one.oabf")
    oabf_file.save_layers(path, {"w": (dp, sp, None)})
    index = oabf_file.read_index(path)
    assert index["data_offset"] % 4096 == 0
    arrays = index["layers"][0]["arrays"]
    assert all(a["offset"] % 256 == 0 for a in arrays.values())
    nb, nnz = dp["exponents"].numel(), sp["count"]
    payload_bytes = sum(a["nbytes"] for a in arrays.values())
    assert payload_bytes == 11 * nb + 10 * nnz
    assert os.path.getsize(path) <= index["data_offset"] + payload_bytes + 6 * 256


def test_widened_reference_dtypes_are_stored_natively(tmp_path):
    dp, sp, _ = _layer(64, 256, 5)
    wide = dict(dp)
    wide["exponents"] = dp["exponents"].to(torch.float32)          # triton_kernel.py:147-158
    wide["signs"] = dp["signs"].to(torch.int32)
    wide["payload"] = dp["payload"].reshape(-1)
    path = str(tmp_path / "w.oabf")
    oabf_file.save_layers(path, {"w": (wide, sp, None)})
    gdp, _, _ = oabf_file.load_layers(path)["w"]
    for f in ("exponents", "signs", "payload"):
        assert _same(gdp[f], dp[f]), f
    bad = dict(wide)
    bad["signs"] = dp["signs"].to(torch.int32) + 70000
    with pytest.raises(ValueError, match="outside"):
        oabf_file.save_layers(str(tmp_path / "bad.oabf"), {"w": (bad, sp, None)})


def test_damaged_files_are_refused(tmp_path):
    dp, sp, _ = _layer(64, 256, 6)
    path = str(tmp_path / "d.oabf")
    oabf_file.save_layers(path, {"w": (dp, sp, None)})
    raw = bytearray(open(path, "rb").read())

    def write(name, data):
        p = str(tmp_path / name)
        with open(p, "wb") as f:
            f.write(bytes(data))
        return p

    with pytest.raises(oabf_file.OABFFileError, match="not an OABF file"):
        oabf_file.load_layers(write("magic.oabf", b"NOPE" + raw[4:]))
    v2 = bytearray(raw)
    v2[5] = 2
    with pytest.raises(oabf_file.OABFFileError, match="version"):
        oabf_file.load_layers(write("v2.oabf", v2))
    with pytest.raises(oabf_file.OABFFileError, match="truncated"):
        oabf_file.load_layers(write("short.oabf", raw[:-100]))
    index = oabf_file.read_index(path)
    a = index["layers"][0]["arrays"]["payload"]
    flip = bytearray(raw)
    flip[index["data_offset"] + a["offset"] + 7] ^= 0x10
    p = write("flip.oabf", flip)
    oabf_file.load_layers(p)                                         # not checked by default
    with pytest.raises(oabf_file.OABFFileError, match="checksum"):
        oabf_file.load_layers(p, verify=True)
    head_len = int(np.frombuffer(bytes(raw[8:16]), dtype=np.uint64)[0])
    idx = json.loads(bytes(raw[16:16 + head_len]).decode())
    idx["format"] = "oabx"                                           # same length
    body = json.dumps(idx).encode()
    assert len(body) == head_len
    other = raw[:16] + body + raw[16 + head_len:]
    with pytest.raises(oabf_file.OABFFileError, match="unsupported index"):
        oabf_file.load_layers(write("other.oabf", other))


@pytest.mark.gpu
def test_model_save_and_load_without_recompression(tmp_path):
    transformers = pytest.importorskip("transformers")
    from flashbfp_b200 import OABFCompressor
    from flashbfp_b200.linear import OABFLinear, check_device_errors
    from flashbfp_b200.model import compress_gemma_model, find_linear_layers

    cfg = transformers.Gemma3TextConfig(vocab_size=512, hidden_size=256, intermediate_size=512,
                                        num_hidden_layers=2, num_attention_heads=4,
                                        num_key_value_heads=2, head_dim=64,
                                        max_position_embeddings=128, sliding_window=64)
    dev = torch.device("cuda", 0)

    def fresh():
        torch.manual_seed(3)
        return transformers.Gemma3ForCausalLM(cfg).eval().to(dev, torch.bfloat16)

    a = compress_gemma_model(fresh(), OABFCompressor())
    path = str(tmp_path / "tiny.oabf")
    n = oabf_file.save_compressed_model(a, path)
    assert n == 14
    b = fresh()
    names = [full for _, _, _, full in find_linear_layers(b)]
    oabf_file.load_compressed_model(b, path, dev)
    mods_a = {nm: m for nm, m in a.named_modules() if isinstance(m, OABFLinear)}
    mods_b = {nm: m for nm, m in b.named_modules() if isinstance(m, OABFLinear)}
    assert sorted(mods_a) == sorted(mods_b) and len(mods_b) == len(names)
    for nm in mods_a:
        pa, pb = mods_a[nm].packed, mods_b[nm].packed
        for f in ("exps", "signs", "payload"):
            assert torch.equal(getattr(pa, f), getattr(pb, f)), (nm, f)
        assert pa.nnz == pb.nnz
        for x, y in zip(pa.coo, pb.coo):
            assert torch.equal(x, y), nm
    ids = torch.randint(0, 512, (1, 16), generator=torch.Generator().manual_seed(0)).to(dev)
    with torch.no_grad():
        la = a(ids).logits.float()
        lb = b(ids).logits.float()
    check_device_errors(dev)
    rel = ((la - lb).norm() / la.norm()).item()
    assert rel <= 1e-3, rel
