"""CUDA path vs the oracle and the reference's golden outputs (B200).

Bit-exact: packed exponent/sign/payload bytes, outlier indices and values, dequantised
weights (fp32 bits including -0.0, and bf16). GEMV/GEMM outputs: rel-L2 <= 1e-2 against the
fp64 dequantize-then-matmul of the oracle and against the reference's own forward outputs.
"""
import hashlib

import numpy as np
import pytest
import torch

from oracle import oabf
from golden_io import case_names, load, fullsize

pytestmark = pytest.mark.gpu

CASES = case_names()
GEMM_TOL = 1e-2          # north-star bound for bf16 activations with fp32 accumulation


@pytest.fixture(scope="module", autouse=True)
def _setup():
    from flashbfp_b200 import build
    build.build()
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)


def _dev():
    return torch.device("cuda", 0)


def _w_tensor(g):
    W = torch.from_numpy(g["W"])
    return (W.to(torch.bfloat16) if g["dtype"] == "bf16" else W).to(_dev())


def _dense_payload(g, dev):
    return {
        "exponents": torch.from_numpy(g["exponents"]).to(dev),
        "signs": torch.from_numpy(g["signs"]).to(dev),
        "payload": torch.from_numpy(g["payload"]).to(dev),
        "orig_shape": torch.Size(g["orig_shape"]),
        "padded_shape": g["padded_shape"],
    }


def _sparse(g, dev):
    return {"block_idx": torch.from_numpy(g["block_idx"]).to(dev),
            "offset": torch.from_numpy(g["offset"]).to(dev),
            "value": torch.from_numpy(g["value"]).to(dev), "count": g["count"]}


def _dequant(dp, out_dtype):
    from flashbfp_b200 import _lib
    L = _lib.lib()
    n, k = dp["orig_shape"]
    kpad, npad = dp["padded_shape"]
    out = torch.empty(n, k, dtype=out_dtype, device=dp["exponents"].device)
    _lib.check(L.fbfp_dequant(_lib.ptr(dp["exponents"]), _lib.ptr(dp["signs"]), _lib.ptr(dp["payload"]),
                              n, k, kpad, _lib.DTYPE_CODE[out_dtype], _lib.ptr(out), k,
                              _lib.stream_ptr(out.device)), "dequant")
    return out


def _dequant_full(dp, sp, out_dtype=torch.float32):
    from flashbfp_b200 import _lib
    L = _lib.lib()
    W = _dequant(dp, out_dtype)
    n, k = dp["orig_shape"]
    kpad, _ = dp["padded_shape"]
    if sp["count"]:
        _lib.check(L.fbfp_scatter_outliers(_lib.ptr(sp["block_idx"]), _lib.ptr(sp["offset"]),
                                           _lib.ptr(sp["value"]), sp["count"], kpad, n, k,
                                           _lib.DTYPE_CODE[out_dtype], _lib.ptr(W), k,
                                           _lib.stream_ptr(W.device)), "scatter")
    return W


# ---------------------------------------------------------------------------------------
# dequantisation
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("name", CASES)
def test_dequant_fp32_bit_exact(name):
    g = load(name)
    W = _dequant(_dense_payload(g, _dev()), torch.float32).cpu().numpy()
    np.testing.assert_array_equal(W.view(np.uint32), g["Wdeq_f32"].astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("name", CASES)
def test_dequant_bf16_bit_exact(name):
    g = load(name)
    W = _dequant(_dense_payload(g, _dev()), torch.bfloat16).float().cpu().numpy()
    np.testing.assert_array_equal(W.view(np.uint32), g["Wdeq_bf16fb"].astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("name", CASES)
def test_dequant_full_with_outliers(name):
    g = load(name)
    dev = _dev()
    W = _dequant_full(_dense_payload(g, dev), _sparse(g, dev)).cpu().numpy()
    ref = oabf.dequantize_full(_dense_payload_np(g), _sparse_np(g))
    np.testing.assert_array_equal(W.view(np.uint32), ref.view(np.uint32))


def _dense_payload_np(g):
    return {k: g[k] for k in ("exponents", "signs", "payload", "orig_shape", "padded_shape")}


def _sparse_np(g):
    return {"block_idx": g["block_idx"], "offset": g["offset"], "value": g["value"], "count": g["count"]}


# ---------------------------------------------------------------------------------------
# compressor
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("name", CASES)
def test_threshold(name):
    from flashbfp_b200 import OABFCompressor
    g = load(name)
    thr = OABFCompressor(16, 64).compute_dynamic_threshold(_w_tensor(g))
    ref = g["threshold"]
    if np.isnan(ref):
        assert np.isnan(thr)
    elif g["dtype"] == "bf16":
        assert thr == ref
    else:
        assert abs(np.float32(thr) - np.float32(ref)) <= np.spacing(np.float32(ref))
    assert thr == oabf.compute_dynamic_threshold(g["W"], g["dtype"]) or np.isnan(thr)


def _assert_bytes(dp, sp, g):
    assert tuple(dp["padded_shape"]) == g["padded_shape"]
    assert tuple(dp["orig_shape"]) == g["orig_shape"]
    assert dp["exponents"].dtype == torch.int8 and dp["signs"].dtype == torch.int16
    assert dp["payload"].dtype == torch.int32 and tuple(dp["payload"].shape) == g["payload"].shape
    np.testing.assert_array_equal(dp["exponents"].cpu().numpy(), g["exponents"])
    np.testing.assert_array_equal(dp["signs"].cpu().numpy(), g["signs"])
    np.testing.assert_array_equal(dp["payload"].cpu().numpy(), g["payload"])
    assert sp["count"] == g["count"]
    assert sp["block_idx"].dtype == torch.int32 and sp["value"].dtype == torch.float16
    np.testing.assert_array_equal(sp["block_idx"].cpu().numpy(), g["block_idx"])
    np.testing.assert_array_equal(sp["offset"].cpu().numpy(), g["offset"])
    np.testing.assert_array_equal(sp["value"].cpu().numpy().view(np.uint16), g["value_bits"])


@pytest.mark.parametrize("name", CASES)
def test_pack_bytes_given_threshold(name):
    from flashbfp_b200 import OABFCompressor
    g = load(name)
    thr = g["threshold"]
    dp, sp = OABFCompressor(16, 64).compress_matrix_device(_w_tensor(g), threshold=thr)
    _assert_bytes(dp, sp, g)


@pytest.mark.parametrize("name", CASES)
def test_compress_matrix_end_to_end(name):
    """Public API, own threshold, CPU tensors out (compressor.py:34-117)."""
    from flashbfp_b200 import OABFCompressor
    g = load(name)
    dp, sp = OABFCompressor(block_size=16, tile_size=64).compress_matrix(_w_tensor(g))
    assert not dp["exponents"].is_cuda and isinstance(sp["count"], int)
    _assert_bytes(dp, sp, g)


def test_fullsize_digests():
    """Config-1 (4096x4096 fp32, seed 0) and a 2048x3840 bf16 decode layer at full size."""
    from flashbfp_b200 import OABFCompressor, workloads
    ref = fullsize()
    h = lambda t: hashlib.sha256(t.cpu().numpy().tobytes()).hexdigest()
    for name, W in workloads.fullsize_cases().items():
        r = ref[name]
        comp = OABFCompressor(16, 64)
        thr = comp.compute_dynamic_threshold(W.cuda())
        assert thr == r["threshold"]
        dp, sp = comp.compress_matrix_device(W.cuda())
        assert sp["count"] == r["count"]
        assert h(dp["exponents"]) == r["sha256_exponents"]
        assert h(dp["signs"]) == r["sha256_signs"]
        assert h(dp["payload"]) == r["sha256_payload"]
        assert h(sp["block_idx"]) == r["sha256_block_idx"]
        assert h(sp["offset"]) == r["sha256_offset"]
        assert h(sp["value"]) == r["sha256_value"]


def test_compress_roundtrip_properties_large():
    """Decode-layer sized bf16 matrix (15360 x 3840): dequant(compress(W)) + outliers
    reproduces W within the format's quantisation bound, and every outlier is exact."""
    from flashbfp_b200 import OABFCompressor, workloads
    W = workloads.decode_weight(15360, 3840, seed=3, device="cuda")
    dp, sp = OABFCompressor().compress_matrix_device(W)
    Wf = _dequant_full(dp, sp).float()
    Wt = W.float()
    err = (Wf - Wt).abs()
    # per-block bound: the mantissa grid step is 2^e/15, the saturated top element loses < 2^e
    e = dp["exponents"].view(-1, 240).float()[:15360]
    bound = torch.repeat_interleave(torch.exp2(e + 1), 16, dim=1).clamp(min=1e-7)
    assert bool((err <= bound).all())
    gi = sp["block_idx"].long() * 16 + sp["offset"].long()
    vals = Wt.reshape(-1)[gi]
    assert torch.equal(Wf.reshape(-1)[gi], sp["value"].float())
    assert torch.equal(sp["value"], vals.half())
    assert bool((gi[1:] > gi[:-1]).all())                        # ascending flat order


# ---------------------------------------------------------------------------------------
# fused GEMV (decode) and OABFLinear
# ---------------------------------------------------------------------------------------
def _oracle_linear_np(g, X, bias):
    return oabf.linear_reference(X, _dense_payload_np(g), _sparse_np(g), bias)


@pytest.mark.parametrize("name", CASES)
def test_linear_vs_reference_forward(name):
    from flashbfp_b200 import OABFCompressor, OABFLinear
    g = load(name)
    n, k = g["orig_shape"]
    has_bias = "bias" in g
    lin = OABFLinear(k, n, bias=has_bias).cuda()
    if has_bias:
        with torch.no_grad():
            lin.bias.copy_(torch.from_numpy(g["bias"]))
    lin.load_from_weight(_w_tensor(g), OABFCompressor(16, 64), torch.device("cuda", 0))
    for X, xdt, Yref in g["xs"]:
        Xt = torch.from_numpy(X).to(torch.bfloat16 if xdt == "bf16" else torch.float32).cuda()
        Y = lin(Xt)
        assert Y.shape == Yref.shape
        exact = _oracle_linear_np(g, Xt.float().cpu().numpy(), g.get("bias"))
        assert oabf.rel_l2(Y.float().cpu().numpy(), exact) <= GEMM_TOL
        assert oabf.rel_l2(Y.float().cpu().numpy(), Yref) <= GEMM_TOL


@pytest.mark.parametrize("m", [1, 2, 3, 4, 7, 8, 9, 15, 16, 17, 40])
@pytest.mark.parametrize("shape", [(192, 256), (100, 70), (4096, 3840), (3840, 4096), (200, 3856),
                                   (3840, 15360)])
def test_linear_vs_torch_fp32(m, shape):
    """OABFLinear vs a plain PyTorch fp32 dequantize-then-matmul of the same weights."""
    from flashbfp_b200 import OABFCompressor, OABFLinear, workloads
    n, k = shape
    W = workloads.decode_weight(n, k, seed=n + k, device="cuda")
    lin = OABFLinear(k, n, bias=False).cuda()
    comp = OABFCompressor()
    lin.load_from_weight(W, comp, torch.device("cuda", 0))
    dp, sp = comp.compress_matrix_device(W)
    Wf = _dequant_full(dp, sp)
    X = workloads.activations(m, k, seed=m, device="cuda")
    Y = lin(X)
    from flashbfp_b200.linear import check_device_errors
    check_device_errors()
    ref = X.float() @ Wf.t()
    rel = ((Y.float() - ref).norm() / ref.norm()).item()
    assert rel <= GEMM_TOL, rel
    assert rel <= 5e-3, rel          # bf16 output rounding dominates; fp32 accumulation


def test_oabf_gemm_dense_only_and_reference_layouts():
    """oabf_gemm returns only the dense part and accepts the reference's GPU-side widened
    layout (fp32 exponents, int32 signs, flat int32 payload; triton_kernel.py:147-158)."""
    from flashbfp_b200 import oabf_gemm
    g = load("decode_t3_bf16")
    X = torch.from_numpy(g["xs"][1][0]).to(torch.bfloat16).cuda()
    dp = _dense_payload(g, "cpu")
    Y = oabf_gemm(X, dp).float().cpu().numpy()
    Wd = oabf.dequantize_dense(g["exponents"], g["signs"], g["payload"], g["padded_shape"], g["orig_shape"])
    exact = X.float().cpu().numpy().astype(np.float64) @ Wd.astype(np.float64).T
    assert oabf.rel_l2(Y, exact) <= GEMM_TOL
    wide = dict(dp)
    wide["exponents"] = dp["exponents"].float()
    wide["signs"] = dp["signs"].to(torch.int32)
    wide["payload"] = dp["payload"].reshape(-1)
    Y2 = oabf_gemm(X, wide).float().cpu().numpy()
    np.testing.assert_array_equal(Y, Y2)


def test_workspace_left_clean_and_repeatable():
    from flashbfp_b200 import OABFCompressor, OABFLinear, workloads
    from flashbfp_b200.linear import _WORKSPACES
    W = workloads.decode_weight(3840, 15360, seed=9, device="cuda")
    lin = OABFLinear(15360, 3840, bias=True).cuda()
    with torch.no_grad():
        lin.bias.normal_()
    lin.load_from_weight(W, OABFCompressor(), torch.device("cuda", 0))
    X = workloads.activations(5, 15360, seed=1, device="cuda")
    Y1 = lin(X)
    Y2 = lin(X)
    torch.cuda.synchronize()
    for ws in _WORKSPACES.values():
        assert int(ws.count_nonzero()) == 0
    # the fp32 partial sums of different chunks meet through atomics: order may differ
    assert ((Y1.float() - Y2.float()).abs().max() <= 1e-2 * Y1.float().abs().max())


def test_state_dict_reference_keys_and_roundtrip():
    from flashbfp_b200 import OABFCompressor, OABFLinear
    g = load("decode_t3_bf16")
    n, k = g["orig_shape"]
    lin = OABFLinear(k, n, bias=True).cuda()
    lin.load_from_weight(_w_tensor(g), OABFCompressor(), torch.device("cuda", 0))
    sd = lin.state_dict()
    assert sorted(sd.keys()) == sorted(str(s) for s in g["state_dict_keys"])
    assert sd["_dp_exponents"].dtype == torch.float32 and sd["_dp_signs"].dtype == torch.int32
    assert sd["_sp_r_idx"].dtype == torch.int64 and sd["_sp_v_val"].dtype == torch.float32
    np.testing.assert_array_equal(sd["_dp_signs"].cpu().numpy(), g["signs"].astype(np.int32))
    np.testing.assert_array_equal(sd["_sp_r_idx"].cpu().numpy(), g["r_idx"])
    np.testing.assert_array_equal(sd["_sp_c_idx"].cpu().numpy(), g["c_idx"])
    lin2 = OABFLinear(k, n, bias=True).cuda()
    lin2.load_state_dict({kk: v.clone() for kk, v in sd.items()})
    X = torch.from_numpy(g["xs"][0][0]).to(torch.bfloat16).cuda()
    assert torch.allclose(lin(X).float(), lin2(X).float(), rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("name", CASES)
def test_load_state_dict_assembled_from_reference_arrays(name):
    """A state dict in the reference's own form (triton_kernel.py:232-291, 370-379): exponents as
    fp32, signs and flattened payload as int32, outliers as int64 (input row, output column)
    pairs with fp32 values, the fp32 `_sp_value` buffer, built from the fixture's arrays (not from
    this package's compressor), loads (:381-423) and reproduces the reference's forward outputs."""
    from flashbfp_b200 import OABFLinear
    g = load(name)
    n, k = g["orig_shape"]
    has_bias = "bias" in g
    sd = {"_dp_exponents": torch.from_numpy(g["exponents"].astype(np.float32)),
          "_dp_signs": torch.from_numpy(g["signs"].astype(np.int32)),
          "_dp_payload": torch.from_numpy(g["payload"].astype(np.int32).reshape(-1)),
          "_sp_value": torch.from_numpy(g["value"].astype(np.float32))}
    if g["count"]:
        sd.update({"_sp_r_idx": torch.from_numpy(g["r_idx"].astype(np.int64)),
                   "_sp_c_idx": torch.from_numpy(g["c_idx"].astype(np.int64)),
                   "_sp_v_val": torch.from_numpy(g["v_val"].astype(np.float32))})
    if has_bias:
        sd["bias"] = torch.from_numpy(g["bias"].astype(np.float32))
    lin = OABFLinear(k, n, bias=has_bias).cuda()
    lin.load_state_dict(sd)
    for X, xdt, Yref in g["xs"]:
        Xt = torch.from_numpy(X).to(torch.bfloat16 if xdt == "bf16" else torch.float32).cuda()
        Y = lin(Xt)
        assert Y.shape == Yref.shape
        assert oabf.rel_l2(Y.float().cpu().numpy(), Yref) <= GEMM_TOL
        exact = _oracle_linear_np(g, Xt.float().cpu().numpy(), g.get("bias"))
        assert oabf.rel_l2(Y.float().cpu().numpy(), exact) <= GEMM_TOL


def test_errors_fail_loudly():
    from flashbfp_b200 import OABFCompressor, OABFLinear
    lin = OABFLinear(32, 64, bias=False)
    with pytest.raises(RuntimeError):
        lin(torch.zeros(1, 32, device="cuda"))
    with pytest.raises(ValueError):
        OABFCompressor().compress_matrix(torch.zeros(0, 16, device="cuda"))
    with pytest.raises(ValueError):
        OABFCompressor(block_size=8).compress_matrix(torch.ones(4, 16, device="cuda"))
    lin.load_from_weight(torch.randn(64, 32) * 0.02, OABFCompressor(), torch.device("cuda", 0))
    with pytest.raises(RuntimeError):
        lin(torch.zeros(1, 32))                                 # CPU activations: no CPU path
