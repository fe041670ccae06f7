"""The CPU oracle against the reference's own outputs (golden fixtures).

These pin the restatement in ``oracle/oabf.py`` before it is trusted as the
checker for the CUDA kernels."""
import hashlib

import numpy as np
import pytest

from oracle import oabf
from golden_io import case_names, load, fullsize

CASES = case_names()


def test_fixtures_present():
    assert len(CASES) >= 10


@pytest.mark.parametrize("name", CASES)
def test_threshold_matches_reference(name):
    g = load(name)
    thr = oabf.compute_dynamic_threshold(g["W"], g["dtype"])
    if np.isnan(g["threshold"]):
        assert np.isnan(thr)
    elif g["dtype"] == "bf16":
        assert thr == g["threshold"]
    else:
        # fp32: torch's float cascade mean / non-CR pow and sqrt can move the
        # last ulp; the restatement must agree to within one ulp.
        assert abs(np.float32(thr) - np.float32(g["threshold"])) <= np.spacing(np.float32(g["threshold"]))


@pytest.mark.parametrize("name", CASES)
def test_packed_bytes_bit_exact(name):
    g = load(name)
    dp, sp = oabf.compress_matrix(g["W"], g["dtype"], threshold=g["threshold"])
    assert dp["padded_shape"] == g["padded_shape"]
    assert dp["orig_shape"] == g["orig_shape"]
    np.testing.assert_array_equal(dp["exponents"], g["exponents"])
    np.testing.assert_array_equal(dp["signs"], g["signs"])
    np.testing.assert_array_equal(dp["payload"], g["payload"])
    assert sp["count"] == g["count"]
    np.testing.assert_array_equal(sp["block_idx"], g["block_idx"])
    np.testing.assert_array_equal(sp["offset"], g["offset"])
    np.testing.assert_array_equal(sp["value"].view(np.uint16), g["value_bits"])


@pytest.mark.parametrize("name", CASES)
def test_dequant_bit_exact(name):
    g = load(name)
    W = oabf.dequantize_dense(g["exponents"], g["signs"], g["payload"], g["padded_shape"], g["orig_shape"])
    # bit patterns, so -0.0 from sign=1/m=0 must match too
    np.testing.assert_array_equal(W.view(np.uint32), g["Wdeq_f32"].astype(np.float32).view(np.uint32))
    Wb = oabf.dequantize_dense_bf16_fallback(g["exponents"], g["signs"], g["payload"],
                                            g["padded_shape"], g["orig_shape"])
    np.testing.assert_array_equal(Wb.view(np.uint32), g["Wdeq_bf16fb"].astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("name", CASES)
def test_outlier_rcv(name):
    g = load(name)
    sp = {"block_idx": g["block_idx"], "offset": g["offset"], "value": g["value"], "count": g["count"]}
    n, k = g["orig_shape"]
    r, c, v = oabf.outlier_rcv(sp, g["padded_shape"], k, n)
    if "r_idx" in g:
        np.testing.assert_array_equal(r, g["r_idx"])
        np.testing.assert_array_equal(c, g["c_idx"])
        np.testing.assert_array_equal(v, g["v_val"])
    else:
        assert r.size == 0


@pytest.mark.parametrize("name", CASES)
def test_linear_matches_reference_forward(name):
    g = load(name)
    dp = {k: g[k] for k in ("exponents", "signs", "payload", "orig_shape", "padded_shape")}
    sp = {"block_idx": g["block_idx"], "offset": g["offset"], "value": g["value"], "count": g["count"]}
    for X, xdt, Yref in g["xs"]:
        Y = oabf.linear_reference(X, dp, sp, g.get("bias"))
        tol = 1e-5 if xdt == "fp32" else 2e-2   # reference forward runs bf16 matmul + bf16 index_add
        assert oabf.rel_l2(Yref, Y) <= tol


def test_edge_cases_present():
    """The crafted edge fixture exercises -0.0, int16/int32 wrap and the log2 codes."""
    g = load("edge_fp32")
    W = g["Wdeq_f32"].astype(np.float32)
    assert np.any((W == 0) & np.signbit(W))                      # -0.0 from sign=1, m=0
    assert np.any(g["signs"] < 0)                                # int16 wrap (bit 15)
    assert np.any(g["payload"] < 0)                              # int32 wrap (nibble 7 >= 8)
    assert g["exponents"].min() == -27                           # all-zero / tiny blocks
    ex = oabf.floor_log2_torch(np.array([np.float32(2.0 ** -16) * np.float32(1 - 11 * 2.0 ** -24)]), "fp32")
    assert ex[0] == -16


def test_log2_bump_tables():
    """torch's CPU floor(log2) is exact except the top codes of each binade:
    fp32 11/5/2/1 codes for binades <=-17 / -16..-9 / -8..-5 / -4..-3, bf16 10/5/2/1."""
    f = oabf.log2_bump_counts("fp32", -30, -3)
    b = oabf.log2_bump_counts("bf16", -30, -3)
    for e in range(-30, -2):
        exp_f = 11 if e <= -17 else 5 if e <= -9 else 2 if e <= -5 else 1
        exp_b = 10 if e <= -17 else 5 if e <= -9 else 2 if e <= -5 else 1
        assert f[e] == exp_f, (e, f[e])
        assert b[e] == exp_b, (e, b[e])


@pytest.mark.slow
def test_fullsize_digests():
    """Config-1 full size (4096x4096 fp32, seed 0) and a 2048x3840 bf16 decode
    layer: the oracle's packed bytes hash to the reference's."""
    from flashbfp_b200 import workloads
    ref = fullsize()
    for name, W in workloads.fullsize_cases().items():
        r = ref[name]
        dp, sp = oabf.compress_matrix(W.float().numpy(), r["dtype"], threshold=r["threshold"])
        assert sp["count"] == r["count"]
        h = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
        assert h(dp["exponents"]) == r["sha256_exponents"]
        assert h(dp["signs"]) == r["sha256_signs"]
        assert h(dp["payload"]) == r["sha256_payload"]
        assert h(sp["block_idx"]) == r["sha256_block_idx"]
        assert h(sp["offset"]) == r["sha256_offset"]
        assert h(sp["value"]) == r["sha256_value"]
