"""Decode GEMV on stage records (fbfp_records_build, fbfp_gemv_records) on the B200.

* The records the GPU builds equal, byte for byte, the numpy model of the layout
  (record_layout.py), which the CPU tests tie to the oracle.
* fbfp_gemv_records vs the fp64 oracle (dequantise-then-matmul with outliers, bias) within the
  north-star 1e-2, and vs the reference-layout GEMV (fbfp_gemv) within fp32 summation-order
  noise, for token counts 1..16, partial 128-row groups, fp32 and bf16 outputs, the dense part
  alone, records whose outliers overflow the staging area, and graph replays of many launches in
  a row (consecutive GEMVs overlapping through programmatic dependent launch).
"""
import numpy as np
import pytest
import torch

from oracle import oabf
from golden_io import load
import record_layout as RL

pytestmark = pytest.mark.gpu

GEMM_TOL = 1e-2


@pytest.fixture(scope="module", autouse=True)
def _setup():
    from flashbfp_b200 import build
    build.build()


def _dev():
    return torch.device("cuda", 0)


def _packed(n, k, seed, frac=0.015, scale=20.0):
    from flashbfp_b200 import OABFCompressor, packed, workloads
    W = workloads.decode_weight(n, k, seed=seed, frac=frac, scale=scale, device=_dev())
    dp, sp = OABFCompressor().compress_matrix_device(W)
    pw = packed.from_compressed(dp, sp, _dev()).build_records()
    torch.cuda.synchronize()
    return pw, dp, sp


def _np(dp, sp):
    d = {k: (dp[k].cpu().numpy() if torch.is_tensor(dp[k]) else dp[k])
         for k in ("exponents", "signs", "payload", "orig_shape", "padded_shape")}
    s = {k: sp[k].cpu().numpy() for k in ("block_idx", "offset", "value")}
    s["count"] = int(sp["count"])
    return d, s


def _run(pw, X, bias=None, out_dtype=torch.bfloat16, outliers=True, tensor_cores=False):
    from flashbfp_b200 import linear
    Y = torch.full((X.shape[0], pw.n_out), float("nan"), dtype=out_dtype, device=X.device)
    ws = linear.gemv_workspace(X.device, pw.npad)
    linear.gemv_records(X, pw, Y, ws, bias, outliers, tensor_cores=tensor_cores)
    linear.check_device_errors()
    return Y


def test_records_bytes_match_layout_model():
    from flashbfp_b200 import packed
    g = load("decode_t3_bf16")
    dp = {"exponents": torch.from_numpy(g["exponents"]), "signs": torch.from_numpy(g["signs"]),
          "payload": torch.from_numpy(g["payload"]), "orig_shape": torch.Size(g["orig_shape"]),
          "padded_shape": g["padded_shape"]}
    sp = {"block_idx": torch.from_numpy(g["block_idx"]), "offset": torch.from_numpy(g["offset"]),
          "value": torch.from_numpy(g["value"]), "count": g["count"]}
    pw = packed.from_compressed(dp, sp, _dev()).build_records()
    kpad, npad = g["padded_shape"]
    n, k = g["orig_shape"]
    tiles = RL.outlier_tiles(g["block_idx"], g["offset"], g["value_bits"], npad, kpad, n, k)
    ref = RL.build_records(g["exponents"], g["signs"], g["payload"], npad, kpad, tiles)
    got = pw.records.cpu().numpy()
    assert got.size >= ref.size
    np.testing.assert_array_equal(got[:ref.size], ref)
    assert not got[ref.size:].any()
    # a synthetic matrix with every exponent from -128 to 120 and a partial row group
    rng = np.random.default_rng(5)
    npad, kpad = 192, 512
    nb = npad * kpad // 16
    exps = (np.arange(nb) % 249 - 128).astype(np.int8)
    signs = rng.integers(-32768, 32768, size=nb).astype(np.int16)
    payload = rng.integers(-2**31, 2**31, size=(nb, 2), dtype=np.int64).astype(np.int32)
    dp = {"exponents": torch.from_numpy(exps), "signs": torch.from_numpy(signs),
          "payload": torch.from_numpy(payload), "orig_shape": torch.Size((npad, kpad)),
          "padded_shape": (kpad, npad)}
    pw = packed.from_compressed(dp, None, _dev(), build_tiles=False)
    pw.build_records()
    ref = RL.build_records(exps, signs, payload, npad, kpad)
    got = pw.records.cpu().numpy()
    np.testing.assert_array_equal(got[:ref.size], ref)


def test_records_refuse_exponents_beyond_a_biased_byte():
    from flashbfp_b200 import packed
    npad, kpad = 64, 256
    nb = npad * kpad // 16
    exps = np.full(nb, -5, dtype=np.int8)
    exps[7] = 121
    dp = {"exponents": torch.from_numpy(exps), "signs": torch.zeros(nb, dtype=torch.int16),
          "payload": torch.zeros(nb, 2, dtype=torch.int32), "orig_shape": torch.Size((npad, kpad)),
          "padded_shape": (kpad, npad)}
    pw = packed.from_compressed(dp, None, _dev(), build_tiles=False)
    with pytest.raises(ValueError):
        pw.build_records()


@pytest.mark.parametrize("m,tc", [(1, False), (1, True), (3, True), (8, True), (9, True), (16, True)],
                         ids=["1-cuda-cores", "1-tensor-cores", "3", "8", "9", "16"])
@pytest.mark.parametrize("shape", [(192, 512), (1000, 3840), (3840, 4096), (2048, 15360)])
def test_gemv_records_vs_oracle_and_reference_layout(m, tc, shape):
    from flashbfp_b200 import workloads, _lib
    n, k = shape
    pw, dp, sp = _packed(n, k, seed=n + 3 * k)
    X = workloads.activations(m, k, seed=m + 1, device=_dev())
    bias = torch.randn(n, device=_dev(), dtype=torch.float32) * 0.1
    Y = _run(pw, X, bias, torch.float32, tensor_cores=tc)
    dpn, spn = _np(dp, sp)
    exact = oabf.linear_reference(X.float().cpu().numpy(), dpn, spn, bias.cpu().numpy())
    assert oabf.rel_l2(Y.cpu().numpy(), exact) <= 1e-3
    # the reference-layout tensor-core GEMV gives the same sums up to fp32 ordering
    L = _lib.lib()
    Y2 = torch.empty_like(Y)
    ws = torch.zeros(L.fbfp_gemv_workspace_bytes(16, pw.npad), dtype=torch.uint8, device=_dev())
    _lib.check(L.fbfp_gemv(_lib.ptr(X), 1, m, X.stride(0), _lib.ptr(pw.exps), _lib.ptr(pw.signs),
                           _lib.ptr(pw.payload), pw.n_out, pw.k_in, pw.kpad, pw.npad, _lib.ptr(pw.entries),
                           _lib.ptr(pw.seg_ptr), _lib.ptr(bias), 0, _lib.ptr(Y2), 0, Y2.stride(0),
                           _lib.ptr(ws), _lib.stream_ptr(_dev())), "fbfp_gemv")
    torch.cuda.synchronize()
    assert torch.allclose(Y, Y2, rtol=1e-5, atol=1e-5 * float(Y2.abs().max()))


@pytest.mark.parametrize("m", [1, 4])
def test_gemv_records_dense_only_and_bf16_out(m):
    from flashbfp_b200 import workloads
    pw, dp, sp = _packed(2048, 3840, seed=77)
    X = workloads.activations(m, 3840, seed=3, device=_dev())
    Y = _run(pw, X, None, torch.bfloat16, outliers=False)
    dpn, _ = _np(dp, sp)
    Wd = oabf.dequantize_dense(dpn["exponents"], dpn["signs"], dpn["payload"], dpn["padded_shape"],
                               dpn["orig_shape"]).astype(np.float64)
    exact = X.float().cpu().numpy().astype(np.float64) @ Wd.T
    assert oabf.rel_l2(Y.float().cpu().numpy(), exact) <= 5e-3


def test_gemv_records_dense_only_back_to_back():
    """Dense-only and full launches alternating, 24 in a row on four matrices: every result
    equals its single-launch value (the dense-only path releases no stage before it has landed)."""
    from flashbfp_b200 import linear, workloads
    mats = [_packed(4096, 3840, seed=700 + j)[0] for j in range(4)]
    X = workloads.activations(1, 3840, seed=2, device=_dev())
    ref = {(j, o): _run(mats[j], X, None, torch.float32, outliers=o) for j in range(4) for o in (True, False)}
    ws = linear.gemv_workspace(_dev(), 4096)
    outs = [torch.empty(1, 4096, dtype=torch.float32, device=_dev()) for _ in range(24)]
    for r in range(24):
        linear.gemv_records(X, mats[r % 4], outs[r], ws, None, bool(r % 2))
    linear.check_device_errors()
    for r in range(24):
        e = ref[(r % 4, bool(r % 2))]
        assert torch.allclose(outs[r], e, rtol=1e-5, atol=1e-5 * float(e.abs().max())), r


@pytest.mark.parametrize("m", [1, 16])
def test_gemv_records_outliers_beyond_the_staging_area(m):
    """20% heavy-tailed outliers: many records carry more entries than the kernel stages in shared
    memory (1208), and the rest come from global memory."""
    from flashbfp_b200 import workloads
    pw, dp, sp = _packed(1024, 3840, seed=11, frac=0.2, scale=20.0)
    seg = pw.seg_ptr[: (1024 // 128) * 15 + 1].long()
    assert int((seg[1:] - seg[:-1]).max()) > 1208
    X = workloads.activations(m, 3840, seed=5, device=_dev())
    Y = _run(pw, X, None, torch.float32)
    dpn, spn = _np(dp, sp)
    exact = oabf.linear_reference(X.float().cpu().numpy(), dpn, spn)
    assert oabf.rel_l2(Y.cpu().numpy(), exact) <= 1e-3


def test_gemv_records_graph_of_back_to_back_launches():
    """48 launches alternating between two matrices in one CUDA graph (each launch overlaps the
    previous one's tail): every output equals the eager result."""
    from flashbfp_b200 import linear, workloads
    mats = [_packed(n, k, seed=300 + i)[0] for i, (n, k) in enumerate([(3840, 4096), (8192, 3840)])]
    xs = [workloads.activations(1, pw.k_in, seed=9 + i, device=_dev()) for i, pw in enumerate(mats)]
    outs = [torch.empty(1, mats[i % 2].n_out, dtype=torch.bfloat16, device=_dev()) for i in range(48)]
    wss = [torch.zeros(linear.gemv_workspace(_dev(), pw.npad).numel(), dtype=torch.uint8, device=_dev())
           for pw in mats]
    ref = [_run(mats[j], xs[j], None, torch.bfloat16) for j in range(2)]
    st = torch.cuda.Stream(_dev())
    st.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        for i in range(48):
            linear.gemv_records(xs[i % 2], mats[i % 2], outs[i], wss[i % 2])
    torch.cuda.synchronize()
    with torch.cuda.graph(g, stream=st):
        for i in range(48):
            linear.gemv_records(xs[i % 2], mats[i % 2], outs[i], wss[i % 2])
    for _ in range(3):
        for o in outs:
            o.fill_(float("nan"))
        with torch.cuda.stream(st):
            g.replay()
        torch.cuda.synchronize()
        for i in range(48):
            r = ref[i % 2].float()
            assert torch.allclose(outs[i].float(), r, rtol=2e-2, atol=2e-2 * float(r.abs().max())), i
    for ws in wss:
        assert int(ws.count_nonzero()) == 0
    del g
