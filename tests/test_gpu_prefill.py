"""Prefill GEMM (fbfp_gemm_prefill, tcgen05) against a PyTorch fp32 dequantize-then-matmul.

The weights' dequantisation itself is pinned bit-exact to the oracle by test_gpu_parity.py; here
the full product Y = X @ W_full^T (+ bias) at prefill token counts is compared within the bf16
bound (rel-L2 <= 1e-2; fp32 accumulation leaves the bf16 output rounding dominant).
"""
import pytest
import torch

from flashbfp_b200 import OABFCompressor, OABFLinear, _lib, packed, workloads
from flashbfp_b200.linear import check_device_errors, gemv_workspace, packed_linear, prefill_eligible

pytestmark = pytest.mark.gpu

GEMM_TOL = 1e-2


@pytest.fixture(scope="module", autouse=True)
def _setup():
    from flashbfp_b200 import build
    build.build()
    torch.backends.cuda.matmul.allow_tf32 = False


def _dequant_full(dp, sp):
    L = _lib.lib()
    n, k = dp["orig_shape"]
    kpad, _ = dp["padded_shape"]
    dev = dp["exponents"].device
    W = torch.empty(n, k, dtype=torch.float32, device=dev)
    st = _lib.stream_ptr(dev)
    _lib.check(L.fbfp_dequant(_lib.ptr(dp["exponents"]), _lib.ptr(dp["signs"]), _lib.ptr(dp["payload"]),
                              n, k, kpad, _lib.DTYPE_CODE[torch.float32], _lib.ptr(W), k, st), "dequant")
    if sp["count"]:
        _lib.check(L.fbfp_scatter_outliers(_lib.ptr(sp["block_idx"]), _lib.ptr(sp["offset"]),
                                           _lib.ptr(sp["value"]), sp["count"], kpad, n, k,
                                           _lib.DTYPE_CODE[torch.float32], _lib.ptr(W), k, st), "scatter")
    return W


_CACHE = {}


def _layer(n, k):
    if (n, k) not in _CACHE:
        dev = torch.device("cuda", 0)
        W = workloads.decode_weight(n, k, seed=3 * n + k, device=dev)
        dp, sp = OABFCompressor().compress_matrix_device(W)
        _CACHE[(n, k)] = (packed.from_compressed(dp, sp, dev), _dequant_full(dp, sp), dp)
    return _CACHE[(n, k)]


def _rel(Y, ref):
    return ((Y.float() - ref).norm() / ref.norm()).item()


@pytest.mark.parametrize("m", [17, 64, 255, 256, 257, 512, 1000])
@pytest.mark.parametrize("shape", [(4096, 3840), (192, 256), (3840, 4096)])
def test_prefill_vs_torch_fp32(m, shape):
    n, k = shape
    pw, Wf, _ = _layer(n, k)
    X = workloads.activations(m, k, seed=m, device="cuda")
    assert prefill_eligible(X, pw)
    Y = packed_linear(X, pw)
    check_device_errors()
    rel = _rel(Y, X.float() @ Wf.t())
    assert rel <= 5e-3, rel
    assert rel <= GEMM_TOL


def test_prefill_large_k_and_many_tokens():
    """down-projection shape (K = 15360, 60 stages per tile) at 2048 tokens."""
    pw, Wf, _ = _layer(3840, 15360)
    X = workloads.activations(2048, 15360, seed=5, device="cuda")
    Y = packed_linear(X, pw)
    check_device_errors()
    assert _rel(Y, X.float() @ Wf.t()) <= 5e-3


def test_prefill_bias_fp32_out_and_strided_x():
    pw, Wf, _ = _layer(4096, 3840)
    base = workloads.activations(300, 3848, seed=9, device="cuda")
    X = base[:, :3840]                                  # leading dimension 3848
    bias = torch.randn(4096, device="cuda", dtype=torch.bfloat16)
    Y = packed_linear(X, pw, bias=bias, out_dtype=torch.float32)
    check_device_errors()
    ref = X.float() @ Wf.t() + bias.float()
    assert Y.dtype == torch.float32
    # fp32 output: what remains is the bf16 rounding of the outlier values (bf16(15 v) in the
    # product, as the reference rounds v to the activation dtype), about 1.6e-3 here
    assert _rel(Y, ref) <= 5e-3


def test_prefill_dense_only_matches_oabf_gemm_semantics():
    """with_outliers=False gives the dense part only (oabf_gemm, triton_kernel.py:130-195)."""
    pw, _, dp = _layer(4096, 3840)
    n, k = dp["orig_shape"]
    L = _lib.lib()
    Wd = torch.empty(n, k, dtype=torch.float32, device="cuda")
    _lib.check(L.fbfp_dequant(_lib.ptr(dp["exponents"]), _lib.ptr(dp["signs"]), _lib.ptr(dp["payload"]),
                              n, k, dp["padded_shape"][0], _lib.DTYPE_CODE[torch.float32], _lib.ptr(Wd), k,
                              _lib.stream_ptr(Wd.device)), "dequant")
    X = workloads.activations(512, k, seed=2, device="cuda")
    Y = packed_linear(X, pw, with_outliers=False)
    assert _rel(Y, X.float() @ Wd.t()) <= 5e-3


def test_prefill_module_path_and_repeatability():
    """OABFLinear.forward routes M > 16 to the prefill kernel (3-D input, fp32 bias); two calls
    agree bit for bit and match the fp32 reference."""
    n, k = 3840, 4096
    W = workloads.decode_weight(n, k, seed=77, device="cuda")
    comp = OABFCompressor()
    lin = OABFLinear(k, n, bias=True).cuda()
    lin.load_from_weight(W, comp, torch.device("cuda", 0))
    with torch.no_grad():
        lin.bias.copy_(torch.randn(n, device="cuda") * 0.1)
    dp, sp = comp.compress_matrix_device(W)
    Wf = _dequant_full(dp, sp)
    X = workloads.activations(700, k, seed=4, device="cuda").reshape(7, 100, k)
    Y1 = lin(X)
    Y2 = lin(X)
    check_device_errors()
    assert Y1.shape == (7, 100, n)
    assert torch.equal(Y1, Y2)
    ref = X.reshape(700, k).float() @ Wf.t() + lin.bias.float()
    assert _rel(Y1.reshape(700, n), ref) <= 5e-3


def test_prefill_rejects_fp32_activations_at_the_abi():
    pw, _, _ = _layer(192, 256)
    L = _lib.lib()
    X = torch.zeros(64, 256, dtype=torch.float32, device="cuda")
    Y = torch.empty(64, 192, dtype=torch.float32, device="cuda")
    ws = gemv_workspace(X.device, pw.npad)
    st = L.fbfp_gemm_prefill(_lib.ptr(X), _lib.DTYPE_CODE[torch.float32], 64, 256, _lib.ptr(pw.exps),
                             _lib.ptr(pw.signs), _lib.ptr(pw.payload), pw.n_out, pw.k_in, pw.kpad, pw.npad,
                             None, None, None, 0, _lib.ptr(Y), _lib.DTYPE_CODE[torch.float32], 192,
                             _lib.ptr(ws), _lib.stream_ptr(X.device))
    assert st == 1 and b"bf16" in L.fbfp_last_error()


def test_fp32_activations_still_run_through_the_gemv_chunks():
    pw, Wf, _ = _layer(192, 256)
    X = torch.randn(40, 256, device="cuda")
    Y = packed_linear(X, pw)
    check_device_errors()
    assert _rel(Y, X.float() @ Wf.t()) <= GEMM_TOL
