"""Edge cases of the fused kernels against a PyTorch fp32 dequantize-then-matmul.

* outlier-heavy weights: more outlier entries per 128-row x 256-column stage than either kernel
  stages in shared memory (2048 for the decode GEMV, 1024 for the prefill GEMM), so the rest is
  read from global memory;
* a matrix without any outlier (uniform weights keep every value under the threshold);
* a last 128-row group that is only partly backed by the matrix (n_out = 130, npad = 192: the
  tensor copies read zeros for rows 192-255);
* bias with fp32 output at the largest decode batch (M = 16);
* an empty batch.
"""
import pytest
import torch

from flashbfp_b200 import OABFCompressor, packed, workloads, _lib
from flashbfp_b200.linear import check_device_errors, packed_linear

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _setup():
    from flashbfp_b200 import build
    build.build()
    torch.backends.cuda.matmul.allow_tf32 = False


def _full(dp, sp):
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


def _run(W, ms, bias=None, out_dtype=None, tol=5e-3):
    dev = W.device
    dp, sp = OABFCompressor().compress_matrix_device(W)
    pw = packed.from_compressed(dp, sp, dev)
    Wf = _full(dp, sp)
    for m in ms:
        X = workloads.activations(m, W.shape[1], seed=m, device=dev)
        Y = packed_linear(X, pw, bias=bias, out_dtype=out_dtype)
        check_device_errors()
        ref = X.float() @ Wf.t()
        if bias is not None:
            ref = ref + bias.float()
        rel = ((Y.float() - ref).norm() / ref.norm()).item()
        assert rel <= tol, (m, rel)
    return sp["count"], pw


def test_outlier_heavy_matrix_overflows_the_staged_window():
    W = workloads.decode_weight(1024, 3840, seed=3, frac=0.2, device="cuda")
    count, pw = _run(W, [1, 4, 16, 64, 300])
    per_stage = count / ((1024 / 128) * (3840 / 256))
    assert per_stage > 2048, per_stage          # both kernels fall back to global reads


def test_matrix_without_outliers():
    g = torch.Generator(device="cuda").manual_seed(5)
    W = ((torch.rand(512, 3840, generator=g, device="cuda") * 2 - 1) * 0.01).to(torch.bfloat16)
    count, _ = _run(W, [1, 16, 100])
    assert count == 0


def test_partly_filled_last_row_group():
    W = workloads.decode_weight(130, 3840, seed=6, device="cuda")
    _, pw = _run(W, [1, 7, 16, 33])
    assert pw.npad == 192 and pw.npad % 128 != 0 and pw.n_out == 130


def test_bias_fp32_output_at_m16():
    W = workloads.decode_weight(2048, 3840, seed=8, device="cuda")
    bias = torch.randn(2048, device="cuda") * 0.5
    _run(W, [16], bias=bias, out_dtype=torch.float32, tol=5e-3)


def test_empty_batch():
    W = workloads.decode_weight(256, 512, seed=9, device="cuda")
    dp, sp = OABFCompressor().compress_matrix_device(W)
    pw = packed.from_compressed(dp, sp, W.device)
    Y = packed_linear(torch.empty(0, 512, dtype=torch.bfloat16, device="cuda"), pw)
    assert Y.shape == (0, 256)
