"""Two-pass prefill (fbfp_gemm_expanded): expansion of the packed matrix into a bf16 scratch of
15 x its values, then a cuBLASLt bf16 GEMM scaled by 1/15.

The expansion is pinned bit-exact: dense elements s * m * 2^e (restated here in torch from the
packed arrays) and outliers bf16(15 v). The product is compared with a PyTorch fp32
dequantize-then-matmul within the bf16 bound, and with the fused tcgen05 prefill kernel, which
multiplies the same bf16 operand.
"""
import pytest
import torch

from flashbfp_b200 import OABFCompressor, _lib, packed, workloads
from flashbfp_b200.linear import (check_device_errors, expanded_eligible, gemm_expanded,
                                  packed_linear)

pytestmark = pytest.mark.gpu


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
        W = workloads.decode_weight(n, k, seed=5 * n + k, device=dev)
        dp, sp = OABFCompressor().compress_matrix_device(W)
        _CACHE[(n, k)] = (packed.from_compressed(dp, sp, dev), _dequant_full(dp, sp))
    return _CACHE[(n, k)]


def _rel(Y, ref):
    return ((Y.float() - ref).norm() / ref.norm()).item()


def _expected_x15(pw):
    """15 x W_full as bf16 from the packed arrays: s * m * 2^e per dense element (exact), then
    bf16(15 v) at every outlier."""
    n, kpad, k = pw.n_out, pw.kpad, pw.k_in
    kb = kpad // 16
    E = pw.exps.reshape(-1)[: n * kb].reshape(n, kb).int()
    S = pw.signs.reshape(-1)[: n * kb].reshape(n, kb).int() & 0xFFFF
    P = pw.payload.reshape(-1, 2)[: n * kb].reshape(n, kb, 2)
    j = torch.arange(16, device=P.device)
    word = torch.where(j < 8, P[..., 0:1], P[..., 1:2])
    m = (word >> (4 * (j % 8))) & 0xF
    val = torch.ldexp(m.float(), E.unsqueeze(-1).expand(-1, -1, 16))
    val = torch.where(((S.unsqueeze(-1) >> j) & 1) == 1, -val, val)
    out = val.reshape(n, kpad)[:, :k].to(torch.bfloat16)
    if pw.nnz:
        b, o, v = pw.coo
        g = b.long() * 16 + o.long()
        r, c = g % kpad, g // kpad
        keep = (r < k) & (c < n)
        v15 = (15.0 * v.view(torch.float16).float()).to(torch.bfloat16)
        out[c[keep], r[keep]] = v15[keep]
    return out


@pytest.mark.parametrize("index", ["tiles", "coo"])
@pytest.mark.parametrize("shape", [(4096, 3840), (192, 256), (200, 520)])
def test_expansion_bit_exact(shape, index):
    """Outliers from the tile-grouped index (written inside the expansion) or from the COO list
    (a separate scatter): the same bits either way."""
    n, k = shape
    pw, _ = _layer(n, k)
    assert pw.entries is not None and pw.nnz > 0
    L = _lib.lib()
    ldo = (k + 7) // 8 * 8
    out = torch.full((n, ldo), -1, dtype=torch.int16, device="cuda")
    b, o, v = pw.coo if index == "coo" else (None, None, None)
    ent, seg = (pw.entries, pw.seg_ptr) if index == "tiles" else (None, None)
    _lib.check(L.fbfp_expand_x15(_lib.ptr(pw.exps), _lib.ptr(pw.signs), _lib.ptr(pw.payload), n, k, pw.kpad,
                                 _lib.ptr(b), _lib.ptr(o), _lib.ptr(v), pw.nnz if index == "coo" else 0,
                                 _lib.ptr(ent), _lib.ptr(seg), pw.npad, _lib.ptr(out), ldo,
                                 _lib.stream_ptr(out.device)), "fbfp_expand_x15")
    exp = _expected_x15(pw).view(torch.int16)
    assert torch.equal(out[:, :k], exp)
    if ldo > k:                                  # columns past k_in are left alone
        assert bool((out[:, k:] == -1).all())


@pytest.mark.parametrize("m", [17, 64, 512, 1000])
@pytest.mark.parametrize("shape", [(4096, 3840), (192, 256), (3840, 4096), (200, 520)])
def test_expanded_vs_torch_fp32_and_fused(m, shape):
    n, k = shape
    pw, Wf = _layer(n, k)
    X = workloads.activations(m, k, seed=m + 1, device="cuda")
    Y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    assert expanded_eligible(X, pw, None, Y)
    gemm_expanded(X, pw, Y)
    check_device_errors()
    ref = X.float() @ Wf.t()
    assert _rel(Y, ref) <= 5e-3
    if pw.kpad % 256 == 0:                       # the fused kernel multiplies the same operand
        Yf = packed_linear(X, pw, prefill="fused")
        check_device_errors()
        assert _rel(Y, Yf.float()) <= 3e-3


def test_expanded_bias_dense_only_and_dispatch():
    pw, Wf = _layer(4096, 3840)
    X = workloads.activations(600, 3840, seed=8, device="cuda")
    bias = (torch.randn(4096, device="cuda") * 0.1).to(torch.bfloat16)
    Y = packed_linear(X, pw, bias=bias)          # 600 >= EXPANDED_MIN_M: the two-pass path
    check_device_errors()
    assert _rel(Y, X.float() @ Wf.t() + bias.float()) <= 5e-3
    Y2 = packed_linear(X, pw, bias=bias, prefill="expanded")
    assert torch.equal(Y, Y2)                    # the same algorithm twice: bit for bit
    Yd = packed_linear(X, pw, with_outliers=False, prefill="expanded")
    Yfd = packed_linear(X, pw, with_outliers=False, prefill="fused")
    check_device_errors()
    assert _rel(Yd, Yfd.float()) <= 3e-3


def test_expanded_fp32_bias_module_path():
    """OABFLinear with an fp32 bias gives fp32 outputs (dtype promotion): from EXPANDED_MIN_M
    tokens on the two-pass path writes them directly (fp32 output and bias in the GEMM)."""
    from flashbfp_b200 import OABFLinear
    n, k = 3840, 4096
    W = workloads.decode_weight(n, k, seed=78, device="cuda")
    comp = OABFCompressor()
    lin = OABFLinear(k, n, bias=True).cuda()
    lin.load_from_weight(W, comp, torch.device("cuda", 0))
    with torch.no_grad():
        lin.bias.copy_(torch.randn(n, device="cuda") * 0.1)
    dp, sp = comp.compress_matrix_device(W)
    Wf = _dequant_full(dp, sp)
    X = workloads.activations(1024, k, seed=6, device="cuda").reshape(4, 256, k)
    Y = lin(X)
    check_device_errors()
    assert Y.dtype == torch.float32 and Y.shape == (4, 256, n)
    ref = X.reshape(1024, k).float() @ Wf.t() + lin.bias.float()
    assert _rel(Y.reshape(1024, n), ref) <= 5e-3
    Yf = packed_linear(X.reshape(1024, k), lin._pw, lin.bias, torch.float32, prefill="fused")
    check_device_errors()
    assert _rel(Y.reshape(1024, n), Yf) <= 3e-3


def test_expanded_rejects_small_scratch():
    pw, _ = _layer(192, 256)
    L = _lib.lib()
    X = torch.zeros(64, 256, dtype=torch.bfloat16, device="cuda")
    Y = torch.empty(64, 192, dtype=torch.bfloat16, device="cuda")
    small = torch.empty(4096, dtype=torch.uint8, device="cuda")
    st = L.fbfp_gemm_expanded(_lib.ptr(X), 64, 256, _lib.ptr(pw.exps), _lib.ptr(pw.signs), _lib.ptr(pw.payload),
                              pw.n_out, pw.k_in, pw.kpad, None, None, None, 0, None, None, pw.npad, None,
                              _lib.ptr(Y), _lib.DTYPE_CODE[torch.bfloat16], 192, _lib.ptr(small), small.numel(),
                              _lib.stream_ptr(X.device))
    assert st == 1 and b"scratch" in L.fbfp_last_error()
