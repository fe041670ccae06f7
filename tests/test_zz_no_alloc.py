"""fbfp_gemv_noalloc: the decode GEMV for callers that cannot allocate device memory.

Such callers (a plugin inside a host application whose memory pool owns the GPU, a thin
foreign-language binding with no device allocator) cannot hand fbfp_gemv a workspace, so this
entry point uses scratch compiled into the library. These tests call it through the C ABI
and check, on two calls in a row, that it returns what fbfp_gemv returns with a caller
workspace, and that it refuses matrices too large for its built-in scratch.
The file sorts last so that a run stopping at the first failure has run everything else.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

GEMM_TOL = 1e-2


def _setup():
    from flashbfp_b200 import build, _lib
    build.build()
    return _lib, _lib.lib()


def _packed(n, k, seed):
    from flashbfp_b200 import OABFCompressor, packed, workloads
    dev = torch.device("cuda", 0)
    W = workloads.decode_weight(n, k, seed=seed, device=dev)
    dp, sp = OABFCompressor().compress_matrix_device(W)
    return packed.from_compressed(dp, sp, dev)


def _args(_lib, X, pw, Y):
    return (_lib.ptr(X), _lib.DTYPE_CODE[X.dtype], X.shape[0], X.stride(0), _lib.ptr(pw.exps),
            _lib.ptr(pw.signs), _lib.ptr(pw.payload), pw.n_out, pw.k_in, pw.kpad, pw.npad,
            _lib.ptr(pw.entries), _lib.ptr(pw.seg_ptr), None, 0, _lib.ptr(Y),
            _lib.DTYPE_CODE[Y.dtype], Y.stride(0))


# (4096, 3840) runs on the tcgen05 kernel, (200, 3856) on the mma.sync kernel
@pytest.mark.parametrize("shape,m", [((4096, 3840), 1), ((4096, 3840), 16), ((200, 3856), 5)])
def test_noalloc_matches_workspace_gemv_twice(shape, m):
    _lib, L = _setup()
    from flashbfp_b200 import workloads
    dev = torch.device("cuda", 0)
    pw = _packed(*shape, seed=shape[0] + m)
    X = workloads.activations(m, pw.k_in, seed=m, device=dev)
    st = _lib.stream_ptr(dev)
    ws = torch.zeros(L.fbfp_gemv_workspace_bytes(16, pw.npad), dtype=torch.uint8, device=dev)
    ref = torch.empty(m, pw.n_out, dtype=torch.bfloat16, device=dev)
    _lib.check(L.fbfp_gemv(*_args(_lib, X, pw, ref), _lib.ptr(ws), st), "fbfp_gemv")
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        _lib.check(L.fbfp_gemv_noalloc(*_args(_lib, X, pw, out), st), "fbfp_gemv_noalloc")
        torch.cuda.synchronize()
        rel = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
        assert rel <= GEMM_TOL, rel


def test_noalloc_rejects_matrices_beyond_its_scratch():
    _lib, L = _setup()
    dev = torch.device("cuda", 0)
    X = torch.zeros(16, 16, dtype=torch.bfloat16, device=dev)
    dummy = torch.zeros(64, dtype=torch.int32, device=dev)
    npad = 1 << 20                            # needs ~64 MiB of scratch at m = 16
    st = L.fbfp_gemv_noalloc(_lib.ptr(X), 1, 16, 16, _lib.ptr(dummy), _lib.ptr(dummy), _lib.ptr(dummy),
                             npad, 16, 16, npad, None, None, None, 0, _lib.ptr(X), 1, npad,
                             _lib.stream_ptr(dev))
    assert st == 1
    assert b"scratch" in L.fbfp_last_error()
