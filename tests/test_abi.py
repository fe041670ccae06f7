"""The C-ABI library loads and exports every entry point include/flashbfp.h declares.
No compute calls: these run without a GPU."""
import ctypes

import pytest

from flashbfp_b200 import _lib, build


@pytest.fixture(scope="module")
def L():
    build.build()
    return _lib.lib()


def test_header_symbols_exported(L):
    syms = _lib.header_symbols()
    assert len(syms) >= 13
    for s in syms:
        assert hasattr(L, s), s
    # every prototype the binding declares is in the header too
    assert set(_lib._PROTOS) <= set(syms)


def test_identity(L):
    assert L.fbfp_abi_version() == 1
    assert L.fbfp_status_string(0) == b"ok"
    assert L.fbfp_status_string(5) == b"device-side wait timed out"


def test_argument_errors_without_gpu(L):
    # null pointers are rejected before any CUDA call
    st = L.fbfp_gemv(None, 1, 1, 16, None, None, None, 16, 16, 16, 64, None, None, None, 0,
                     None, 1, 16, None, None)
    assert st == 1
    assert b"null" in L.fbfp_last_error()
    st = L.fbfp_dequant(None, None, None, 1, 1, 16, 0, None, 1, None)
    assert st == 1
    # the no-allocation entry checks its arguments before it touches the device or the stream
    st = L.fbfp_gemv_noalloc(None, 1, 1, 16, None, None, None, 16, 16, 16, 64, None, None, None, 0,
                             None, 1, 16, None)
    assert st == 1
    assert b"null" in L.fbfp_last_error()
    with pytest.raises(ValueError):
        _lib.check(1, "probe")
    with pytest.raises(NotImplementedError):
        _lib.check(2, "probe")


def test_workspace_sizes(L):
    assert L.fbfp_gemv_workspace_bytes(16, 4096) >= 16 * 4096 * 4 + 256 * 4
    assert L.fbfp_compress_scratch_bytes(4096, 3840, 3840, 4096) >= 4096 * 240 * 2
    assert L.fbfp_outlier_tiles_scratch_bytes(4096, 3840) >= 256 * 4 * 16 * 4
