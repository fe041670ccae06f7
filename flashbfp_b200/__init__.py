"""FlashBFP-B200: OABF (outlier-aware block floating point) weight streaming on B200.

Public API mirrors the reference package ``flash_bfp`` (``flash_bfp/__init__.py:1-8``):
``OABFCompressor``, ``oabf_gemm``, ``OABFLinear``; ``compress_gemma_model`` lives in
``flashbfp_b200.model`` as in the reference (``flash_bfp/model.py:5``).
The CUDA library ``libflashbfp.so`` is loaded on first use; every op raises if it
is missing or if its tensors are not on a CUDA device. There is no CPU fallback.
"""
__all__ = ["OABFCompressor", "oabf_gemm", "OABFLinear"]


def __getattr__(name):
    if name == "OABFCompressor":
        from .compressor import OABFCompressor
        return OABFCompressor
    if name in ("oabf_gemm", "OABFLinear"):
        from . import linear
        return getattr(linear, name)
    raise AttributeError(name)
