"""``oabf_gemm`` and ``OABFLinear`` on B200 kernels.

Mirrors flash_bfp/triton_kernel.py: ``oabf_gemm(X, dense_payload)`` (:130-195) returns the
dense part ``X @ deq(W)^T`` (no outliers) in X's dtype; ``OABFLinear`` (:198-423) keeps the
constructor, ``load_from_weight``, ``forward`` and the ``state_dict`` key layout. Unlike
the reference there is no CPU fallback: inputs must be CUDA tensors and the CUDA library
must be built, otherwise the call raises.

Device-resident form of a layer (``packed.py``): the reference's packed bytes (11 per 16
weights) plus each outlier twice, in the reference's COO form (10 bytes, kept for state_dict,
slicing and saving) and grouped for the fused kernels (4 bytes). ``packed_linear`` sends up to
16 tokens per launch through the decode GEMV and more through the tcgen05 prefill GEMM;
``packed_linear_allreduce`` is the row-parallel GEMV with the cross-rank sum fused in.
"""
from __future__ import annotations

from typing import Dict

import torch

from . import _lib
from .compressor import padded_dims
from .packed import PackedWeight, from_compressed

# ------------------------------------------------------------------------------------
# per-(device, stream) zero-initialised GEMV workspaces (the kernel leaves them zeroed)
# ------------------------------------------------------------------------------------
_WORKSPACES: Dict[tuple, torch.Tensor] = {}


def gemv_workspace(device: torch.device, npad: int) -> torch.Tensor:
    L = _lib.lib()
    need = L.fbfp_gemv_workspace_bytes(16, npad)
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(need, dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def check_device_errors(device=None) -> None:
    """Synchronise and raise if a GEMV on `device` gave up a bounded device-side wait. The
    workspace of a GEMV that gave up may hold partial sums and counters, so it is returned to
    zero before the error is raised: later GEMVs on it are correct again."""
    L = _lib.lib()
    for (idx, sptr), ws in list(_WORKSPACES.items()):
        if device is not None and torch.device(device).index != idx:
            continue
        with torch.cuda.device(idx):
            try:
                _lib.check(L.fbfp_gemv_check(_lib.ptr(ws), _lib.ctypes.c_void_p(sptr)), "fbfp_gemv_check")
            except _lib.FlashBFPError:
                ws.zero_()
                torch.cuda.synchronize(idx)
                raise


GEMV_RESIDENT, GEMV_DENSE_ONLY, GEMV_TENSOR_CORES = 1, 4, 8


def records_eligible(X: torch.Tensor, pw: PackedWeight) -> bool:
    """Whether the stage-record GEMV takes X (at most 16 tokens per launch) on pw (its records
    built by ``PackedWeight.build_records``). ``packed_linear`` sends it one-token launches."""
    return (pw.records is not None and X.dtype == torch.bfloat16 and X.stride(1) == 1
            and X.stride(0) % 8 == 0 and X.data_ptr() % 16 == 0 and pw.k_in % 8 == 0)


def gemv_records(X: torch.Tensor, pw: PackedWeight, Y: torch.Tensor, ws: torch.Tensor,
                 bias: torch.Tensor | None = None, with_outliers: bool = True, reducer=None,
                 tensor_cores: bool = False) -> None:
    """Y[:M] = X[:M] @ W^T (+ outliers) (+ bias) for M <= 16 through fbfp_gemv_records; with
    ``reducer`` (an NVLinkAllReduce) the row-parallel sum over its ranks is fused in. One token
    runs on the CUDA cores unless ``tensor_cores``."""
    L = _lib.lib()
    bd = _lib.dtype_code(bias.dtype, "bias") if bias is not None else 0
    flags = ((GEMV_RESIDENT if pw.resident else 0) | (0 if with_outliers else GEMV_DENSE_ONLY)
             | (GEMV_TENSOR_CORES if tensor_cores else 0))
    _lib.check(L.fbfp_gemv_records(_lib.ptr(X), X.shape[0], X.stride(0), _lib.ptr(pw.records), pw.n_out,
                                   pw.k_in, pw.kpad, pw.npad, _lib.ptr(bias), bd, _lib.ptr(Y),
                                   _lib.dtype_code(Y.dtype, "Y"), Y.stride(0), _lib.ptr(ws),
                                   reducer.handle if reducer is not None else None, flags,
                                   _lib.stream_ptr(X.device)), "fbfp_gemv_records")


def prefill_eligible(X: torch.Tensor, pw: PackedWeight) -> bool:
    """Shapes the tcgen05 prefill GEMM takes; others run as 16-token GEMV launches."""
    def a16(t):
        return t.data_ptr() % 16 == 0
    return (X.dtype == torch.bfloat16 and pw.kpad % 256 == 0 and pw.k_in % 8 == 0
            and X.stride(0) % 8 == 0 and a16(X) and a16(pw.payload) and a16(pw.signs) and a16(pw.exps))


# From this many tokens on, bf16 prefill runs in two passes (fbfp_gemm_expanded): the matrix is
# expanded once into a bf16 scratch and multiplied by a cuBLASLt GEMM. Below it the fused
# tcgen05 kernel (fbfp_gemm_prefill) is the faster one, unless it has fewer tiles (128 rows x 256
# tokens) than the GPU has SMs, which the two-pass path also takes from 32 tokens on (measured:
# a 3840x15360 matrix at 128 tokens 83 against 182 us, 8192x3840 45 against 60 us; a
# 30720x3840 one, 240 fused tiles, keeps the fused kernel: 111 against 154 us).
EXPANDED_MIN_M = 512
EXPANDED_MIN_M_FEW_TILES = 32
_EXPAND_SCRATCH: Dict[int, torch.Tensor] = {}
_SM_COUNT: Dict[int, int] = {}


def expanded_preferred(M: int, pw: PackedWeight, device) -> bool:
    """Whether packed_linear sends M tokens to the two-pass path (when eligible)."""
    idx = torch.device(device).index or 0
    if idx not in _SM_COUNT:
        _SM_COUNT[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    tiles = -(-pw.npad // 128) * -(-M // 256)
    return M >= EXPANDED_MIN_M or (M >= EXPANDED_MIN_M_FEW_TILES and tiles < _SM_COUNT[idx])


def expanded_eligible(X: torch.Tensor, pw: PackedWeight, bias: torch.Tensor | None,
                      Y: torch.Tensor) -> bool:
    """Whether fbfp_gemm_expanded takes this call: bf16 activations, a bf16 or fp32 output with a
    bias (if any) of the same type, 16-byte aligned rows, and not inside a CUDA-graph capture
    (the scratch may have to grow)."""
    def ok(t):
        return (t.stride(-1) == 1 and (t.stride(0) * t.element_size()) % 16 == 0
                and t.data_ptr() % 16 == 0)
    return (X.dtype == torch.bfloat16 and Y.dtype in (torch.bfloat16, torch.float32) and ok(X) and ok(Y)
            and (bias is None or (bias.dtype == Y.dtype and bias.is_contiguous()
                                  and bias.data_ptr() % 16 == 0))
            and pw.k_in % 8 == 0 and not torch.cuda.is_current_stream_capturing())


def expand_scratch(device: torch.device, nbytes: int) -> torch.Tensor:
    """The device's scratch for fbfp_gemm_expanded (kept and grown to the largest request)."""
    idx = torch.device(device).index
    buf = _EXPAND_SCRATCH.get(idx)
    if buf is None or buf.numel() < nbytes:
        _EXPAND_SCRATCH.pop(idx, None)
        buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _EXPAND_SCRATCH[idx] = buf
    return buf


def gemm_expanded(X: torch.Tensor, pw: PackedWeight, Y: torch.Tensor, bias: torch.Tensor | None = None,
                  with_outliers: bool = True) -> None:
    """Y = X @ W^T (+ outliers) (+ bias) in two passes (fbfp_gemm_expanded): the packed matrix
    expanded into a bf16 scratch as 15 x its values, then a cuBLASLt bf16 GEMM scaled by 1/15."""
    L = _lib.lib()
    need = L.fbfp_gemm_expanded_scratch_bytes(pw.n_out, pw.kpad)
    scratch = expand_scratch(X.device, need)
    # the outliers as the COO list (a separate scatter launch): writing them inside the
    # expansion from the tile-grouped index measured no faster (one more dependent load chain
    # per block)
    coo = pw.coo if (with_outliers and pw.nnz > 0) else None
    b, o, v = coo if coo is not None else (None, None, None)
    _lib.check(L.fbfp_gemm_expanded(_lib.ptr(X), X.shape[0], X.stride(0), _lib.ptr(pw.exps), _lib.ptr(pw.signs),
                                    _lib.ptr(pw.payload), pw.n_out, pw.k_in, pw.kpad, _lib.ptr(b), _lib.ptr(o),
                                    _lib.ptr(v), pw.nnz if coo is not None else 0,
                                    None, None, pw.npad, _lib.ptr(bias), _lib.ptr(Y),
                                    _lib.dtype_code(Y.dtype, "Y"), Y.stride(0), _lib.ptr(scratch), scratch.numel(),
                                    _lib.stream_ptr(X.device)), "fbfp_gemm_expanded")


def packed_linear(X: torch.Tensor, pw: PackedWeight, bias: torch.Tensor | None = None,
                  out_dtype: torch.dtype | None = None, with_outliers: bool = True,
                  out: torch.Tensor | None = None, prefill: str | None = None) -> torch.Tensor:
    """Y[M, n_out] = X[M, k] @ W^T (+ outliers) (+ bias) through the CUDA kernels.

    ``prefill`` picks the path for M > 16: "fused" (fbfp_gemm_prefill), "expanded"
    (fbfp_gemm_expanded, where eligible) or None (``expanded_preferred``)."""
    L = _lib.lib()
    _lib.require_cuda(X, "X")
    if X.dim() != 2:
        raise ValueError("packed_linear expects a 2-D X")
    if X.stride(1) != 1:
        X = X.contiguous()
    M, Kx = X.shape
    if Kx < pw.k_in:
        raise ValueError(f"X has {Kx} columns, the weight needs {pw.k_in}")
    out_dtype = out_dtype or X.dtype
    xd = _lib.dtype_code(X.dtype, "X")
    yd = _lib.dtype_code(out_dtype, "Y")
    Y = out if out is not None else torch.empty(M, pw.n_out, dtype=out_dtype, device=X.device)
    if M == 0:
        return Y
    use_out = with_outliers and pw.nnz > 0 and pw.entries is not None
    entries = pw.entries if use_out else None
    seg_ptr = pw.seg_ptr if use_out else None
    bd = _lib.dtype_code(bias.dtype, "bias") if bias is not None else 0
    ws = gemv_workspace(X.device, pw.npad)
    st = _lib.stream_ptr(X.device)
    if M > 16 and prefill != "fused" and (prefill == "expanded" or expanded_preferred(M, pw, X.device)) \
            and expanded_eligible(X, pw, bias, Y):
        gemm_expanded(X, pw, Y, bias, with_outliers)
        return Y
    if M > 16 and prefill_eligible(X, pw):
        _lib.check(L.fbfp_gemm_prefill(_lib.ptr(X), xd, M, X.stride(0), _lib.ptr(pw.exps),
                                       _lib.ptr(pw.signs), _lib.ptr(pw.payload), pw.n_out, pw.k_in,
                                       pw.kpad, pw.npad, _lib.ptr(entries), _lib.ptr(seg_ptr),
                                       _lib.ptr(bias), bd, _lib.ptr(Y), yd, Y.stride(0), _lib.ptr(ws), st),
                   "fbfp_gemm_prefill")
        return Y
    if M == 1 and records_eligible(X, pw):
        # one token: the stage-record kernel on the CUDA cores (faster than the tcgen05 GEMV
        # at one token; from two tokens on, the tcgen05 GEMV below is the faster one)
        gemv_records(X, pw, Y, ws, bias, with_outliers)
        return Y
    gemv = L.fbfp_gemv_resident if pw.resident else L.fbfp_gemv
    for m0 in range(0, M, 16):
        m = min(16, M - m0)
        _lib.check(gemv(_lib.ptr(X[m0:m0 + m]), xd, m, X.stride(0), _lib.ptr(pw.exps),
                               _lib.ptr(pw.signs), _lib.ptr(pw.payload), pw.n_out, pw.k_in, pw.kpad,
                               pw.npad, _lib.ptr(entries), _lib.ptr(seg_ptr), _lib.ptr(bias), bd,
                               _lib.ptr(Y[m0:m0 + m]), yd, Y.stride(0), _lib.ptr(ws), st),
                   "fbfp_gemv")
    return Y


def fused_shard_eligible(pw: PackedWeight, max_elems: int) -> bool:
    """Whether the tensor-core GEMV takes shard pw (kpad a multiple of 256, k_in of 8, aligned
    arrays) and 16 x n_out values fit the exchange buffers of ``max_elems`` elements."""
    return (pw.kpad % 256 == 0 and pw.k_in % 8 == 0 and 16 * pw.n_out <= max_elems
            and all(t.data_ptr() % 16 == 0 for t in (pw.exps, pw.signs, pw.payload)))


def fused_exchange_eligible(X: torch.Tensor, pw: PackedWeight, max_elems: int) -> bool:
    """Whether ``packed_linear_allreduce`` can run X (at most 16 tokens per launch) on pw: the
    tensor-core GEMV's operand rules and room for 16 x n_out values in the exchange buffers."""
    return (X.is_cuda and X.dim() == 2 and X.dtype == torch.bfloat16 and X.stride(1) == 1
            and X.stride(0) % 8 == 0 and X.data_ptr() % 16 == 0 and fused_shard_eligible(pw, max_elems))


def packed_linear_allreduce(X: torch.Tensor, pw: PackedWeight, reducer, bias: torch.Tensor | None = None,
                            out_dtype: torch.dtype | None = None,
                            out: torch.Tensor | None = None) -> torch.Tensor:
    """Row-parallel shard product with the exchange fused into the GEMV (fbfp_gemv_allreduce):
    every rank of ``reducer`` (an ``NVLinkAllReduce``) calls it with its K slice X and shard pw,
    and gets Y = bias + the sum over ranks of X_r @ W_r^T, identical on all ranks."""
    L = _lib.lib()
    if not fused_exchange_eligible(X, pw, reducer.max_elems):
        raise ValueError("packed_linear_allreduce: operands not eligible for the fused exchange")
    M = X.shape[0]
    out_dtype = out_dtype or X.dtype
    Y = out if out is not None else torch.empty(M, pw.n_out, dtype=out_dtype, device=X.device)
    if M == 0:
        return Y
    use_out = pw.nnz > 0 and pw.entries is not None
    entries = pw.entries if use_out else None
    seg_ptr = pw.seg_ptr if use_out else None
    bd = _lib.dtype_code(bias.dtype, "bias") if bias is not None else 0
    xd = _lib.dtype_code(X.dtype, "X")
    yd = _lib.dtype_code(out_dtype, "Y")
    ws = gemv_workspace(X.device, pw.npad)
    st = _lib.stream_ptr(X.device)
    if M == 1 and records_eligible(X, pw):
        gemv_records(X, pw, Y, ws, bias, True, reducer)
        return Y
    for m0 in range(0, M, 16):
        m = min(16, M - m0)
        _lib.check(L.fbfp_gemv_allreduce(_lib.ptr(X[m0:m0 + m]), xd, m, X.stride(0), _lib.ptr(pw.exps),
                                         _lib.ptr(pw.signs), _lib.ptr(pw.payload), pw.n_out, pw.k_in,
                                         pw.kpad, pw.npad, _lib.ptr(entries), _lib.ptr(seg_ptr),
                                         _lib.ptr(bias), bd, _lib.ptr(Y[m0:m0 + m]), yd, Y.stride(0),
                                         _lib.ptr(ws), reducer.handle, 1 if pw.resident else 0, st),
                   "fbfp_gemv_allreduce")
    return Y


def oabf_gemm(X: torch.Tensor, dense_payload: Dict) -> torch.Tensor:
    """Dense part of the OABF product, ``X @ deq(W)^T`` in X's dtype (triton_kernel.py:130-195).

    ``dense_payload`` is the compressor's dict; its tensors may live on the CPU (they are
    copied to X's device) and may use the reference's widened GPU dtypes (fp32 exponents,
    int32 signs, flat int32 payload; triton_kernel.py:101-110,147-158).
    """
    _lib.require_cuda(X, "X")
    pw = from_compressed(dense_payload, None, X.device, build_tiles=False)
    with torch.cuda.device(X.device):
        return packed_linear(X, pw, None, X.dtype, with_outliers=False)


class OABFLinear(torch.nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = True):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.has_bias = bias
        self.compressed = False
        self._payload_meta = {}
        self._sparse_meta = {}
        # serialisation placeholders with the reference's names (triton_kernel.py:209-211);
        # state_dict() fills them from the compact device form
        self.register_buffer("_dp_exponents", torch.empty(0, dtype=torch.float32))
        self.register_buffer("_sp_value", torch.empty(0, dtype=torch.float32))
        if bias:
            self.bias = torch.nn.Parameter(torch.zeros(out_features))
        else:
            self.register_parameter("bias", None)
        self._pw: PackedWeight | None = None

    def _apply(self, fn, *args, **kwargs):
        super()._apply(fn, *args, **kwargs)
        if self._pw is not None:
            self._pw.apply(fn)                 # integer tensors: dtype casts leave them alone
        return self

    # -- triton_kernel.py:218-293 --------------------------------------------------------
    def load_from_weight(self, W: torch.Tensor, compressor, device):
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("OABFLinear runs on a CUDA device (FlashBFP-B200 has no CPU path)")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        if W.device.type == "meta":
            W = torch.zeros(W.shape, dtype=W.dtype)
        with torch.cuda.device(device):
            W = W.to(device)
            if hasattr(compressor, "compress_matrix_device"):
                dp, sp = compressor.compress_matrix_device(W)
            else:
                dp, sp = compressor.compress_matrix(W)
        self.load_compressed(dp, sp, device)

    def load_compressed(self, dp: Dict, sp: Dict, device) -> None:
        """Adopt the compressor's (dense_payload, sparse_outliers) dicts."""
        kpad, npad = dp["padded_shape"]
        count = int(sp["count"])
        if count:
            b = sp["block_idx"].to(device).long()
            o = sp["offset"].to(device).long()
            g = b * 16 + o
            if bool((b < 0).any()) or bool((o < 0).any()) or bool((o >= 16).any()) \
                    or bool((g // kpad >= npad).any()):
                raise IndexError("FlashBFP Compressor Error: outlier index out of padded bounds "
                                 f"[0, {kpad - 1}] x [0, {npad - 1}]")
        with torch.cuda.device(device):
            pw = from_compressed(dp, sp, device, build_tiles=False)
            pw.n_out, pw.k_in = self.out_features, self.in_features
            pw.build_tiles()
        self._pw = pw
        self._payload_meta = {"padded_shape": (pw.kpad, pw.npad),
                              "orig_shape": tuple(int(v) for v in dp["orig_shape"])}
        self._sparse_meta = {"count": count}
        self.compressed = True

    @property
    def packed(self) -> PackedWeight:
        if not self.compressed:
            raise RuntimeError("Weight matrix has not been compressed and loaded.")
        return self._pw

    # -- triton_kernel.py:295-368 --------------------------------------------------------
    def forward(self, X: torch.Tensor) -> torch.Tensor:
        if not self.compressed:
            raise RuntimeError("Weight matrix has not been compressed and loaded.")
        _lib.require_cuda(X, "X")
        orig_shape = X.shape
        in_dev = X.device
        pw = self._pw
        Xf = X.reshape(-1, self.in_features)
        if Xf.device != pw.device:
            Xf = Xf.to(pw.device)
        bias = self.bias
        if bias is not None and bias.device != pw.device:
            bias = bias.to(pw.device)
        out_dtype = X.dtype if bias is None else torch.promote_types(X.dtype, bias.dtype)
        with torch.cuda.device(pw.device):
            Y = packed_linear(Xf, pw, bias, out_dtype, with_outliers=True)
        if Y.device != in_dev:
            Y = Y.to(in_dev)
        return Y.view(*orig_shape[:-1], self.out_features)

    # -- triton_kernel.py:370-423: reference key layout ---------------------------------
    def _reference_tensors(self):
        pw = self._pw
        out = {
            "_dp_exponents": pw.exps.to(torch.float32),
            "_dp_signs": pw.signs.to(torch.int32),
            "_dp_payload": pw.payload.reshape(-1).clone(),
        }
        if pw.nnz:
            bidx, off, val = pw.coo
            g = bidx.long() * 16 + off.long()
            r = g % pw.kpad
            c = g // pw.kpad
            keep = (r < self.in_features) & (c < self.out_features)
            out["_sp_value"] = val.view(torch.float16).to(torch.float32)
            out["_sp_r_idx"] = r[keep]
            out["_sp_c_idx"] = c[keep]
            out["_sp_v_val"] = val.view(torch.float16)[keep].to(torch.float32)
        else:
            out["_sp_value"] = torch.empty(0, dtype=torch.float32, device=pw.device)
        return out

    def state_dict(self, *args, destination=None, prefix="", keep_vars=False):
        state = super().state_dict(destination=destination, prefix=prefix, keep_vars=keep_vars)
        if self.compressed:
            for k, v in self._reference_tensors().items():
                state[prefix + k] = v
        return state

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                              unexpected_keys, error_msgs):
        keys = ["_dp_exponents", "_dp_signs", "_dp_payload", "_sp_value", "_sp_r_idx", "_sp_c_idx",
                "_sp_v_val"]
        got = {k: state_dict.pop(prefix + k) for k in keys if prefix + k in state_dict}
        for k in ("_dp_exponents", "_sp_value"):       # let the placeholder buffers load empty
            state_dict[prefix + k] = torch.empty(0, dtype=torch.float32)
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys,
                                      unexpected_keys, error_msgs)
        for k in ("_dp_exponents", "_sp_value"):
            state_dict.pop(prefix + k, None)
        if not {"_dp_signs", "_dp_payload", "_dp_exponents"} <= set(got):
            return
        # padded shape from the layer dimensions with block 16 / tile 64 (triton_kernel.py:405-411)
        kpad, npad = padded_dims(self.out_features, self.in_features, 16, 64)
        if self._pw is not None:
            device = self._pw.device
        elif self.bias is not None and self.bias.is_cuda:
            device = self.bias.device
        else:
            device = torch.device("cuda", torch.cuda.current_device())
        dp = {
            "exponents": got["_dp_exponents"].to(device),
            "signs": got["_dp_signs"].to(device),
            "payload": got["_dp_payload"].to(device),
            "orig_shape": torch.Size((self.out_features, self.in_features)),
            "padded_shape": (kpad, npad),
        }
        if "_sp_r_idx" in got:
            r = got["_sp_r_idx"].to(device).long()
            c = got["_sp_c_idx"].to(device).long()
            g = c * kpad + r
            order = torch.argsort(g)
            g = g[order]
            sp = {"block_idx": (g // 16).to(torch.int32), "offset": (g % 16).to(torch.int32),
                  "value": got["_sp_v_val"].to(device)[order].to(torch.float16),
                  "count": int(g.numel())}
        else:
            z = torch.zeros(0, dtype=torch.int32, device=device)
            sp = {"block_idx": z, "offset": z.clone(),
                  "value": torch.zeros(0, dtype=torch.float16, device=device), "count": 0}
        self.load_compressed(dp, sp, device)


def _main(argv=None) -> None:
    """``python -m flashbfp_b200.linear [N K M [path [reps]]]``: time ``packed_linear`` on a seeded
    N x K OABF weight (N(0, 0.02) bf16 with 1.5% heavy-tailed outliers, compressed on the GPU) at M
    bf16 tokens, after two warm-up calls; ``path`` is fused, expanded or auto (the default
    choice). Prints the time per call and the tensor rate."""
    import json
    import sys
    from . import workloads
    from .compressor import OABFCompressor
    args = sys.argv[1:] if argv is None else list(argv)
    n, k, m = (int(args[0]), int(args[1]), int(args[2])) if len(args) >= 3 else (30720, 3840, 2048)
    path = args[3] if len(args) >= 4 else "auto"
    reps = int(args[4]) if len(args) >= 5 else 5
    if path not in ("fused", "expanded", "auto"):
        raise SystemExit("path must be fused, expanded or auto")
    dev = torch.device("cuda", torch.cuda.current_device())
    W = workloads.decode_weight(n, k, seed=21, device=dev)
    dp, sp = OABFCompressor().compress_matrix_device(W)
    del W
    pw = from_compressed(dp, sp, dev)
    X = workloads.activations(m, k, seed=11, device=dev)
    Y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    choice = None if path == "auto" else path
    for _ in range(2):
        packed_linear(X, pw, out=Y, prefill=choice)
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        packed_linear(X, pw, out=Y, prefill=choice)
    b.record()
    torch.cuda.synchronize(dev)
    check_device_errors(dev)
    ms = a.elapsed_time(b) / reps
    print(json.dumps({"shape": [n, k], "m": m, "path": path, "ms": round(ms, 4),
                      "tflops": round(2.0 * m * n * k / ms / 1e9, 1)}))


if __name__ == "__main__":
    _main()
