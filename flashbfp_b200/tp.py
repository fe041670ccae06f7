"""Tensor parallelism for OABF linears: one process per GPU.

Column-parallel linears (q/k/v/gate/up: they share the layer input and feed per-head or
element-wise work) keep a slice of output rows on every rank and need no collective.
Row-parallel linears (o/down: their input is already sharded by the previous column-parallel
layer) keep a slice of the input in whole 256-column stages, and the ranks' fp32 partial
outputs are summed: inside the GEMV itself over NVLink peer memory (``NVLinkAllReduce`` handle
with ``packed_linear_allreduce``), by a separate peer-memory all-reduce kernel, or by the
process group's all-reduce. The outlier threshold of the reference is a whole-matrix statistic
(flash_bfp/compressor.py:11-32), so every shard is compressed with the threshold of the whole
matrix; its bytes then equal the corresponding slice of the whole matrix's compression.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import packed

COLUMN_PARALLEL = ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj")
ROW_PARALLEL = ("o_proj", "down_proj")
# Row-parallel shards split K in whole 256-column stages (16 blocks of 16), the tensor-core
# GEMV's K unit: down_proj's 15360 columns at TP 8 become 1792/2048-column shards that the
# tensor-core kernel (and its fused exchange) takes, instead of 1920 that it cannot.
ROW_K_ALIGN = 256


def mode_of(name: str) -> str:
    """'column' or 'row' for a linear's module name (matched by suffix)."""
    base = name.rsplit(".", 1)[-1]
    if base in COLUMN_PARALLEL:
        return "column"
    if base in ROW_PARALLEL:
        return "row"
    raise ValueError(f"no tensor-parallel mode for {name!r}")


def split(total: int, rank: int, world: int, align: int = 1) -> Tuple[int, int]:
    """[lo, hi) of an even split of `total` items in units of `align` (remainder to the last)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    units = (total + align - 1) // align
    lo = rank * units // world * align
    hi = min(total, (rank + 1) * units // world * align)
    return lo, hi


def weight_slice(W: torch.Tensor, name: str, rank: int, world: int) -> torch.Tensor:
    """This rank's part of W [N, K]: output rows (column-parallel) or a K range in whole
    256-column stages (row-parallel)."""
    n, k = W.shape
    if mode_of(name) == "column":
        r0, r1 = split(n, rank, world, align=16)
        return W[r0:r1]
    c0, c1 = split(k, rank, world, align=ROW_K_ALIGN)
    return W[:, c0:c1]


def input_range(name: str, k: int, rank: int, world: int) -> Tuple[int, int]:
    """Columns of the layer input a row-parallel shard reads ([0, k) for column-parallel)."""
    if mode_of(name) == "column":
        return 0, k
    return split(k, rank, world, align=ROW_K_ALIGN)


def compress_shard(W: torch.Tensor, name: str, rank: int, world: int, compressor):
    """(dense_payload, sparse_outliers) of this rank's slice, with the whole matrix's threshold."""
    thr = compressor.compute_dynamic_threshold(W)
    return compressor.compress_matrix_device(weight_slice(W, name, rank, world), threshold=thr)


def slice_packed(pw: packed.PackedWeight, name: str, rank: int, world: int,
                 tiles: bool = True) -> packed.PackedWeight:
    """This rank's slice of a whole-matrix compression (the same bytes compress_shard makes)."""
    if mode_of(name) == "column":
        r0, r1 = split(pw.n_out, rank, world, align=16)
        return packed.shard_rows(pw, r0, r1 if r1 < pw.n_out else pw.npad, tiles=tiles)
    c0, c1 = split(pw.k_in, rank, world, align=ROW_K_ALIGN)
    return packed.shard_cols(pw, c0 // 16, (c1 + 15) // 16, tiles=tiles)


class DecoderPlan:
    """How a decoder's weights split over `world` ranks (whole-model tensor parallelism).

    * attention: whole heads. Rank r holds query heads [r*hq, (r+1)*hq) and KV heads
      [r*hkv, (r+1)*hkv) (hq = n_heads / world, hkv = n_kv_heads / world): its q/k/v rows, its
      KV cache, and the matching input columns of o_proj (row-parallel);
    * MLP: the intermediate dimension in whole 256-column stages, the same range for the rows of
      gate_proj and up_proj (column-parallel) and the input columns of down_proj (row-parallel);
    * lm_head: vocabulary rows in units of 64 (vocab-parallel logits, local argmax).
    Embeddings and norms are replicated."""

    def __init__(self, n_heads: int, n_kv_heads: int, head_dim: int, inter: int, vocab: int,
                 rank: int, world: int):
        if n_heads % world or n_kv_heads % world:
            raise ValueError(f"{n_heads} query / {n_kv_heads} KV heads do not split over {world} ranks")
        if not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside world {world}")
        self.rank, self.world, self.head_dim = rank, world, head_dim
        self.hq, self.hkv = n_heads // world, n_kv_heads // world
        self.q_rows = (rank * self.hq * head_dim, (rank + 1) * self.hq * head_dim)
        self.kv_rows = (rank * self.hkv * head_dim, (rank + 1) * self.hkv * head_dim)
        self.inter = split(inter, rank, world, align=ROW_K_ALIGN)
        self.vocab = split(vocab, rank, world, align=64)

    @classmethod
    def from_config(cls, cfg, rank: int, world: int) -> "DecoderPlan":
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        return cls(cfg.num_attention_heads, cfg.num_key_value_heads, head_dim, cfg.intermediate_size,
                   cfg.vocab_size, rank, world)

    def ranges(self, name: str) -> Tuple[str, int, int]:
        """(mode, lo, hi) of this rank's part of linear `name`: output rows [lo, hi) for
        'column', input columns [lo, hi) for 'row'."""
        base = name.rsplit(".", 1)[-1]
        if base == "q_proj":
            return ("column",) + self.q_rows
        if base in ("k_proj", "v_proj"):
            return ("column",) + self.kv_rows
        if base == "o_proj":
            return ("row",) + self.q_rows
        if base in ("gate_proj", "up_proj"):
            return ("column",) + self.inter
        if base == "down_proj":
            return ("row",) + self.inter
        raise ValueError(f"no tensor-parallel split for {name!r}")

    def slice(self, W: torch.Tensor, name: str) -> torch.Tensor:
        mode, lo, hi = self.ranges(name)
        return W[lo:hi] if mode == "column" else W[:, lo:hi]

    def compress(self, W: torch.Tensor, name: str, compressor):
        """(dense_payload, sparse_outliers) of this rank's part of W, with the whole matrix's
        outlier threshold (so its bytes equal that part of the whole matrix's compression)."""
        thr = compressor.compute_dynamic_threshold(W)
        return compressor.compress_matrix_device(self.slice(W, name).contiguous(), threshold=thr)


def argmax_slots(logits: torch.Tensor, vocab_offset: int, rank: int, world: int,
                 slots: torch.Tensor) -> None:
    """Vocab-parallel greedy pick, first half, for every row of ``logits`` (this rank's
    vocabulary columns): write the row's (max logit, global index of its first maximum) into
    slots [row, 2 rank : 2 rank + 2] of the zeroed fp32 ``slots`` (rows x 2 world values).
    Summing the ranks' slots (any all-reduce) then gathers every rank's pair exactly: each slot
    has one non-zero contributor, and indices below 2^24 are exact in fp32."""
    lg = logits.reshape(-1, logits.shape[-1]).float()
    val, idx = torch.max(lg, dim=-1)
    sl = slots.view(lg.shape[0], 2 * world)
    sl[:, 2 * rank].copy_(val)
    sl[:, 2 * rank + 1].copy_((idx + vocab_offset).float())


def argmax_pick(slots: torch.Tensor, world: int) -> torch.Tensor:
    """Second half: per row, the global index (int64) of the largest of the gathered maxima, the
    lowest rank's on ties, which is the first maximum over the whole vocabulary because the ranks
    hold ascending vocabulary ranges. Stays on the device (a gather, not indexing by a 0-d
    tensor, which would read it back to the host and break a CUDA graph capture)."""
    pairs = slots.view(-1, world, 2)
    best = torch.argmax(pairs[..., 0], dim=-1, keepdim=True)
    return pairs[..., 1].gather(1, best).reshape(-1).long()


def all_reduce_sum(y: torch.Tensor, group=None, reducer: Optional["NVLinkAllReduce"] = None) -> torch.Tensor:
    """Sum of the ranks' fp32 partial outputs (row-parallel exchange), in place: through the
    NVLink peer-memory reducer when one is given, else the process group's all-reduce."""
    if reducer is not None:
        return reducer(y)
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group)
    return y


class NVLinkAllReduce:
    """One-shot fp32 sum all-reduce over NVLink peer memory (csrc/allreduce.cu) for the
    row-parallel exchange. Every rank creates one (collectively: the CUDA IPC handles of the
    ranks' buffers are exchanged through the process group) on its current CUDA device; calls
    must be made by all ranks in the same order. Capturable in CUDA graphs."""

    def __init__(self, max_elems: int, group=None):
        import ctypes
        import torch.distributed as dist
        from . import _lib
        self._L = L = _lib.lib()
        self._lib = _lib
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_elems = int(max_elems)
        h = ctypes.c_void_p()
        ipc = ctypes.create_string_buffer(int(L.fbfp_allreduce_ipc_handle_bytes()))
        _lib.check(L.fbfp_allreduce_create(self.world, self.rank, self.max_elems, ctypes.byref(h), ipc),
                   "fbfp_allreduce_create")
        self._h = h
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(ipc.raw), group=group)
        for p in range(self.world):
            if p != self.rank:
                _lib.check(L.fbfp_allreduce_open_peer(h, p, handles[p]), "fbfp_allreduce_open_peer")
        dist.barrier(group=group)

    @property
    def handle(self):
        """The C-ABI handle (for fbfp_gemv_allreduce)."""
        return self._h

    def __call__(self, y: torch.Tensor) -> torch.Tensor:
        if y.dtype != torch.float32 or not y.is_contiguous():
            raise ValueError("NVLinkAllReduce sums contiguous fp32 tensors")
        self._lib.check(self._L.fbfp_allreduce_sum_f32(self._h, self._lib.ptr(y), y.numel(),
                                                       self._lib.stream_ptr(y.device)),
                        "fbfp_allreduce_sum_f32")
        return y

    def set_timeout(self, timeout_s: float) -> None:
        """Bound of every device-side wait on a peer's words, for this handle's all-reduce calls
        and the GEMV exchanges fused with it (two seconds unless changed; 1 us .. 60 s)."""
        self._lib.check(self._L.fbfp_allreduce_set_timeout(self._h, max(1, int(round(timeout_s * 1e6)))),
                        "fbfp_allreduce_set_timeout")

    def check(self, device=None) -> None:
        """Synchronise and raise if a call gave up waiting for a rank."""
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._lib.check(self._L.fbfp_allreduce_check(self._h, self._lib.stream_ptr(dev)),
                        "fbfp_allreduce_check")

    def close(self) -> None:
        if self._h:
            self._L.fbfp_allreduce_destroy(self._h)
            self._h = None


class TPLinear(torch.nn.Module):
    """One rank's shard of an OABF linear. forward(X) takes the full layer input for
    column-parallel shards and returns this rank's output columns; for row-parallel shards it
    takes the full input, reads its own K range, and returns the complete (all-reduced) output."""

    def __init__(self, pw: packed.PackedWeight, name: str, rank: int, world: int, k_full: int,
                 bias: Optional[torch.Tensor] = None, group=None,
                 reducer: Optional[NVLinkAllReduce] = None):
        super().__init__()
        self.pw, self.mode, self.rank, self.world, self.group = pw, mode_of(name), rank, world, group
        self.reducer = reducer
        self.fused_max_tokens = 64      # decode sizes: beyond this, prefill GEMM + separate exchange
        # the fused exchange only if every rank's shard takes it (collective: all ranks agree)
        self.fused_ok = False
        if reducer is not None and self.mode == "row":
            import torch.distributed as dist
            from .linear import fused_shard_eligible
            flags = [None] * world
            dist.all_gather_object(flags, fused_shard_eligible(pw, reducer.max_elems), group=group)
            self.fused_ok = all(flags)
        self.k0, self.k1 = input_range(name, k_full, rank, world)
        self.bias = bias

    def forward(self, X: torch.Tensor) -> torch.Tensor:
        from .linear import fused_exchange_eligible, packed_linear, packed_linear_allreduce
        lead = X.shape[:-1]
        X2 = X.reshape(-1, X.shape[-1])
        if self.mode == "column":
            Y = packed_linear(X2, self.pw, self.bias)
        elif (self.fused_ok and X2.shape[0] <= self.fused_max_tokens
              and fused_exchange_eligible(X2[:, self.k0:self.k1], self.pw, self.reducer.max_elems)):
            # exchange fused into the GEMV epilogue: bias added once, after the sum
            Y = packed_linear_allreduce(X2[:, self.k0:self.k1], self.pw, self.reducer, self.bias, X.dtype)
        else:
            Y = packed_linear(X2[:, self.k0:self.k1], self.pw, None, torch.float32)
            all_reduce_sum(Y, self.group, self.reducer)
            if self.bias is not None:
                Y = Y + self.bias.float()
            Y = Y.to(X.dtype)
        return Y.reshape(*lead, Y.shape[-1])
