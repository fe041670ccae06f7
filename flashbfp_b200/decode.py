"""One Gemma-3 decode token on the GPU, replayed from a single CUDA graph.

The linears run as OABF GEMVs (q|k|v and gate|up fused into one launch each); the work between
them runs in the kernels of csrc/decode.cu: the scaled embedding, the RMSNorms (the post-norm,
residual add and next pre-norm between a layer's halves in one kernel), q/k RMSNorm with the
rotary embedding and the KV-cache append, decode attention (GQA, sliding window on the layers
that have one) and the GeGLU activation. lm_head stays an uncompressed bf16 linear, as in the
reference, whose model surgery leaves it alone (flash_bfp/model.py:23-28), and the greedy pick
is an argmax. The token and its position live on the device, so one replay is one token with no
host work in between.

A prompt goes through ``prefill`` as one chunk of rows: the same kernels over M rows at
consecutive positions (causal attention per row), the linears as M-token launches (the tcgen05
prefill GEMM once M > 16), and logits for the last row only.

``GemmaDecoder.from_hf`` takes a Hugging Face Gemma-3 causal LM after ``compress_gemma_model``;
``GemmaDecoder(...)`` takes the parts directly (used by the benchmark's random-init 12B-class
model).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch

from . import _lib
from .linear import packed_linear, packed_linear_allreduce
from .packed import PackedWeight, concat_rows


@dataclass
class DecoderShape:
    hidden: int
    inter: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    layer_types: Sequence[str]            # "sliding_attention" / "full_attention" per layer
    sliding_window: int
    query_pre_attn_scalar: float
    rms_norm_eps: float = 1e-6
    rope_theta_local: float = 10000.0
    rope_theta_global: float = 1000000.0


@dataclass
class DecodeLayer:
    """One decoder layer's weights: OABF PackedWeights (or, for the uncompressed baseline,
    dense bf16 [N, K] tensors in their place)."""
    qkv: PackedWeight                     # q | k | v rows
    o: PackedWeight
    gate_up: PackedWeight                 # gate | up rows
    down: PackedWeight
    input_ln: torch.Tensor                # bf16 RMSNorm weights (applied as 1 + w)
    post_attn_ln: torch.Tensor
    pre_ffn_ln: torch.Tensor
    post_ffn_ln: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor


def _dims(w) -> tuple:
    """(rows, columns) of a layer weight: a PackedWeight, or a dense bf16 [N, K] tensor (the
    uncompressed baseline decoder)."""
    if isinstance(w, PackedWeight):
        return w.n_out, w.k_in
    return int(w.shape[0]), int(w.shape[1])


def rope_tables(theta: float, head_dim: int, max_ctx: int, device) -> tuple:
    """bf16 cos/sin rows for positions 0..max_ctx-1, computed as the Hugging Face Gemma-3 rotary
    embedding computes them (fp32 inverse frequencies, fp32 angles, cos/sin, then bf16)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.float32) / head_dim))
    pos = torch.arange(max_ctx, dtype=torch.float32, device=device)
    freqs = pos[:, None] * inv.to(device)[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(torch.bfloat16).contiguous(), emb.sin().to(torch.bfloat16).contiguous()


class GemmaDecoder:
    """One rank's decoder. Without ``reducer`` the layers hold whole matrices. With ``reducer``
    (an ``NVLinkAllReduce`` over the tensor-parallel ranks) they hold this rank's parts as
    ``tp.DecoderPlan`` splits them: q|k|v rows of its heads, o_proj input columns of its heads,
    gate|up rows and down_proj input columns of its intermediate range; ``lm_head`` holds its
    vocabulary rows starting at ``vocab_offset``. The row-parallel sums run inside the o_proj
    and down_proj GEMVs, the residual stream and norms are replicated (identical bits on every
    rank), and the greedy pick gathers each rank's (max logit, index) through the same
    reducer."""

    def __init__(self, shape: DecoderShape, layers: List[DecodeLayer], embed: torch.Tensor,
                 final_norm: torch.Tensor, lm_head: torch.Tensor, max_ctx: int, device=None,
                 max_prefill: int = 128, reducer=None, vocab_offset: int = 0, batch: int = 1):
        self.L = _lib.lib()
        self.shape, self.layers = shape, layers
        dev = torch.device(device) if device is not None else embed.device
        self.device = dev
        s = shape
        self.reducer = reducer
        self.world = reducer.world if reducer is not None else 1
        self.rank = reducer.rank if reducer is not None else 0
        if len(layers) != len(s.layer_types):
            raise ValueError(f"{len(layers)} layers but {len(s.layer_types)} layer types")
        if s.head_dim % 16 or s.head_dim > 256 or max_ctx + 8 * s.head_dim > 10000:
            raise ValueError("head_dim must be a multiple of 16 up to 256, and max_ctx + 8 * head_dim "
                             "at most 10000")
        if s.n_heads % self.world or s.n_kv_heads % self.world:
            raise ValueError(f"heads ({s.n_heads} / {s.n_kv_heads}) do not split over {self.world} ranks")
        self.hq, self.hkv = s.n_heads // self.world, s.n_kv_heads // self.world
        self.inter_l = _dims(layers[0].gate_up)[0] // 2 if layers else s.inter
        q_rows = (self.hq + 2 * self.hkv) * s.head_dim
        for i, ly in enumerate(layers):
            # the fused rows must hold the heads back to back (each part's rows a multiple of 64)
            (nq, _), (ngu, _), (no, ko), (nd, kd) = (_dims(ly.qkv), _dims(ly.gate_up), _dims(ly.o),
                                                     _dims(ly.down))
            if nq != q_rows or ngu != 2 * self.inter_l or no != s.hidden or nd != s.hidden \
                    or ko != self.hq * s.head_dim or kd != self.inter_l:
                raise ValueError(f"layer {i}: row / column counts do not match the shape on "
                                 f"{self.world} rank(s) (q|k|v {nq} vs {q_rows}, gate|up {ngu} vs "
                                 f"{2 * self.inter_l}, o in {ko}, down in {kd})")
        if self.world == 1 and self.inter_l != s.inter:
            raise ValueError(f"gate|up holds {2 * self.inter_l} rows, not {2 * s.inter}")
        self.max_ctx = int(max_ctx)
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.embed = embed.to(**bf).contiguous()
        self.final_norm = final_norm.to(**bf).contiguous()
        self.lm_head = lm_head.to(**bf).contiguous()
        self.vocab_offset = int(vocab_offset)
        self.vocab_l = self.lm_head.shape[0]
        self.embed_scale = float(s.hidden) ** 0.5
        self.scaling = float(s.query_pre_attn_scalar) ** -0.5
        self.rope = {
            "sliding_attention": rope_tables(s.rope_theta_local, s.head_dim, self.max_ctx, dev),
            "full_attention": rope_tables(s.rope_theta_global, s.head_dim, self.max_ctx, dev),
        }
        B = self.batch = int(batch)
        if not 1 <= B <= 64:
            raise ValueError(f"batch {B} outside [1, 64]")
        cache = (len(layers), B, self.hkv, self.max_ctx, s.head_dim)      # per layer and sequence
        self.k_cache = torch.zeros(cache, **bf)
        self.v_cache = torch.zeros(cache, **bf)
        self.seq_stride = self.hkv * self.max_ctx * s.head_dim
        self.max_rows = max(1, int(max_prefill))             # rows of a prompt chunk
        R = max(self.max_rows, B)
        self.h = torch.zeros(R, s.hidden, **bf)              # residual stream
        self.x = torch.zeros(R, s.hidden, **bf)              # normalised input of the next linear
        self.qkv = torch.zeros(R, q_rows, **bf)
        self.q = torch.zeros(R, self.hq * s.head_dim, **bf)
        self.attn = torch.zeros(R, self.hq * s.head_dim, **bf)
        self.o = torch.zeros(R, s.hidden, **bf)
        self.gu = torch.zeros(R, 2 * self.inter_l, **bf)
        self.act = torch.zeros(R, self.inter_l, **bf)
        self.down = torch.zeros(R, s.hidden, **bf)
        self.logits = torch.zeros(B, self.vocab_l, **bf)     # per sequence: this rank's vocabulary rows
        if reducer is not None:
            from .linear import fused_shard_eligible
            if reducer.max_elems < max(R * s.hidden, 2 * self.world * B):
                raise ValueError(f"the reducer holds {reducer.max_elems} values; a prompt chunk of "
                                 f"{R} rows needs {R * s.hidden}")
            self.fused_rows = all(fused_shard_eligible(pw, reducer.max_elems)
                                  for ly in layers for pw in (ly.o, ly.down))
            self.pick = torch.zeros(B, 2 * self.world, dtype=torch.float32, device=dev)
            self.row_f32 = torch.zeros(R, s.hidden, dtype=torch.float32, device=dev)
        self.ids = torch.zeros(R, dtype=torch.int64, device=dev)    # a prompt chunk's ids
        self.tok = torch.zeros(B, dtype=torch.int64, device=dev)    # per sequence: current / next token
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)    # per sequence: its position
        self.attn_scratch = torch.zeros(
            self.L.fbfp_decode_attention_step_scratch_bytes(B, self.hq, s.head_dim, self.max_ctx),
            dtype=torch.uint8, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.stream = torch.cuda.Stream(dev)

    # -- construction from a Hugging Face Gemma-3 model after compress_gemma_model -----------
    @classmethod
    def from_hf(cls, model, max_ctx: int, device=None, max_prefill: int = 128,
                reducer=None, batch: int = 1) -> "GemmaDecoder":
        """The decoder of a Gemma-3 causal LM after ``compress_gemma_model``; with ``reducer``,
        of a model compressed with ``compress_gemma_model(..., rank=r, world=reducer.world)``
        on every rank (this rank's shards; lm_head rows split here)."""
        cfg = model.config
        if getattr(cfg, "final_logit_softcapping", None) or getattr(cfg, "attn_logit_softcapping", None):
            raise NotImplementedError("logit soft-capping is not supported")
        rope = cfg.rope_parameters
        shape = DecoderShape(
            hidden=cfg.hidden_size, inter=cfg.intermediate_size, n_heads=cfg.num_attention_heads,
            n_kv_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim, vocab=cfg.vocab_size,
            layer_types=list(cfg.layer_types), sliding_window=int(cfg.sliding_window),
            query_pre_attn_scalar=float(cfg.query_pre_attn_scalar), rms_norm_eps=float(cfg.rms_norm_eps),
            rope_theta_local=float(rope["sliding_attention"]["rope_theta"]),
            rope_theta_global=float(rope["full_attention"]["rope_theta"]))
        inner = model.model
        from .linear import OABFLinear
        for i, lyr in enumerate(inner.layers):
            mods = (lyr.self_attn.q_proj, lyr.self_attn.k_proj, lyr.self_attn.v_proj, lyr.self_attn.o_proj,
                    lyr.mlp.gate_proj, lyr.mlp.up_proj, lyr.mlp.down_proj)
            if not all(isinstance(m, OABFLinear) and m.compressed for m in mods):
                raise TypeError(f"layer {i} is not compressed: run compress_gemma_model first")
        dev = torch.device(device) if device is not None else inner.embed_tokens.weight.device
        layers = []
        with torch.cuda.device(dev):
            for lyr in inner.layers:
                at, mlp = lyr.self_attn, lyr.mlp
                layers.append(DecodeLayer(
                    qkv=concat_rows([at.q_proj.packed, at.k_proj.packed, at.v_proj.packed]),
                    o=at.o_proj.packed,
                    gate_up=concat_rows([mlp.gate_proj.packed, mlp.up_proj.packed]),
                    down=mlp.down_proj.packed,
                    input_ln=lyr.input_layernorm.weight.data, post_attn_ln=lyr.post_attention_layernorm.weight.data,
                    pre_ffn_ln=lyr.pre_feedforward_layernorm.weight.data,
                    post_ffn_ln=lyr.post_feedforward_layernorm.weight.data,
                    q_norm=at.q_norm.weight.data, k_norm=at.k_norm.weight.data))
        for ly in layers:
            for f in ("input_ln", "post_attn_ln", "pre_ffn_ln", "post_ffn_ln", "q_norm", "k_norm"):
                setattr(ly, f, getattr(ly, f).to(device=dev, dtype=torch.bfloat16).contiguous())
        lm_head, v0 = model.lm_head.weight.data, 0
        if reducer is not None:
            from .tp import DecoderPlan
            plan = DecoderPlan.from_config(cfg, reducer.rank, reducer.world)
            for i, lyr in enumerate(inner.layers):
                if getattr(lyr.self_attn.o_proj, "tp_range", None) != plan.q_rows or \
                        getattr(lyr.mlp.down_proj, "tp_range", None) != plan.inter:
                    raise ValueError(f"layer {i} was not compressed for rank {reducer.rank} of "
                                     f"{reducer.world} (compress_gemma_model(..., rank, world))")
            v0, v1 = plan.vocab
            lm_head = lm_head[v0:v1]
        elif any(hasattr(m, "tp_mode") for m in model.modules()):
            raise ValueError("the model holds tensor-parallel shards: pass the reducer")
        return cls(shape, layers, inner.embed_tokens.weight.data, inner.norm.weight.data,
                   lm_head, max_ctx, dev, max_prefill, reducer=reducer, vocab_offset=v0, batch=batch)

    # -- one token ---------------------------------------------------------------------------
    def _linear(self, x: torch.Tensor, pw, out: torch.Tensor) -> None:
        if isinstance(pw, PackedWeight):
            packed_linear(x, pw, None, torch.bfloat16, out=out)
        else:                                                 # a dense bf16 weight (baseline)
            torch.matmul(x, pw.t(), out=out)

    def _row_linear(self, x: torch.Tensor, pw, out: torch.Tensor) -> None:
        """o_proj / down_proj: on several ranks the sum of the ranks' partial products, fused
        into the GEMV for decode-sized chunks, else a separate peer-memory all-reduce."""
        if self.reducer is None:
            self._linear(x, pw, out)
            return
        m = x.shape[0]
        if self.fused_rows and m <= 64:
            packed_linear_allreduce(x, pw, self.reducer, None, torch.bfloat16, out=out)
        else:
            y = self.row_f32[:m]
            packed_linear(x, pw, None, torch.float32, out=y)
            self.reducer(y)
            out.copy_(y)

    def _pick(self, logits: torch.Tensor, tok: torch.Tensor, slots) -> None:
        """Greedy tokens of `logits` rows into `tok`: argmax over this rank's vocabulary rows,
        then (several ranks) every rank's (max, index) gathered through the reducer (a sum of
        one-hot slots is exact) and the first maximum taken."""
        if self.reducer is None:
            tok.copy_(torch.argmax(logits, dim=-1))
            return
        from .tp import argmax_pick, argmax_slots
        slots.zero_()
        argmax_slots(logits, self.vocab_offset, self.rank, self.world, slots)
        self.reducer(slots)
        tok.copy_(argmax_pick(slots, self.world))

    def _layers(self, m: int, chunk_seq: Optional[int]) -> None:
        """Every layer over rows 0..m-1 of the activation buffers: with chunk_seq = b, a prompt
        chunk of sequence b at positions pos[b] .. pos[b] + m - 1 (causal over the chunk);
        with chunk_seq = None, one new token per sequence (m = batch)."""
        L, s, st = self.L, self.shape, _lib.stream_ptr(self.device)
        P = _lib.ptr
        eps = float(s.rms_norm_eps)
        h, x, qkv, q, attn = self.h[:m], self.x[:m], self.qkv[:m], self.q[:m], self.attn[:m]
        o, gu, act, down = self.o[:m], self.gu[:m], self.act[:m], self.down[:m]
        for li, ly in enumerate(self.layers):
            kind = s.layer_types[li]
            cos_t, sin_t = self.rope[kind]
            window = s.sliding_window if kind == "sliding_attention" else 0
            self._linear(x, ly.qkv, qkv)
            if chunk_seq is None:
                _lib.check(L.fbfp_decode_attention_step(
                    P(qkv), m, self.hq, self.hkv, s.head_dim, P(ly.q_norm), P(ly.k_norm), eps, P(cos_t),
                    P(sin_t), P(self.pos), self.max_ctx, P(self.k_cache[li]), P(self.v_cache[li]),
                    self.seq_stride, window, self.scaling, P(self.attn_scratch), P(attn), P(self.err), st),
                    "fbfp_decode_attention_step")
            else:
                b = chunk_seq
                kc, vc, pos = self.k_cache[li, b], self.v_cache[li, b], self.pos[b:b + 1]
                _lib.check(L.fbfp_qk_rope_cache(P(qkv), m, self.hq, self.hkv, s.head_dim, P(ly.q_norm),
                                                P(ly.k_norm), eps, P(cos_t), P(sin_t), P(pos), self.max_ctx,
                                                P(q), P(kc), P(vc), P(self.err), st), "fbfp_qk_rope_cache")
                _lib.check(L.fbfp_decode_attention(P(q), m, P(kc), P(vc), self.hq, self.hkv, s.head_dim,
                                                   self.max_ctx, P(pos), window, self.scaling, P(attn), st),
                           "fbfp_decode_attention")
            self._row_linear(attn, ly.o, o)
            _lib.check(L.fbfp_post_residual_norm(P(o), m, P(ly.post_attn_ln), P(h), P(ly.pre_ffn_ln), eps,
                                                 s.hidden, P(x), st), "fbfp_post_residual_norm")
            self._linear(x, ly.gate_up, gu)
            _lib.check(L.fbfp_geglu(P(gu), m, self.inter_l, P(act), st), "fbfp_geglu")
            self._row_linear(act, ly.down, down)
            nxt = self.layers[li + 1].input_ln if li + 1 < len(self.layers) else self.final_norm
            _lib.check(L.fbfp_post_residual_norm(P(down), m, P(ly.post_ffn_ln), P(h), P(nxt), eps,
                                                 s.hidden, P(x), st), "fbfp_post_residual_norm")

    def _embed(self, ids: torch.Tensor, m: int) -> None:
        L, s, st = self.L, self.shape, _lib.stream_ptr(self.device)
        P = _lib.ptr
        _lib.check(L.fbfp_embed(P(ids), m, P(self.embed), s.vocab, s.hidden, self.embed_scale, P(self.h),
                                P(self.err), st), "fbfp_embed")
        _lib.check(L.fbfp_rmsnorm(P(self.h), m, P(self.layers[0].input_ln), float(s.rms_norm_eps), s.hidden,
                                  P(self.x), st), "fbfp_rmsnorm")

    def _enqueue(self, m: int, seq: int = 0) -> None:
        """A prompt chunk of m tokens (self.ids[:m]) of sequence seq: every layer, then the logits
        of the last row into self.logits[seq], the greedy pick into self.tok[seq] and pos[seq] += m."""
        self._embed(self.ids, m)
        self._layers(m, seq)
        torch.matmul(self.x[m - 1:m], self.lm_head.t(), out=self.logits[seq:seq + 1])   # bf16 lm_head
        self._pick(self.logits[seq:seq + 1], self.tok[seq:seq + 1],
                   self.pick[seq:seq + 1] if self.reducer is not None else None)
        _lib.check(self.L.fbfp_advance_position(_lib.ptr(self.pos[seq:seq + 1]), m, _lib.stream_ptr(self.device)),
                   "fbfp_advance_position")

    def _enqueue_step(self) -> None:
        """One new token for every sequence: tokens self.tok at positions self.pos; leaves the
        logits in self.logits, the greedy next tokens in self.tok and advances every position."""
        B = self.batch
        self._embed(self.tok, B)
        self._layers(B, None)
        torch.matmul(self.x[:B], self.lm_head.t(), out=self.logits)          # bf16 lm_head (cuBLAS)
        self._pick(self.logits, self.tok, self.pick if self.reducer is not None else None)
        _lib.check(self.L.fbfp_advance_positions(_lib.ptr(self.pos), B, _lib.stream_ptr(self.device)),
                   "fbfp_advance_positions")

    def prefill(self, ids: Sequence[int], seq: int = 0) -> None:
        """Run a prompt chunk of sequence ``seq`` at positions pos[seq] .. (at most max_prefill
        tokens): fills its KV cache, leaves the last row's logits in self.logits[seq], the greedy
        next token in self.tok[seq], and advances pos[seq] by len(ids)."""
        m = len(ids)
        if not 1 <= m <= self.max_rows:
            raise ValueError(f"a prompt chunk holds 1..{self.max_rows} tokens (got {m})")
        if not 0 <= seq < self.batch:
            raise ValueError(f"sequence {seq} outside the batch of {self.batch}")
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            self.ids[:m].copy_(torch.as_tensor(list(ids), dtype=torch.int64), non_blocking=False)
            self._enqueue(m, seq)

    def reset(self, pos=0) -> None:
        """Set the positions (an int for every sequence, or one per sequence) and clear the error
        word, in order with the decoder's stream."""
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            if isinstance(pos, int):
                self.pos.fill_(pos)
            else:
                self.pos.copy_(torch.as_tensor(list(pos), dtype=torch.int32), non_blocking=False)
            self.err.zero_()

    def capture(self) -> None:
        """Record one token step as a CUDA graph (after one eager step that sets the kernels up;
        the positions are restored, and the cache rows that step wrote are rewritten later)."""
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            saved_tok, saved_pos = self.tok.clone(), self.pos.clone()
            self._enqueue_step()
            self.tok.copy_(saved_tok)
            self.pos.copy_(saved_pos)
            self.stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                self._enqueue_step()
        self.graph = g

    def step(self) -> None:
        """One token per sequence: embeds self.tok[b] at position self.pos[b], leaves the greedy
        next tokens in self.tok and the logits in self.logits, and advances every position."""
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            if self.graph is not None:
                self.graph.replay()
            else:
                self._enqueue_step()

    def check(self) -> None:
        """Raise if a kernel met an out-of-range token (1) or position (2)."""
        self.stream.synchronize()
        e = int(self.err.item())
        if e:
            self.reset(self.pos.tolist())          # clears the error word on the decoder's stream
            raise RuntimeError({1: "token id outside the vocabulary",
                                2: f"position outside the KV cache ({self.max_ctx})"}.get(e, f"error {e}"))

    def generate(self, prompt, n_new: int):
        """Greedy continuation: ``prompt`` is one list of ids (batch 1; returns a list) or one
        list per sequence of the batch (returns a list of lists). Prompts are prefilled in chunks
        of max_prefill tokens, then all sequences decode together, one token each per step."""
        single = len(prompt) == 0 or not isinstance(prompt[0], (list, tuple))
        prompts = [list(prompt)] if single else [list(p) for p in prompt]
        if len(prompts) != self.batch:
            raise ValueError(f"{len(prompts)} prompts for a batch of {self.batch}")
        if max(len(p) for p in prompts) + n_new > self.max_ctx or min(len(p) for p in prompts) < 1:
            raise ValueError("prompt + new tokens exceed the KV cache (or a prompt is empty)")
        self.reset(0)
        for b, p in enumerate(prompts):
            for i in range(0, len(p), self.max_rows):
                self.prefill(p[i:i + self.max_rows], seq=b)
        out = [[] for _ in prompts]
        for _ in range(n_new):
            self.stream.synchronize()
            for b, t in enumerate(self.tok.tolist()):
                out[b].append(int(t))
            self.step()
        self.check()
        return out[0] if single else out

    def release(self) -> None:
        if self.graph is not None:
            self.graph.reset()
            self.graph = None
