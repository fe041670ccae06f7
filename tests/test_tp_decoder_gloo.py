"""Whole-decoder tensor parallelism on CPU ranks (gloo): the split of ``tp.DecoderPlan`` and the
collective algebra of ``GemmaDecoder`` with a reducer, on a small Gemma-3-style decoder in fp64.

Every rank keeps its query / KV heads (their q|k|v rows, KV cache and o_proj input columns), its
intermediate range (gate and up rows, down_proj input columns) and its vocabulary rows of
lm_head; o_proj and down_proj partial outputs are summed over the ranks, the residual stream and
norms are replicated, and the greedy pick gathers each rank's (max logit, index) by summing
one-hot slots (``tp.argmax_slots`` / ``tp.argmax_pick``, the functions the decoder runs on the
GPU). The sharded forward must reproduce the unsharded one: logits to 1e-12, the same token.
"""
import math
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

H, NH, NKV, HD, INTER, VOCAB, LAYERS, T = 128, 8, 4, 16, 1024, 320, 2, 6


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights():
    g = torch.Generator().manual_seed(3)

    def r(*shape, scale=0.05):
        return torch.randn(*shape, generator=g, dtype=torch.float64) * scale

    layers = []
    for _ in range(LAYERS):
        layers.append({"q_proj": r(NH * HD, H), "k_proj": r(NKV * HD, H), "v_proj": r(NKV * HD, H),
                       "o_proj": r(H, NH * HD), "gate_proj": r(INTER, H), "up_proj": r(INTER, H),
                       "down_proj": r(H, INTER), "ln": r(4, H, scale=0.1), "qn": r(HD, scale=0.1),
                       "kn": r(HD, scale=0.1)})
    return {"embed": r(VOCAB, H, scale=1.0), "final": r(H, scale=0.1), "lm_head": r(VOCAB, H),
            "layers": layers}


def _rms(x, w, eps=1e-6):
    return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps) * (1.0 + w)


def _rope(x, pos):
    inv = 1.0 / (10000.0 ** (torch.arange(0, HD, 2, dtype=torch.float64) / HD))
    ang = pos[:, None].double() * inv[None, :]
    cos, sin = torch.cat([ang.cos()] * 2, -1), torch.cat([ang.sin()] * 2, -1)
    half = torch.cat([-x[..., HD // 2:], x[..., :HD // 2]], -1)
    return x * cos[:, None, :] + half * sin[:, None, :]


def _forward(Wt, ids, slice_fn, hq, hkv, reduce_fn):
    """Causal forward of the prompt `ids`; returns (logits of the last position over the rows
    lm_head holds, final hidden state). slice_fn(W, name) gives the part of W a rank holds."""
    pos = torch.arange(len(ids))
    h = Wt["embed"][ids] * math.sqrt(H)
    for ly in Wt["layers"]:
        x = _rms(h, ly["ln"][0])
        q = (x @ slice_fn(ly["q_proj"], "q_proj").T).view(T, hq, HD)
        k = (x @ slice_fn(ly["k_proj"], "k_proj").T).view(T, hkv, HD)
        v = (x @ slice_fn(ly["v_proj"], "v_proj").T).view(T, hkv, HD)
        q, k = _rope(_rms(q, ly["qn"]), pos), _rope(_rms(k, ly["kn"]), pos)
        rep = hq // hkv
        k, v = k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)
        s = torch.einsum("thd,shd->hts", q, k) / math.sqrt(HD)
        s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1)[None], float("-inf"))
        a = torch.einsum("hts,shd->thd", torch.softmax(s, -1), v).reshape(T, hq * HD)
        o = reduce_fn(a @ slice_fn(ly["o_proj"], "o_proj").T)
        h = h + _rms(o, ly["ln"][1])
        x = _rms(h, ly["ln"][2])
        gate = x @ slice_fn(ly["gate_proj"], "gate_proj").T
        up = x @ slice_fn(ly["up_proj"], "up_proj").T
        act = torch.nn.functional.gelu(gate, approximate="tanh") * up
        d = reduce_fn(act @ slice_fn(ly["down_proj"], "down_proj").T)
        h = h + _rms(d, ly["ln"][3])
    return _rms(h[-1:], Wt["final"]), h


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from flashbfp_b200 import tp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        Wt = _weights()
        ids = torch.tensor([5, 77, 300, 12, 250, 3])
        # unsharded
        xf, hf = _forward(Wt, ids, lambda W, n: W, NH, NKV, lambda y: y)
        logits_full = (xf @ Wt["lm_head"].T).reshape(-1)
        tok_full = int(torch.argmax(logits_full))
        # this rank's shards
        plan = tp.DecoderPlan(NH, NKV, HD, INTER, VOCAB, rank, world)

        def allreduce(y):
            y = y.clone()
            dist.all_reduce(y)
            return y

        x, h = _forward(Wt, ids, plan.slice, plan.hq, plan.hkv, allreduce)
        torch.testing.assert_close(h, hf, rtol=1e-12, atol=1e-12)        # replicated stream
        v0, v1 = plan.vocab
        logits = (x @ Wt["lm_head"][v0:v1].T).reshape(-1)
        torch.testing.assert_close(logits, logits_full[v0:v1], rtol=1e-12, atol=1e-12)
        slots = torch.zeros(2 * world, dtype=torch.float32)
        tp.argmax_slots(logits, v0, rank, world, slots)
        dist.all_reduce(slots)
        assert int(tp.argmax_pick(slots, world)) == tok_full
        # ties across ranks resolve to the lowest global index, as one argmax would
        tie = torch.zeros(v1 - v0)
        tie[-1] = 1.0
        slots.zero_()
        tp.argmax_slots(tie, v0, rank, world, slots)
        dist.all_reduce(slots)
        # every rank's maximum sits on its last row: the first over the vocabulary is rank 0's
        assert int(tp.argmax_pick(slots, world)) == tp.DecoderPlan(NH, NKV, HD, INTER, VOCAB, 0, world).vocab[1] - 1
        q.put((rank, "ok"))
    except Exception as e:                      # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_whole_decoder_tensor_parallel_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {r: "ok" for r in range(world)}, results


@pytest.mark.parametrize("cfg", [(16, 8, 256, 15360, 262208), (64, 8, 128, 28672, 128256)],
                         ids=["gemma3-12b", "70b-class"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_decoder_plan_covers_every_dimension(cfg, world):
    """The plan's ranges tile heads, intermediate and vocabulary exactly; the MLP range (gate and
    up rows, down_proj input columns) is in whole 256-column stages; o_proj's input columns are
    the rank's query heads."""
    from flashbfp_b200 import tp
    nh, nkv, hd, inter, vocab = cfg
    plans = [tp.DecoderPlan(nh, nkv, hd, inter, vocab, r, world) for r in range(world)]
    for attr, total in (("q_rows", nh * hd), ("kv_rows", nkv * hd), ("inter", inter), ("vocab", vocab)):
        rs = [getattr(p, attr) for p in plans]
        assert rs[0][0] == 0 and rs[-1][1] == total and all(a[1] == b[0] for a, b in zip(rs, rs[1:])), attr
    for p in plans:
        assert p.ranges("model.layers.0.self_attn.o_proj") == ("row",) + p.q_rows
        assert p.ranges("model.layers.0.mlp.down_proj") == ("row",) + p.inter
        assert p.ranges("gate_proj") == p.ranges("up_proj") == ("column",) + p.inter
        assert (p.inter[1] - p.inter[0]) % tp.ROW_K_ALIGN == 0
        assert (p.q_rows[1] - p.q_rows[0]) % 256 == 0 or hd * p.hq < 256
    with pytest.raises(ValueError):
        tp.DecoderPlan(16, 8, 256, 15360, 262208, 0, 16)          # 8 KV heads over 16 ranks
