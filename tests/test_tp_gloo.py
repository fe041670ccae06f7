"""Tensor-parallel host logic on 2 CPU ranks (gloo): shard plans, whole-matrix-threshold shards
whose bytes equal the slice of the whole compression, and the exchange that recombines them.

The per-rank products are computed with the oracle's dequantize-then-matmul (fp64), standing in
for the GPU kernels, so what is tested is the sharding and the collective algebra:
column-parallel outputs concatenate (all_gather) and row-parallel partial outputs sum
(all_reduce) to the unsharded result.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oabf

N, K = 256, 320           # 2 ranks: 128-row shards; K in whole 256-column stages: 256 + 64 columns


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights():
    rng = np.random.default_rng(7)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    pos = rng.choice(N * K, size=N * K // 60, replace=False)
    W.reshape(-1)[pos] = (rng.standard_t(3, size=pos.size) * 20 * 0.02).astype(np.float32)
    X = rng.standard_normal((5, K)).astype(np.float32)
    return W, X


def _packed_cpu(dp, sp):
    from flashbfp_b200 import packed
    dpt = {"exponents": torch.from_numpy(dp["exponents"]), "signs": torch.from_numpy(dp["signs"]),
           "payload": torch.from_numpy(dp["payload"]), "orig_shape": dp["orig_shape"],
           "padded_shape": dp["padded_shape"]}
    spt = {"block_idx": torch.from_numpy(sp["block_idx"]), "offset": torch.from_numpy(sp["offset"]),
           "value": torch.from_numpy(sp["value"]), "count": sp["count"]}
    return packed.from_compressed(dpt, spt, "cpu", build_tiles=False)


def _dicts(pw):
    """PackedWeight (CPU) -> oracle dicts."""
    b, o, v = pw.coo
    dp = {"exponents": pw.exps.numpy(), "signs": pw.signs.numpy(), "payload": pw.payload.numpy(),
          "orig_shape": (pw.n_out, pw.k_in), "padded_shape": (pw.kpad, pw.npad)}
    sp = {"block_idx": b.numpy(), "offset": o.numpy(), "value": v.view(torch.float16).numpy(),
          "count": int(b.numel())}
    return dp, sp


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from flashbfp_b200 import tp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        W, X = _weights()
        thr = oabf.compute_dynamic_threshold(W, "fp32")
        full_dp, full_sp = oabf.compress_matrix(W, "fp32", threshold=thr)
        full = _packed_cpu(full_dp, full_sp)
        Y_full = oabf.linear_reference(X, full_dp, full_sp)
        for name in ("gate_proj", "down_proj"):
            Wt = torch.from_numpy(W)
            Ws = tp.weight_slice(Wt, name, rank, world).numpy()
            # the shard compressed alone with the whole matrix's threshold ...
            dp, sp = oabf.compress_matrix(Ws, "fp32", threshold=thr)
            # ... has exactly the bytes of the slice of the whole compression
            sl_dp, sl_sp = _dicts(tp.slice_packed(full, name, rank, world, tiles=False))
            for key in ("exponents", "signs", "payload"):
                np.testing.assert_array_equal(dp[key].reshape(-1), sl_dp[key].reshape(-1), err_msg=key)
            for key in ("block_idx", "offset"):
                np.testing.assert_array_equal(sp[key], sl_sp[key], err_msg=key)
            np.testing.assert_array_equal(sp["value"].view(np.int16), sl_sp["value"].view(np.int16))
            assert tuple(dp["padded_shape"]) == tuple(sl_dp["padded_shape"])
            k0, k1 = tp.input_range(name, K, rank, world)
            Y_part = oabf.linear_reference(X[:, k0:k1], dp, sp)
            if tp.mode_of(name) == "column":
                parts = [torch.zeros(5, N // world, dtype=torch.float64) for _ in range(world)]
                dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(Y_part, dtype=np.float64)))
                Y = torch.cat(parts, dim=1).numpy()
            else:
                y = torch.from_numpy(np.ascontiguousarray(Y_part, dtype=np.float64))
                tp.all_reduce_sum(y)
                Y = y.numpy()
            np.testing.assert_allclose(Y, Y_full, rtol=1e-9, atol=1e-9)
        q.put((rank, "ok"))
    except Exception as e:                      # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_split_plans_cover_exactly():
    from flashbfp_b200 import tp
    for total, world, align in [(15360, 8, 16), (4096, 8, 16), (8192, 3, 16), (100, 2, 1), (3840, 4, 16)]:
        got = [tp.split(total, r, world, align) for r in range(world)]
        assert got[0][0] == 0 and got[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
        assert all(lo % align == 0 for lo, _ in got)
    assert tp.mode_of("model.layers.3.mlp.down_proj") == "row"
    assert tp.mode_of("q_proj") == "column"
    with pytest.raises(ValueError):
        tp.mode_of("lm_head")


def test_row_parallel_shards_are_whole_stages():
    """Row-parallel shards of the 12B-class linears split K in whole 256-column stages at TP 2, 4
    and 8 (so every shard takes the tensor-core GEMV and its fused exchange), covering K exactly;
    the weight slice and the input range agree."""
    from flashbfp_b200 import tp, workloads
    for name in ("o_proj", "down_proj"):
        n, k = workloads.GEMMA12B_LAYER[name]
        W = torch.zeros(n, k)
        for world in (2, 4, 8):
            ranges = [tp.input_range(name, k, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == k
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            assert all((hi - lo) % tp.ROW_K_ALIGN == 0 and hi > lo for lo, hi in ranges), (name, world, ranges)
            sizes = [hi - lo for lo, hi in ranges]
            assert max(sizes) - min(sizes) <= tp.ROW_K_ALIGN
            for r, (lo, hi) in enumerate(ranges):
                assert tp.weight_slice(W, name, r, world).shape == (n, hi - lo)
    assert tp.input_range("q_proj", 3840, 1, 4) == (0, 3840)


def test_tensor_parallel_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results
