"""Failure detection on the GPU: a rank that joins and then never makes its call.

Rank 1 creates its all-reduce handle (rank 0 maps rank 1's buffer) and then never calls. Rank 0's
all-reduce and its fused GEMV exchanges (reference-layout tensor-core GEMV; stage-record GEMV on
the CUDA cores and on the tensor cores) wait for words that nothing writes. Each wait is bounded
by the handle's timeout (50 ms here): the kernel records the rank it gave up on and returns, the
host check raises FBFP_ERR_TIMEOUT naming rank 1 within a second, the error is cleared by the
check, and the context stays usable (a later GEMV on the same workspace is correct).

Replaces the reference's failure handling, a silent CPU fallback on any GPU error
(flash_bfp/triton_kernel.py:139-165). Runs on two GPUs when present (with one successful call
first), else with both ranks' processes on one GPU; there only rank 0 launches kernels, so no two
kernels wait on one another. NVLS is off (the handle uses plain peer stores anyway)."""
import os
import socket
import time
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2
TIMEOUT_S = 0.05


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _expect_timeout(fn, what):
    from flashbfp_b200._lib import FlashBFPError
    t0 = time.time()
    try:
        fn()
    except FlashBFPError as e:
        msg = str(e)
        assert "timed out" in msg and "rank 1" in msg, (what, msg)
        assert time.time() - t0 < 5.0, (what, time.time() - t0)
        return msg
    raise AssertionError(f"{what}: no timeout reported")


def _worker(rank, port, q, two_gpus):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank if two_gpus else 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        from flashbfp_b200 import build
        build.build()
        from flashbfp_b200 import OABFCompressor, packed, tp, workloads
        from flashbfp_b200.linear import (check_device_errors, gemv_records, gemv_workspace,
                                          packed_linear, packed_linear_allreduce)
        from flashbfp_b200.tp import NVLinkAllReduce
        from oracle import oabf
        import numpy as np

        def fresh():
            ar = NVLinkAllReduce(16 * 4096)
            ar.set_timeout(TIMEOUT_S)
            return ar

        # 1. the standalone all-reduce
        ar = fresh()
        if two_gpus:                       # both ranks call once: the handle works
            y = torch.full((3840,), 1.0 + rank, device=dev)
            ar(y)
            ar.check(dev)
            assert bool((y == 3.0).all())
        if rank == 0:
            y = torch.ones(3840, device=dev)
            ar(y)
            _expect_timeout(lambda: ar.check(dev), "all-reduce")
            ar.check(dev)                  # the error was reported once and cleared
        dist.barrier()                     # rank 1's buffer stays mapped until rank 0 is done
        ar.close()

        # 2. the fused exchange of the row-parallel GEMVs (o_proj shard, K split over 2 ranks)
        n, k = workloads.GEMMA12B_LAYER["o_proj"]
        W = workloads.decode_weight(n, k, seed=31, device=dev)
        dp, sp = tp.compress_shard(W, "o_proj", rank, WORLD, OABFCompressor())
        pw = packed.from_compressed(dp, sp, dev).build_records()
        k0, k1 = tp.input_range("o_proj", k, rank, WORLD)
        X = workloads.activations(4, k, seed=7, device=dev)[:, k0:k1].contiguous()
        ws = gemv_workspace(dev, pw.npad)
        variants = {
            "gemv": lambda ar: packed_linear_allreduce(X[:1], pw, ar, None, torch.float32),
            "records-cuda-cores": lambda ar: gemv_records(
                X[:1], pw, torch.empty(1, n, device=dev), ws, reducer=ar),
            "records-tensor-cores": lambda ar: gemv_records(
                X, pw, torch.empty(4, n, device=dev), ws, reducer=ar),
        }
        for what, call in variants.items():
            ar = fresh()
            if rank == 0:
                call(ar)
                _expect_timeout(lambda: check_device_errors(dev), what)
                check_device_errors(dev)
            dist.barrier()
            ar.close()

        # 3. the context and the workspace are usable: rank 0's local partial product is right
        if rank == 0:
            Y = packed_linear(X, pw, None, torch.float32)
            check_device_errors(dev)
            d = {kk: (dp[kk].cpu().numpy() if torch.is_tensor(dp[kk]) else dp[kk])
                 for kk in ("exponents", "signs", "payload", "orig_shape", "padded_shape")}
            s = {kk: sp[kk].cpu().numpy() for kk in ("block_idx", "offset", "value")}
            s["count"] = int(sp["count"])
            exact = oabf.linear_reference(X.float().cpu().numpy(), d, s)
            assert oabf.rel_l2(Y.cpu().numpy(), exact) <= 1e-2
        dist.barrier()
        q.put((rank, "ok"))
    except Exception as e:                 # reported to the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("two_gpus", [False, True], ids=["one-gpu", "two-gpus"])
def test_silent_rank_times_out(two_gpus):
    if two_gpus and torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, q, two_gpus)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res
