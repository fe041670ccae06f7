"""fbfp_allreduce_* (one-shot fp32 all-reduce over NVLink peer memory) on 2 GPUs.

Needs at least two GPUs (skipped otherwise); one process per GPU, the IPC handles exchanged
through a gloo process group. The sum is taken in rank order, so the result equals
y0 + y1 computed in fp32 exactly, on both ranks."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data(rank, call, n):
    g = torch.Generator().manual_seed(1000 * call + rank)
    return torch.randn(n, generator=g)


def _worker(rank, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        from flashbfp_b200 import build
        build.build()
        from flashbfp_b200.tp import NVLinkAllReduce
        dev = torch.device("cuda", rank)
        ar = NVLinkAllReduce(16 * 3840)
        # consecutive calls, vectorised (n % 4 == 0) and scalar (n % 4 != 0) paths
        for call, n in enumerate([3840, 3840, 61440, 1001, 3840, 7]):
            y = _data(rank, call, n).to(dev)
            ar(y)
            exp = _data(0, call, n) + _data(1, call, n)
            assert torch.equal(y.cpu(), exp), (call, n)
        ar.check(dev)
        # captured in a CUDA graph: the call counter lives on the device, so replays advance it
        y = torch.zeros(3840, device=dev)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            ar(y)                                  # warm-up call outside the capture
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            ar(y)
        for rep in range(3):
            y.copy_(_data(rank, 100 + rep, 3840).to(dev))
            g.replay()
            torch.cuda.synchronize(dev)
            exp = _data(0, 100 + rep, 3840) + _data(1, 100 + rep, 3840)
            assert torch.equal(y.cpu(), exp), rep
        ar.check(dev)
        g.reset()
        dist.barrier()
        ar.close()
        q.put((rank, "ok"))
    except Exception as e:                          # reported to the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_nvlink_allreduce_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res


def _fused_worker(rank, port, q):
    """fbfp_gemv_allreduce on the row-parallel shards of o_proj and down_proj at TP 2: equal to
    the separate path (fp32 GEMV partials, the NVLink all-reduce, then the bias) up to the order
    of the GEMV's own fp32 partial sums (row groups split across CTAs add into the workspace in
    arrival order, so the tolerance is 1e-5 relative), identical bits on both ranks; mixed with
    standalone all-reduce calls and replayed from a graph."""
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        from flashbfp_b200 import build
        build.build()
        from flashbfp_b200 import OABFCompressor, packed, tp, workloads
        from flashbfp_b200.linear import (check_device_errors, gemv_records, gemv_workspace,
                                          packed_linear, packed_linear_allreduce)
        from flashbfp_b200.tp import NVLinkAllReduce, TPLinear
        dev = torch.device("cuda", rank)
        ar = NVLinkAllReduce(40 * 3840)              # the separate path's 40-token reference
        comp = OABFCompressor()

        def separate(Xs, pw, bias):
            y = packed_linear(Xs, pw, None, torch.float32)
            ar(y)
            return y + bias.float() if bias is not None else y

        def rel(a, b):
            return ((a.float() - b.float()).norm() / b.float().norm()).item()

        def same_on_ranks(t):
            got = [torch.empty_like(t.cpu()) for _ in range(WORLD)]
            dist.all_gather(got, t.cpu().contiguous())
            return all(torch.equal(got[0], g) for g in got)

        for name in ("o_proj", "down_proj"):
            n, k = workloads.GEMMA12B_LAYER[name]
            W = workloads.decode_weight(n, k, seed=n + k, device=dev)      # same W on both ranks
            dp, sp = tp.compress_shard(W, name, rank, WORLD, comp)
            pw = packed.from_compressed(dp, sp, dev)
            k0, k1 = tp.input_range(name, k, rank, WORLD)
            bias = (0.1 * torch.randn(n, generator=torch.Generator().manual_seed(5))).to(dev, torch.bfloat16)
            pwr = packed.from_compressed(dp, sp, dev).build_records()
            ws = gemv_workspace(dev, pwr.npad)
            for m in (1, 5, 16):
                X = workloads.activations(m, k, seed=m, device=dev)
                Xs = X[:, k0:k1]
                ref = separate(Xs, pw, bias)
                Yf = packed_linear_allreduce(Xs, pw, ar, bias, torch.float32)
                Yb = packed_linear_allreduce(Xs, pw, ar, bias, torch.bfloat16)
                check_device_errors(dev)
                assert rel(Yf, ref) <= 1e-5, (name, m, rel(Yf, ref))
                assert rel(Yb, ref) <= 5e-3, (name, m, rel(Yb, ref))      # bf16 rounding of y
                assert same_on_ranks(Yf) and same_on_ranks(Yb), (name, m)
                # the stage-record GEMV with the same exchange fused in (one token on the CUDA
                # cores and on the tensor cores; more on the tensor cores)
                for tc in ((False, True) if m == 1 else (True,)):
                    Yr = torch.empty(m, n, dtype=torch.float32, device=dev)
                    gemv_records(Xs, pwr, Yr, ws, bias, reducer=ar, tensor_cores=tc)
                    check_device_errors(dev)
                    assert rel(Yr, ref) <= 1e-5, (name, m, tc, rel(Yr, ref))
                    assert same_on_ranks(Yr), (name, m, tc)
            # the module path: 40 tokens = three fused launches (16 + 16 + 8)
            lin = TPLinear(pw, name, rank, WORLD, k, bias=bias, reducer=ar)
            X = workloads.activations(40, k, seed=40, device=dev)
            Y = lin(X)
            check_device_errors(dev)
            assert Y.dtype == torch.bfloat16 and same_on_ranks(Y), name
            assert rel(Y, separate(X[:, k0:k1], pw, bias)) <= 5e-3, name
        ar.check(dev)

        # graph: fused GEMV, standalone all-reduce, fused GEMV again (one shared call counter)
        n, k = workloads.GEMMA12B_LAYER["o_proj"]
        W = workloads.decode_weight(n, k, seed=11, device=dev)
        dp, sp = tp.compress_shard(W, "o_proj", rank, WORLD, comp)
        pw = packed.from_compressed(dp, sp, dev)
        k0, k1 = tp.input_range("o_proj", k, rank, WORLD)
        X = torch.zeros(1, k, dtype=torch.bfloat16, device=dev)
        Y1 = torch.empty(1, n, dtype=torch.float32, device=dev)
        Y2 = torch.empty(1, n, dtype=torch.float32, device=dev)
        z = torch.zeros(3840, device=dev)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))

        def body():
            packed_linear_allreduce(X[:, k0:k1], pw, ar, None, torch.float32, out=Y1)
            ar(z)
            packed_linear_allreduce(X[:, k0:k1], pw, ar, None, torch.float32, out=Y2)

        with torch.cuda.stream(s):
            body()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            body()
        for rep in range(3):
            X.copy_(workloads.activations(1, k, seed=200 + rep, device=dev))
            z.copy_(_data(rank, 300 + rep, 3840).to(dev))
            g.replay()
            torch.cuda.synchronize(dev)
            check_device_errors(dev)
            ref = separate(X[:, k0:k1], pw, None)
            assert rel(Y1, ref) <= 1e-5 and rel(Y2, ref) <= 1e-5, rep
            assert same_on_ranks(Y1) and same_on_ranks(Y2), rep
            assert torch.equal(z.cpu(), _data(0, 300 + rep, 3840) + _data(1, 300 + rep, 3840)), rep
        ar.check(dev)
        g.reset()
        dist.barrier()
        ar.close()
        q.put((rank, "ok"))
    except Exception as e:                          # reported to the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_fused_gemv_allreduce_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_fused_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=400) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res
