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
