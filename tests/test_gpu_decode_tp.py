"""Whole-model tensor parallelism of the decode token step on 2 GPUs (one process per GPU).

A tiny random-init Gemma-3 (the same seed on both ranks) is compressed per rank with
``compress_gemma_model(..., rank, world=2)`` and run by ``GemmaDecoder.from_hf(..., reducer)``:
head-parallel attention and KV cache, the MLP split over its intermediate dimension, o_proj and
down_proj summed over the ranks (fused into the GEMV where the shard's K is a whole number of
256-column stages, else through the separate peer-memory all-reduce), vocab-parallel lm_head
with the (max, index) gather. Against the single-GPU decoder of the same model, teacher-forced:
the gathered logits of every position agree within 2e-2 relative L2 (the ranks' partial sums
are added in another order and rounded to bf16 at other points), the greedy token equals the
argmax of the gathered logits and is the same on both ranks, a prompt prefilled as one chunk
continues the same way, and the CUDA graph replay reproduces the eager step.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2
T = 12


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tiny(seed, head_dim):
    import transformers
    cfg = transformers.Gemma3TextConfig(vocab_size=512, hidden_size=256, intermediate_size=512,
                                        num_hidden_layers=2, num_attention_heads=4,
                                        num_key_value_heads=2, head_dim=head_dim,
                                        max_position_embeddings=128, sliding_window=4,
                                        layer_types=["sliding_attention", "full_attention"],
                                        attn_implementation="eager")
    torch.manual_seed(seed)
    model = transformers.Gemma3ForCausalLM(cfg).eval()
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.copy_(0.2 * torch.randn_like(p))
    return model


def _worker(rank, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=120))
    try:
        from flashbfp_b200 import build
        build.build()
        from flashbfp_b200 import OABFCompressor
        from flashbfp_b200.decode import GemmaDecoder
        from flashbfp_b200.linear import check_device_errors
        from flashbfp_b200.model import compress_gemma_model
        from flashbfp_b200.tp import NVLinkAllReduce
        dev = torch.device("cuda", rank)
        ids = torch.randint(0, 512, (T,), generator=torch.Generator().manual_seed(9)).tolist()

        def gathered(local):
            parts = [None] * WORLD
            dist.all_gather_object(parts, local.cpu())
            return torch.cat(parts, dim=-1)

        def rel(a, b):
            return float((a.float() - b.float()).norm() / b.float().norm())

        for head_dim in (64, 128):               # o_proj shard K 128 (separate sum) / 256 (fused)
            single = GemmaDecoder.from_hf(
                compress_gemma_model(_tiny(1, head_dim).to(dev, torch.bfloat16), OABFCompressor()),
                max_ctx=64, max_prefill=32)
            model = compress_gemma_model(_tiny(1, head_dim).to(dev, torch.bfloat16), OABFCompressor(),
                                         rank=rank, world=WORLD)
            ar = NVLinkAllReduce(32 * 256)
            dec = GemmaDecoder.from_hf(model, max_ctx=64, max_prefill=32, reducer=ar)
            assert dec.hq == 2 and dec.hkv == 1 and dec.k_cache.shape[2] == 1
            assert dec.fused_rows == (head_dim == 128)
            for mode in ("eager", "graph"):
                if mode == "graph":
                    dec.capture()
                    single.capture()
                dec.reset(0)
                single.reset(0)
                for t, tok in enumerate(ids):
                    for d in (dec, single):
                        with torch.cuda.stream(d.stream):
                            d.tok.fill_(int(tok))
                        d.step()
                        d.stream.synchronize()
                    full = gathered(dec.logits[0].float())
                    ref = single.logits[0].float().cpu()
                    assert rel(full, ref) <= 2e-2, (head_dim, mode, t, rel(full, ref))
                    picked = int(dec.tok[0])
                    assert picked == int(torch.argmax(full)), (head_dim, mode, t)
                    both = [None] * WORLD
                    dist.all_gather_object(both, picked)
                    assert both[0] == both[1], (head_dim, mode, t, both)
                dec.check()
                ar.check(dev)
                check_device_errors(dev)
            # a prompt prefilled as one chunk, then one decode step
            dec.reset(0)
            single.reset(0)
            dec.prefill(ids[:10])
            single.prefill(ids[:10])
            dec.stream.synchronize()
            single.stream.synchronize()
            full = gathered(dec.logits[0].float())
            assert rel(full, single.logits[0].float().cpu()) <= 2e-2, (head_dim, "prefill")
            dec.step()
            single.step()
            dec.stream.synchronize()
            single.stream.synchronize()
            full = gathered(dec.logits[0].float())
            assert rel(full, single.logits[0].float().cpu()) <= 2e-2, (head_dim, "after prefill")
            dec.check()
            ar.check(dev)
            dec.release()
            single.release()
            dist.barrier()
            ar.close()
        q.put((rank, "ok"))
    except Exception as e:                      # reported to the parent
        import traceback
        q.put((rank, repr(e) + traceback.format_exc()[-1500:]))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_tensor_parallel_decoder_two_gpus():
    pytest.importorskip("transformers")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res
