"""The Gemma-3 decode token step (flashbfp_b200/decode.py, csrc/decode.cu) against Hugging Face.

A tiny random-init Gemma-3 (one sliding-window layer with a window of 4, one global layer) is
compressed with compress_gemma_model and run one token at a time through GemmaDecoder. The
reference is the same model whose targeted linears hold the dequantised OABF weights as plain
bf16 layers, run by Hugging Face over the whole sequence (eager attention, causal and sliding
masks). Per position the logits agree within 2e-2 relative L2: both sides round to bf16 at every
module boundary, but not at the same points inside attention, which this runs in fp32. The same
holds when the prompt goes through prefill as one chunk (20 rows: the linears take the tcgen05
prefill GEMM; 5 rows: 16-token GEMV launches) and decoding continues from it. The CUDA graph
replay reproduces the eager step, and generate() returns in-vocabulary tokens.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

T = 24


def _tiny(seed, sliding_window=4, max_pos=128):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.Gemma3TextConfig(vocab_size=512, hidden_size=256, intermediate_size=512,
                                        num_hidden_layers=2, num_attention_heads=4,
                                        num_key_value_heads=2, head_dim=64,
                                        max_position_embeddings=max_pos, sliding_window=sliding_window,
                                        layer_types=["sliding_attention", "full_attention"],
                                        attn_implementation="eager")
    torch.manual_seed(seed)
    model = transformers.Gemma3ForCausalLM(cfg).eval()
    with torch.no_grad():                       # non-trivial norm weights (HF initialises them to 0)
        for name, p in model.named_parameters():
            if "norm" in name:
                p.copy_(0.2 * torch.randn_like(p))
    return model


def _dequantised_reference(model):
    from flashbfp_b200 import OABFCompressor, _lib
    from flashbfp_b200.model import find_linear_layers
    L = _lib.lib()
    comp = OABFCompressor()
    for _, _, lin, _ in find_linear_layers(model):
        dev = lin.weight.device
        dp, sp = comp.compress_matrix_device(lin.weight.data)
        n, k = dp["orig_shape"]
        kpad, _ = dp["padded_shape"]
        W = torch.empty(n, k, dtype=torch.float32, device=dev)
        st = _lib.stream_ptr(dev)
        _lib.check(L.fbfp_dequant(_lib.ptr(dp["exponents"]), _lib.ptr(dp["signs"]), _lib.ptr(dp["payload"]),
                                  n, k, kpad, _lib.DTYPE_CODE[torch.float32], _lib.ptr(W), k, st), "dequant")
        if sp["count"]:
            _lib.check(L.fbfp_scatter_outliers(_lib.ptr(sp["block_idx"]), _lib.ptr(sp["offset"]),
                                               _lib.ptr(sp["value"]), sp["count"], kpad, n, k,
                                               _lib.DTYPE_CODE[torch.float32], _lib.ptr(W), k, st), "scatter")
        lin.weight.data.copy_(W.to(torch.bfloat16))
    return model


def _run(dec, ids):
    out = []
    dec.reset(0)
    for t in ids:
        with torch.cuda.stream(dec.stream):
            dec.tok.fill_(int(t))
        dec.step()
        dec.stream.synchronize()
        out.append(dec.logits[0].float().clone())
    dec.check()
    return torch.stack(out)


def test_decode_steps_match_hugging_face():
    from flashbfp_b200 import OABFCompressor
    from flashbfp_b200.decode import GemmaDecoder
    from flashbfp_b200.linear import check_device_errors
    from flashbfp_b200.model import compress_gemma_model
    dev = torch.device("cuda", 0)
    model = compress_gemma_model(_tiny(1).to(dev, torch.bfloat16), OABFCompressor())
    ref = _dequantised_reference(_tiny(1).to(dev, torch.bfloat16))
    ids = torch.randint(0, 512, (T,), generator=torch.Generator().manual_seed(7)).tolist()
    dec = GemmaDecoder.from_hf(model, max_ctx=32, max_prefill=20)
    ours = _run(dec, ids)
    check_device_errors(dev)
    with torch.no_grad():
        want = ref(torch.tensor([ids], device=dev)).logits[0].float()
    for i in range(T):
        rel = ((ours[i] - want[i]).norm() / want[i].norm()).item()
        assert rel <= 2e-2, (i, rel)
    # prompt chunks through prefill, then decoding continues from the filled cache
    for n_pre in (20, 5):
        dec.reset(0)
        dec.prefill(ids[:n_pre])
        dec.stream.synchronize()
        got = [dec.logits[0].float().clone()]
        for t in ids[n_pre:n_pre + 4]:
            with torch.cuda.stream(dec.stream):
                dec.tok.fill_(int(t))
            dec.step()
            dec.stream.synchronize()
            got.append(dec.logits[0].float().clone())
        dec.check()
        for j, g in enumerate(got):
            i = n_pre - 1 + j
            rel = ((g - want[i]).norm() / want[i].norm()).item()
            assert rel <= 2e-2, (n_pre, i, rel)
    with pytest.raises(ValueError, match="prompt chunk"):
        dec.prefill(ids[:21])
    # the same steps replayed from the CUDA graph
    dec.capture()
    again = _run(dec, ids)
    rel = ((again - ours).norm() / ours.norm()).item()
    assert rel <= 1e-3, rel
    toks = dec.generate(ids[:4], 6)
    assert len(toks) == 6 and all(0 <= t < 512 for t in toks)
    dec.release()


def test_position_past_the_cache_is_reported():
    from flashbfp_b200 import OABFCompressor
    from flashbfp_b200.decode import GemmaDecoder
    from flashbfp_b200.model import compress_gemma_model
    dev = torch.device("cuda", 0)
    model = compress_gemma_model(_tiny(2).to(dev, torch.bfloat16), OABFCompressor())
    dec = GemmaDecoder.from_hf(model, max_ctx=8, max_prefill=4)
    dec.reset(8)                                 # one past the last cache row: nothing is written
    dec.step()
    with pytest.raises(RuntimeError, match="position outside the KV cache"):
        dec.check()
    with pytest.raises(ValueError, match="exceed"):
        dec.generate([1, 2, 3], 6)


def test_long_context_split_attention_matches_hugging_face():
    """150 positions (the token step's attention splits them over three CTAs per head and
    merges), a sliding window of 100 that starts inside a range: per-position logits of the
    step-by-step decode against Hugging Face over the whole sequence."""
    from flashbfp_b200 import OABFCompressor
    from flashbfp_b200.decode import GemmaDecoder
    from flashbfp_b200.model import compress_gemma_model
    dev = torch.device("cuda", 0)
    n = 150
    model = compress_gemma_model(_tiny(3, 100, 256).to(dev, torch.bfloat16), OABFCompressor())
    ref = _dequantised_reference(_tiny(3, 100, 256).to(dev, torch.bfloat16))
    ids = torch.randint(0, 512, (n,), generator=torch.Generator().manual_seed(8)).tolist()
    dec = GemmaDecoder.from_hf(model, max_ctx=160, max_prefill=8)
    ours = _run(dec, ids)
    with torch.no_grad():
        want = ref(torch.tensor([ids], device=dev)).logits[0].float()
    for i in range(n):
        rel = ((ours[i] - want[i]).norm() / want[i].norm()).item()
        assert rel <= 2e-2, (i, rel)
    dec.release()


def test_batch_decode_matches_single_sequences():
    """Three sequences of different prompt lengths decoding together (one row each, at their own
    positions, in their own caches): teacher-forced, every sequence's logits equal those of the
    same sequence decoded alone (up to the order of fp32 sums in the batched lm_head), eager and
    replayed from the CUDA graph; generate() on the batch returns per-sequence continuations."""
    from flashbfp_b200 import OABFCompressor
    from flashbfp_b200.decode import GemmaDecoder
    from flashbfp_b200.model import compress_gemma_model
    dev = torch.device("cuda", 0)
    model = compress_gemma_model(_tiny(4, 8).to(dev, torch.bfloat16), OABFCompressor())
    g = torch.Generator().manual_seed(12)
    prompts = [torch.randint(0, 512, (L,), generator=g).tolist() for L in (5, 19, 2)]
    follow = [torch.randint(0, 512, (10,), generator=g).tolist() for _ in prompts]
    single = GemmaDecoder.from_hf(model, max_ctx=48, max_prefill=16)
    alone = []
    for p, f in zip(prompts, follow):
        single.reset(0)
        for i in range(0, len(p), 16):
            single.prefill(p[i:i + 16])
        got = []
        for t in f:
            with torch.cuda.stream(single.stream):
                single.tok.fill_(int(t))
            single.step()
            single.stream.synchronize()
            got.append(single.logits[0].float().clone())
        single.check()
        alone.append(torch.stack(got))
    batch = GemmaDecoder.from_hf(model, max_ctx=48, max_prefill=16, batch=3)
    assert batch.k_cache.shape[1] == 3 and batch.pos.shape == (3,)
    for mode in ("eager", "graph"):
        if mode == "graph":
            batch.capture()
        batch.reset(0)
        for b, p in enumerate(prompts):
            for i in range(0, len(p), 16):
                batch.prefill(p[i:i + 16], seq=b)
        assert batch.pos.tolist() == [len(p) for p in prompts]
        for s_ in range(10):
            with torch.cuda.stream(batch.stream):
                batch.tok.copy_(torch.tensor([f[s_] for f in follow], device=dev))
            batch.step()
            batch.stream.synchronize()
            for b in range(3):
                want = alone[b][s_]
                rel = ((batch.logits[b].float() - want).norm() / want.norm()).item()
                assert rel <= 1e-2, (mode, s_, b, rel)
        batch.check()
    outs = batch.generate(prompts, 4)
    assert len(outs) == 3 and all(len(o) == 4 and all(0 <= t < 512 for t in o) for o in outs)
    with pytest.raises(ValueError):
        batch.generate(prompts[:2], 4)
    batch.release()
    single.release()
