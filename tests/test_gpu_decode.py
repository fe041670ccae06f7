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


def _tiny(seed):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.Gemma3TextConfig(vocab_size=512, hidden_size=256, intermediate_size=512,
                                        num_hidden_layers=2, num_attention_heads=4,
                                        num_key_value_heads=2, head_dim=64,
                                        max_position_embeddings=128, sliding_window=4,
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
