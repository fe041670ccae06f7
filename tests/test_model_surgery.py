"""compress_gemma_model (flash_bfp/model.py:5-91) on a tiny random-init HF Gemma3 model.

CPU: the name filter picks exactly the attention and MLP projections of every decoder layer and
leaves lm_head, embeddings and norms alone. GPU: after the surgery the model's logits match those
of the same model whose linears hold the dequantised OABF weights (W_full) as plain bf16 layers,
so the only difference is the kernels' arithmetic.
"""
import pytest
import torch

from flashbfp_b200.model import TARGET_KEYS, find_linear_layers

PROJ = ["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
        "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"]


def _tiny_gemma3(seed=0):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.Gemma3TextConfig(vocab_size=512, hidden_size=256, intermediate_size=512,
                                        num_hidden_layers=2, num_attention_heads=4,
                                        num_key_value_heads=2, head_dim=64,
                                        max_position_embeddings=128, sliding_window=64)
    torch.manual_seed(seed)
    model = transformers.Gemma3ForCausalLM(cfg)
    return model.eval()


def test_filter_selects_attention_and_mlp_projections_only():
    model = _tiny_gemma3()
    names = sorted(full for _, _, _, full in find_linear_layers(model))
    expected = sorted(f"model.model.layers.{i}.{p}" for i in range(2) for p in PROJ)
    assert names == expected
    assert not any("lm_head" in n or "embed" in n for n in names)
    assert set(TARGET_KEYS) == {"self_attn", "mlp", "feed_forward", "lconv1d"}


@pytest.mark.gpu
def test_compressed_model_matches_dequantised_weights():
    from flashbfp_b200 import OABFCompressor, _lib
    from flashbfp_b200.linear import check_device_errors
    from flashbfp_b200.model import compress_gemma_model
    dev = torch.device("cuda", 0)
    model = _tiny_gemma3(seed=1).to(dev, torch.bfloat16)
    ref = _tiny_gemma3(seed=1).to(dev, torch.bfloat16)
    comp = OABFCompressor()
    L = _lib.lib()
    # reference model: every targeted linear gets its dequantised OABF weight (blocks + outliers)
    for parent, sub, lin, _ in find_linear_layers(ref):
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
    compress_gemma_model(model, comp)
    mods = dict(model.named_modules())
    assert type(model.lm_head).__name__ == "Linear"
    for i in range(2):
        for p in PROJ:
            assert type(mods[f"model.layers.{i}.{p}"]).__name__ == "OABFLinear", p
    ids = torch.randint(0, 512, (2, 24), device=dev)
    with torch.no_grad():
        out = model(ids).logits.float()
        exp = ref(ids).logits.float()
    check_device_errors()
    rel = ((out - exp).norm() / exp.norm()).item()
    assert rel <= 2e-2, rel
