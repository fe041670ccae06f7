"""Host-side pieces of the decode token step that need no GPU.

The rotary tables GemmaDecoder hands to the RoPE kernel are bit-identical to the cos/sin the
Hugging Face Gemma-3 rotary embedding produces for the same positions (both rope types), and a
model whose linears were not compressed is refused.
"""
import pytest
import torch

from flashbfp_b200.decode import rope_tables


def _cfg():
    transformers = pytest.importorskip("transformers")
    return transformers, transformers.Gemma3TextConfig(
        vocab_size=128, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, head_dim=64, max_position_embeddings=256,
        sliding_window=4, layer_types=["sliding_attention", "full_attention"])


@pytest.mark.parametrize("layer_type", ["sliding_attention", "full_attention"])
def test_rope_tables_match_hugging_face(layer_type):
    transformers, cfg = _cfg()
    from transformers.models.gemma3.modeling_gemma3 import Gemma3RotaryEmbedding
    rot = Gemma3RotaryEmbedding(cfg)
    n = 200
    x = torch.zeros(1, n, cfg.head_dim, dtype=torch.bfloat16)
    cos, sin = rot(x, torch.arange(n)[None, :], layer_type=layer_type)
    theta = cfg.rope_parameters[layer_type]["rope_theta"]
    c, s = rope_tables(theta, cfg.head_dim, n, "cpu")
    assert c.dtype == torch.bfloat16 and c.shape == (n, cfg.head_dim)
    assert torch.equal(c, cos[0]) and torch.equal(s, sin[0])


def test_uncompressed_model_is_refused():
    transformers, cfg = _cfg()
    from flashbfp_b200.decode import GemmaDecoder
    model = transformers.Gemma3ForCausalLM(cfg)
    with pytest.raises(TypeError, match="compress_gemma_model"):
        GemmaDecoder.from_hf(model, max_ctx=16)
