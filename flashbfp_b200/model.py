"""Model surgery: replace the attention/MLP ``nn.Linear`` layers of a model with OABFLinear.

Mirrors ``compress_gemma_model`` (flash_bfp/model.py:5-91): the same recursive name filter
(``self_attn``, ``mlp``, ``feed_forward``, ``lconv1d``; everything else — ``lm_head``,
embeddings, norms — is left alone), bias copy, compression on the layer's device and
release of the original weights. Compression runs on the GPU; layers whose weights sit on
the CPU or the meta device are compressed on the current CUDA device.
"""
from __future__ import annotations

import gc

import torch

from .compressor import OABFCompressor
from .linear import OABFLinear

TARGET_KEYS = ("self_attn", "mlp", "feed_forward", "lconv1d")


def find_linear_layers(model: torch.nn.Module, name: str = "model"):
    """(parent, attribute, module, dotted name) for every targeted nn.Linear (model.py:16-36)."""
    found = []

    def walk(module, prefix):
        for sub_name, sub in module.named_children():
            full = f"{prefix}.{sub_name}"
            if isinstance(sub, torch.nn.Linear):
                if any(k in full for k in TARGET_KEYS):
                    found.append((module, sub_name, sub, full))
            else:
                walk(sub, full)

    walk(model, name)
    return found


def compress_gemma_model(model: torch.nn.Module, compressor: OABFCompressor,
                         verbose: bool = False) -> torch.nn.Module:
    layers = find_linear_layers(model)
    if verbose:
        print(f"Found {len(layers)} linear projection layers to compress.")
    for parent, sub_name, lin, full in layers:
        dev = lin.weight.device
        if dev.type != "cuda":
            dev = torch.device("cuda", torch.cuda.current_device())
        layer = OABFLinear(lin.in_features, lin.out_features, bias=lin.bias is not None)
        if lin.bias is not None and lin.bias.device.type != "meta":
            layer.bias.data.copy_(lin.bias.data)
        layer = layer.to(dev)
        layer.load_from_weight(lin.weight.data, compressor, device=dev)
        setattr(parent, sub_name, layer)
        del lin.weight
        if lin.bias is not None:
            del lin.bias
        del lin
        if verbose:
            print(f"compressed {full}")
    gc.collect()
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return model
