"""Model surgery: replace the attention/MLP ``nn.Linear`` layers of a model with OABFLinear.

Mirrors ``compress_gemma_model`` (flash_bfp/model.py:5-91): the same recursive name filter
(``self_attn``, ``mlp``, ``feed_forward``, ``lconv1d``; everything else — ``lm_head``,
embeddings, norms — is left alone), bias copy, compression on the layer's device and
release of the original weights. Compression runs on the GPU; layers whose weights sit on
the CPU or the meta device are compressed on the current CUDA device. With ``world`` > 1 each
rank keeps and compresses only its tensor-parallel part of every linear.
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


def _text_config(model):
    cfg = model.config
    return cfg.get_text_config() if hasattr(cfg, "get_text_config") else cfg


def compress_gemma_model(model: torch.nn.Module, compressor: OABFCompressor,
                         verbose: bool = False, *, rank: int | None = None,
                         world: int = 1) -> torch.nn.Module:
    """Replace every targeted linear by an OABFLinear (flash_bfp/model.py:5-91).

    With ``world`` > 1 (tensor parallelism, one process per GPU), rank ``rank`` keeps only its
    part of each linear, split as ``tp.DecoderPlan`` says (whole attention heads; the MLP's
    intermediate dimension in 256-column stages; the row-parallel o_proj / down_proj by input
    columns), compressed with the whole matrix's outlier threshold. The module then holds
    ``tp_mode`` ('column' or 'row') and ``tp_range`` (its rows or input columns); the sharded
    model runs through ``GemmaDecoder.from_hf(..., reducer=...)``, which sums the row-parallel
    partial outputs over the ranks."""
    plan = None
    if world > 1:
        from .tp import DecoderPlan
        if rank is None:
            raise ValueError("tensor-parallel compression needs this process's rank")
        plan = DecoderPlan.from_config(_text_config(model), rank, world)
    layers = find_linear_layers(model)
    if verbose:
        print(f"Found {len(layers)} linear projection layers to compress.")
    for parent, sub_name, lin, full in layers:
        dev = lin.weight.device
        if dev.type != "cuda":
            dev = torch.device("cuda", torch.cuda.current_device())
        W = lin.weight.data
        if plan is None:
            layer = OABFLinear(lin.in_features, lin.out_features, bias=lin.bias is not None)
            if lin.bias is not None and lin.bias.device.type != "meta":
                layer.bias.data.copy_(lin.bias.data)
            layer = layer.to(dev)
            layer.load_from_weight(W, compressor, device=dev)
        else:
            mode, lo, hi = plan.ranges(full)
            n_l, k_l = (hi - lo, lin.in_features) if mode == "column" else (lin.out_features, hi - lo)
            layer = OABFLinear(k_l, n_l, bias=lin.bias is not None).to(dev)
            if lin.bias is not None and lin.bias.device.type != "meta":
                # column-parallel: this rank's outputs; row-parallel: added once after the sum
                layer.bias.data.copy_(lin.bias.data[lo:hi] if mode == "column" else lin.bias.data)
            if W.device.type == "meta":
                W = torch.zeros(W.shape, dtype=W.dtype, device=dev)
            dp, sp = plan.compress(W.to(dev), full, compressor)
            layer.load_compressed(dp, sp, dev)
            layer.tp_mode, layer.tp_range = mode, (lo, hi)
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
