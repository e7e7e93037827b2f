"""Forward-hook integration (drop-in for kvquant/attention_patch.py).

Identical behaviour: hooks on every layer's self_attn.k_proj / v_proj replace
the projection output with quantizer.quantize_k / quantize_v (pre-RoPE key
quantization, per-token values; fake quant, as in the reference's perplexity
path, attention_patch.py:7-38). Hook handles are kept in a module global.
"""
from typing import List

from torch import nn

_PATCHED: List = []


def patch_model(model: nn.Module, quantizer):
    global _PATCHED
    unpatch_model(model)

    hooks = []
    for i, layer in enumerate(model.model.layers):
        k_proj = layer.self_attn.k_proj
        v_proj = layer.self_attn.v_proj

        def make_k_hook(idx):
            def hook(module, inp, out):
                assert out.dim() == 3, f"unexpected k_proj output shape: {out.shape}"
                return quantizer.quantize_k(idx, out)
            return hook

        def make_v_hook(idx):
            def hook(module, inp, out):
                assert out.dim() == 3, f"unexpected v_proj output shape: {out.shape}"
                return quantizer.quantize_v(idx, out)
            return hook

        hooks.append(k_proj.register_forward_hook(make_k_hook(i)))
        hooks.append(v_proj.register_forward_hook(make_v_hook(i)))

    _PATCHED = hooks
    return hooks


def unpatch_model(model: nn.Module = None):
    global _PATCHED
    for h in _PATCHED:
        try:
            h.remove()
        except Exception:
            pass
    _PATCHED = []
