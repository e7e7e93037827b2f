"""Quantized KV cache for Hugging Face causal LMs (LLaMA-style attention).

No counterpart in the reference: its attention_patch.py (kvquant/attention_patch.py:7-38)
fake-quantizes every k_proj / v_proj output, and the model still keeps the
dequantized fp16 keys and values in its own cache. Here the cache holds the packed
codes instead, and decode steps attend over them with the decode kernels:

* prefill (a query of more than one token): the k_proj / v_proj hooks quantize the
  block into appendable packed caches (pre-RoPE keys per channel, values per token,
  KVQuantizer.pack_k / pack_v) and, as the reference's hooks do, hand the fake-quant
  values back to the model, which attends over them with its SDPA path;
* decode (one query token): the hooks append the new token to the packed caches
  (append_keys / append_values; key outlier thresholds 0 by default, the reference's
  per-step semantics: every channel of a one-token block is an outlier), and the
  registered attention function runs decode_attention on the packed cache with the
  model's rotated query.

The Cache object stores no key or value tensor; it only counts positions, so the
model's masks and positions come out as with its dynamic cache.

Supported call pattern: one prefill call, then one-token decode calls, unpadded
batches, the model's default attention scaling 1/sqrt(128). Anything else raises
RuntimeError rather than attending over the wrong positions: a decode step whose
attention mask hides a cached position (a padded batch), a scaling other than
1/sqrt(128), a second multi-token call (chunked prefill, assisted decoding) after
the prefill, and a decode call before any prefill.
"""
from __future__ import annotations

import math

import torch

from .kernels import append_keys, append_values, decode_attention, make_appendable

ATTN_NAME = "kvquant_b200"


def _layer_cls():
    from transformers.cache_utils import CacheLayerMixin

    class KVQuantLayer(CacheLayerMixin):
        """Counts the cached positions of one layer; the codes live in the packed caches."""

        is_sliding = False

        def __init__(self):
            super().__init__()
            self.cumulative_length = 0

        def lazy_initialization(self, key_states, value_states):
            self.dtype, self.device = key_states.dtype, key_states.device
            self.is_initialized = True

        def update(self, key_states, value_states, *args, **kwargs):
            if not self.is_initialized:
                self.lazy_initialization(key_states, value_states)
            self.cumulative_length += key_states.shape[-2]
            return key_states, value_states

        def get_mask_sizes(self, query_length: int):
            return self.cumulative_length + query_length, 0

        def get_seq_length(self) -> int:
            return self.cumulative_length

        def get_max_cache_shape(self) -> int:
            return -1

    return KVQuantLayer


class KVQuantState:
    """The packed caches of every layer and the settings of the hooks."""

    def __init__(self, quantizer, n_layers: int, max_new_tokens: int, inv_freq: torch.Tensor,
                 key_thresholds=None, fake_quant_prefill: bool = True):
        self.quantizer = quantizer
        self.max_new_tokens = int(max_new_tokens)
        self.inv_freq = inv_freq.float()
        self.key_thresholds = key_thresholds  # per layer: tensor [n_kv_heads*128] or None = 0
        self.fake_quant_prefill = fake_quant_prefill
        self.pk = [None] * n_layers
        self.pv = [None] * n_layers

    def thresholds(self, layer: int, pk: dict):
        if self.key_thresholds is not None and self.key_thresholds[layer] is not None:
            return self.key_thresholds[layer]
        return torch.zeros(pk["n_heads"] * 128, dtype=torch.float32, device=pk["q_idx"].device)


def check_decode_call(state: "KVQuantState", layer: int, attention_mask, scaling) -> None:
    """Raises RuntimeError for a decode step the packed cache cannot serve.

    The decode kernels attend over every cached position with softmax scale
    1/sqrt(128); a mask that hides cached positions (left padding) or another
    scaling would silently change the result. The mask is the same for every
    layer, so it is read back (one small device-to-host copy) at layer 0 only.
    """
    if state.pk[layer] is None or state.pv[layer] is None:
        raise RuntimeError("kvquant hf_cache: decode call before the prefill")
    if scaling is not None and abs(float(scaling) * math.sqrt(128.0) - 1.0) > 1e-6:
        raise RuntimeError(f"kvquant hf_cache: attention scaling {scaling} is not 1/sqrt(128), "
                           "the decode kernels' softmax scale")
    if attention_mask is not None and layer == 0:
        m = attention_mask
        hidden = ~m if m.dtype == torch.bool else (m < 0)
        if bool(hidden.any()):
            raise RuntimeError("kvquant hf_cache: the attention mask hides cached positions "
                               "(padded batch); the packed cache attends over all of them")


def check_prefill_call(state: "KVQuantState", layer: int) -> None:
    """Raises RuntimeError for a multi-token call after the prefill: the packed
    cache takes one prefill block, then one token per call."""
    if state.pk[layer] is not None or state.pv[layer] is not None:
        raise RuntimeError("kvquant hf_cache: a multi-token call after the prefill (chunked "
                           "prefill or assisted decoding) is not supported; install a new cache")


def _attention(module, query, key, value, attention_mask, scaling=None, dropout=0.0, **kwargs):
    """Prefill: the model's SDPA path on the fake-quant chunk; decode: the packed cache."""
    state: KVQuantState = module._kvq_state
    if query.shape[2] > 1:
        from transformers.integrations.sdpa_attention import sdpa_attention_forward
        return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                      scaling=scaling, **kwargs)
    layer = module.layer_idx
    check_decode_call(state, layer, attention_mask, scaling)
    q = query[:, :, 0, :]
    out = decode_attention(q, state.pk[layer], state.pv[layer], state.inv_freq)
    return out[:, None], None  # [B, 1, Hq, 128], the layout the model reshapes


def install(model, quantizer, max_new_tokens: int, key_thresholds=None,
            fake_quant_prefill: bool = True):
    """Hooks `model` (a LLaMA-style causal LM with head_dim 128) to keep its KV cache
    quantized; returns the Cache object to pass as past_key_values. One prefill call,
    then at most max_new_tokens one-token decode calls. uninstall(model) undoes it."""
    from transformers import AttentionInterface
    from transformers.cache_utils import Cache

    AttentionInterface.register(ATTN_NAME, _attention)
    # the masks of the SDPA path (transformers builds none for an attention
    # function it does not know): padding reaches the prefill's SDPA call and
    # the decode check above
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS, sdpa_mask
    ALL_MASK_ATTENTION_FUNCTIONS.register(ATTN_NAME, sdpa_mask)
    layers = model.model.layers
    inv = model.model.rotary_emb.inv_freq.detach()
    state = KVQuantState(quantizer, len(layers), max_new_tokens, inv, key_thresholds,
                         fake_quant_prefill)
    hooks = []
    for i, layer in enumerate(layers):
        attn = layer.self_attn
        attn._kvq_state = state

        def k_hook(module, inp, out, idx=i):
            if out.shape[1] > 1:
                check_prefill_call(state, idx)
                p = quantizer.pack_k(idx, out, dequant=state.fake_quant_prefill)
                deq = p.pop("dequant", None)
                state.pk[idx] = make_appendable(p, state.max_new_tokens)
                return deq.to(out.dtype) if deq is not None else out
            pk = state.pk[idx]
            if pk is None:
                raise RuntimeError("kvquant hf_cache: decode call before the prefill")
            append_keys(pk, out, state.thresholds(idx, pk), check=False)
            return out

        def v_hook(module, inp, out, idx=i):
            if out.shape[1] > 1:
                if state.pv[idx] is not None:
                    check_prefill_call(state, idx)
                p = quantizer.pack_v(idx, out, dequant=state.fake_quant_prefill)
                deq = p.pop("dequant", None)
                state.pv[idx] = make_appendable(p, state.max_new_tokens)
                return deq.to(out.dtype) if deq is not None else out
            append_values(state.pv[idx], out, check=False)
            return out

        hooks.append(attn.k_proj.register_forward_hook(k_hook))
        hooks.append(attn.v_proj.register_forward_hook(v_hook))
    model._kvq_hooks = hooks
    model._kvq_prev_attn = model.config._attn_implementation
    model.set_attn_implementation(ATTN_NAME)
    return Cache(layer_class_to_replicate=_layer_cls())


def uninstall(model):
    for h in getattr(model, "_kvq_hooks", []):
        h.remove()
    model._kvq_hooks = []
    if getattr(model, "_kvq_prev_attn", None):
        model.set_attn_implementation(model._kvq_prev_attn)
    for layer in model.model.layers:
        if hasattr(layer.self_attn, "_kvq_state"):
            del layer.self_attn._kvq_state
