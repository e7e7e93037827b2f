"""A Hugging Face LLaMA decoding over the packed quantized cache (kvquant.hf_cache)
against the same model with the reference's integration: the fake-quant k_proj /
v_proj hooks (attention_patch.py) and the model's own fp16 cache.

Both quantize the prefill block the same way, and both quantize each decode token
as a one-token block (every key channel an outlier), so the keys and values they
attend over are the same numbers; the outputs differ only by the decode kernels'
fp16 arithmetic against the model's SDPA.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _model(cuda):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=512,
                      num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=1,
                      head_dim=128, max_position_embeddings=4096, rope_theta=10000.0)
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).to(cuda, torch.float16).eval()
    model.set_attn_implementation("sdpa")
    return model


def _quantizer(model, prompt, bits=4):
    from kvquant.quant.kv_quantizer import KVQuantizer
    ks = {}
    hooks = [layer.self_attn.k_proj.register_forward_hook(
        lambda m, i, o, idx=n: ks.__setitem__(idx, o.detach()))
        for n, layer in enumerate(model.model.layers)]
    with torch.no_grad():
        model(prompt)
    for h in hooks:
        h.remove()
    scales, zeros = [], []
    for n in range(len(model.model.layers)):
        x = ks[n][0, 1:].float()
        lo, hi = x.amin(0), x.amax(0)
        scales.append((hi - lo) / 2)
        zeros.append((hi + lo) / 2)
    cb = torch.linspace(-1, 1, 1 << bits, device=prompt.device)
    L = len(model.model.layers)
    return KVQuantizer([cb] * L, [cb] * L, scales, zeros, k_bits=bits, v_bits=bits,
                       outlier_ratio=0.01, sink_token=True)


def test_quantized_cache_decodes_like_the_reference_hooks(cuda):
    from transformers import DynamicCache
    from kvquant.attention_patch import patch_model, unpatch_model
    from kvquant.hf_cache import install, uninstall
    model = _model(cuda)
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, 512, (1, 300), generator=g).to(cuda)
    quantizer = _quantizer(model, prompt)
    steps = 6

    ref_logits, tokens = [], []
    patch_model(model, quantizer)
    with torch.no_grad():
        cache = DynamicCache()
        out = model(prompt, past_key_values=cache, use_cache=True)
        ref_logits.append(out.logits[:, -1].float())
        for _ in range(steps):
            tok = out.logits[:, -1:].argmax(-1)
            tokens.append(tok)
            out = model(tok, past_key_values=cache, use_cache=True)
            ref_logits.append(out.logits[:, -1].float())
    unpatch_model(model)

    kv = install(model, quantizer, max_new_tokens=steps)
    try:
        got = []
        with torch.no_grad():
            out = model(prompt, past_key_values=kv, use_cache=True)
            got.append(out.logits[:, -1].float())
            for tok in tokens:  # the reference's tokens (teacher forcing)
                out = model(tok, past_key_values=kv, use_cache=True)
                got.append(out.logits[:, -1].float())
        assert kv.get_seq_length() == prompt.shape[1] + steps
    finally:
        uninstall(model)
    assert model.config._attn_implementation == "sdpa"
    # prefill: the same fake-quant keys and values through the same SDPA path
    torch.testing.assert_close(got[0], ref_logits[0], rtol=0, atol=0)
    for s, (a, b) in enumerate(zip(got[1:], ref_logits[1:])):
        err = ((a - b).norm() / b.norm()).item()
        assert err <= 2e-3, (s, err)


def test_padded_batch_and_second_prefill_raise(cuda):
    """A left-padded batch of 2 reaches the decode step with cached pad
    positions masked, which the packed cache cannot honour: it raises. So does
    a second multi-token call after the prefill."""
    from kvquant.hf_cache import install, uninstall
    model = _model(cuda)
    g = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, 512, (2, 64), generator=g).to(cuda)
    quantizer = _quantizer(model, prompt[:1])
    mask = torch.ones_like(prompt)
    mask[1, :5] = 0  # left padding of the second sequence
    kv = install(model, quantizer, max_new_tokens=4)
    try:
        with torch.no_grad():
            out = model(prompt, attention_mask=mask, past_key_values=kv, use_cache=True)
            tok = out.logits[:, -1:].argmax(-1)
            mask2 = torch.cat([mask, torch.ones_like(tok)], 1)
            with pytest.raises(RuntimeError, match="hides cached positions"):
                model(tok, attention_mask=mask2, past_key_values=kv, use_cache=True)
    finally:
        uninstall(model)
    kv = install(model, quantizer, max_new_tokens=4)
    try:
        with torch.no_grad():
            model(prompt[:1], past_key_values=kv, use_cache=True)
            with pytest.raises(RuntimeError, match="after the prefill"):
                model(prompt[:1, :8], past_key_values=kv, use_cache=True)
    finally:
        uninstall(model)
