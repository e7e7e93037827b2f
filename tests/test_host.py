"""Host-side logic of the kvquant package that needs no GPU."""
import numpy as np
import pytest
import torch

from goldens import load_misc


def test_rope_inv_freq_matches_reference_bits():
    from kvquant.kernels.rope_fused import rope_inv_freq
    m = load_misc()
    for base in (10000, 500000):
        got = rope_inv_freq(128, float(base)).numpy()
        np.testing.assert_array_equal(got.view(np.uint32), m[f"inv_freq_b{base}"].view(np.uint32))


def test_ops_reject_cpu_tensors():
    from kvquant.kernels import dense_matvec_lut, sparse_matvec_csr, apply_rope_elementwise
    x = torch.zeros(4, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        dense_matvec_lut(x, torch.zeros(16))
    with pytest.raises(RuntimeError, match="CUDA"):
        sparse_matvec_csr(torch.zeros(3, dtype=torch.int32), torch.zeros(0, dtype=torch.int32),
                          torch.zeros(0, dtype=torch.float16), torch.zeros(4, dtype=torch.float16))
    with pytest.raises(RuntimeError, match="CUDA"):
        apply_rope_elementwise(torch.zeros(1, 2, 3, 8, dtype=torch.float16))


def test_quantizer_rejects_cpu_tensors():
    from kvquant import KVQuantizer
    q = KVQuantizer([torch.zeros(16)], [torch.zeros(16)], [torch.ones(128)], [torch.zeros(128)])
    with pytest.raises(RuntimeError, match="CUDA"):
        q.quantize_k(0, torch.zeros(1, 4, 128, dtype=torch.float16))


def test_missing_library_raises(monkeypatch, tmp_path):
    import kvquant.kernels.cuda_ops as co
    monkeypatch.setattr(co, "_ops", None)
    monkeypatch.setattr(co, "_lib", None)
    monkeypatch.setenv("KVQ_B200_LIB", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="not loadable"):
        co.get_cuda_ops()
    assert not co.cuda_available()


def test_kv_cache_container_bytes():
    from kvquant import QuantizedKVCache
    c = QuantizedKVCache()
    packed = {"q_idx": torch.zeros(2, 3, 2048, dtype=torch.uint8),
              "outlier_values": torch.zeros(10, dtype=torch.float16),
              "outlier_cols": torch.zeros(10, dtype=torch.int16),
              "outlier_rowptr": torch.zeros(13, dtype=torch.int32),
              "scale": torch.zeros(256), "zero": torch.zeros(256), "sink": None, "length": 70}
    c.append_k(1, packed)
    c.append_v(0, packed)
    assert c.k_cache[0] is None and c.seq_len == 70
    assert c.memory_bytes() == 2 * (2 * 3 * 2048 + 20 + 20 + 52 + 2048)
    c.clear()
    assert c.memory_bytes() == 0


def test_dense_sparse_helpers_follow_reference():
    from kvquant.quant.dense_sparse import extract_outliers, pack_csr, unpack_csr
    m = load_misc()
    for dim in (1, -1):
        _, _, mask = extract_outliers(torch.from_numpy(m["eo_x"]), 0.1, dim)
        np.testing.assert_array_equal(mask.numpy(), m[f"eo_mask_dim{dim}"])
    x = torch.tensor([[0, 1.5, 0], [0, 0, 0], [2.0, 0, -1.0]])
    v, c, rp = pack_csr(x)
    assert rp.tolist() == [0, 1, 1, 3] and c.tolist() == [1, 0, 2]
    assert torch.equal(unpack_csr(v, c, rp, 3, 3, dtype=torch.float32), x)


def test_hf_cache_install_and_uninstall():
    """kvquant.hf_cache hooks a LLaMA model and restores it (no forward pass: the
    quantize and decode kernels need the GPU)."""
    from transformers import LlamaConfig, LlamaForCausalLM
    from kvquant.hf_cache import ATTN_NAME, install, uninstall
    cfg = LlamaConfig(vocab_size=64, hidden_size=256, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=2, num_key_value_heads=1, head_dim=128)
    m = LlamaForCausalLM(cfg).eval()
    m.set_attn_implementation("sdpa")
    kv = install(m, quantizer=None, max_new_tokens=4)
    assert m.config._attn_implementation == ATTN_NAME
    assert kv.get_seq_length() == 0 and len(m._kvq_hooks) == 4
    assert all(hasattr(layer.self_attn, "_kvq_state") for layer in m.model.layers)
    uninstall(m)
    assert m.config._attn_implementation == "sdpa" and not m._kvq_hooks
    assert not any(hasattr(layer.self_attn, "_kvq_state") for layer in m.model.layers)


def test_bench_kernel_rates():
    """Per-kernel rates in the bench line: positions and (head, position) pairs per second."""
    import bench
    r = bench.kernel_rates(2, 1000, 32, 1.0, 0.5)
    assert r["key_scores"]["tokens_per_s"] == pytest.approx(2e6)
    assert r["value_output"]["head_tokens_per_s"] == pytest.approx(2 * 1000 * 32 / 0.5e-3)
    assert r["combined"]["tokens_per_s"] == pytest.approx(2000 / 1.5e-3)


def test_hf_cache_layer_counts_positions_only():
    """The Cache layer stores no key or value tensor: it counts positions so the
    model's masks and positions come out as with its dynamic cache."""
    from kvquant.hf_cache import _layer_cls
    layer = _layer_cls()()
    k = torch.zeros(1, 2, 5, 128, dtype=torch.float16)
    out_k, out_v = layer.update(k, k)
    assert out_k is k and out_v is k
    assert layer.get_seq_length() == 5 and layer.get_mask_sizes(1) == (6, 0)
    layer.update(k[:, :, :1], k[:, :, :1])
    assert layer.get_seq_length() == 6 and layer.get_max_cache_shape() == -1
    assert not hasattr(layer, "keys") or layer.keys is None
