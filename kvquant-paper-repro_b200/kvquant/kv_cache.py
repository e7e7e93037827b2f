"""Quantized KV cache container (drop-in for kvquant/kv_cache.py).

Per-layer dict slots as in the reference (kv_cache.py:4-44), filled with the
packed dicts that kvquant.kernels.quantize_keys / quantize_values return:
q_idx (bit-packed codes in 32-token tiles), outlier_values (fp16: the
dequantized key / value at each outlier), outlier_cols (int16 packed
(token_in_tile, channel)), outlier_rowptr (int32 per (head, tile, 16-token
block)), scale and zero, plus the fp16 sink token. memory_bytes
counts each tensor at its real element size (the reference counts int32
columns as 2 bytes and fp32 scales as 2 bytes).
"""
from __future__ import annotations


class QuantizedKVCache:
    def __init__(self):
        self.k_cache = []
        self.v_cache = []
        self.seq_len = 0

    def append_k(self, layer_idx: int, packed_k: dict):
        """kv_cache.py:17-20: stores the layer's packed keys (overwrites the slot)."""
        while len(self.k_cache) <= layer_idx:
            self.k_cache.append(None)
        self.k_cache[layer_idx] = packed_k
        self.seq_len = max(self.seq_len, int(packed_k.get("length", 0)))

    def append_v(self, layer_idx: int, packed_v: dict):
        """kv_cache.py:22-25."""
        while len(self.v_cache) <= layer_idx:
            self.v_cache.append(None)
        self.v_cache[layer_idx] = packed_v

    def append_tokens(self, layer_idx: int, k_new, v_new, key_thresholds=None):
        """Decode-time append of new tokens [B, S_new, C] into the layer's stored
        packed caches (which make_appendable must have produced), in place.
        No counterpart in the reference, whose hooks re-quantize each new block
        (kvquant/attention_patch.py:22-35)."""
        from .kernels import append_keys, append_values
        pk, pv = self.k_cache[layer_idx], self.v_cache[layer_idx]
        if pk is None or pv is None:
            raise RuntimeError(f"append_tokens: layer {layer_idx} holds no cache")
        append_keys(pk, k_new, key_thresholds)
        append_values(pv, v_new)
        self.seq_len = max(self.seq_len, int(pk["length"]))

    def clear(self):
        self.k_cache = []
        self.v_cache = []
        self.seq_len = 0

    def memory_bytes(self) -> int:
        total = 0
        for cache in (self.k_cache, self.v_cache):
            for packed in cache:
                if packed is None:
                    continue
                for key in ("q_idx", "outlier_values", "outlier_cols", "outlier_rowptr",
                            "scale", "zero", "sink"):
                    t = packed.get(key)
                    if t is not None:
                        total += t.numel() * t.element_size()
        return total
