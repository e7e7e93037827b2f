"""The oracle's reference-precision decode (decode_fp16_path): the yardstick
the GPU parity tests use for a row's conditioning. No GPU."""
import numpy as np

from oracle import kvq_oracle as O
import synth


def test_fp16_path_is_the_float64_decode_to_fp16_rounding():
    k, v = synth.make_kv(1, 200, 256, seed=7)
    scale, zero = synth.key_calibration(k)
    cb = np.linspace(-1, 1, 16).astype(np.float32)
    kh = O.quantize_k(k, cb, scale, zero, 0.01, True)["dequant"]
    vh = O.quantize_v(v, cb, 0.01, True)["dequant"]
    q = (synth.make_query(1, 4, 128, seed=8).astype(np.float32) * 0.05).astype(np.float16)
    inv = O.rope_inv_freq(128, 10000.0)
    s, _, o = O.decode_attention(q, kh, vh, 2, inv)
    s16, o16 = O.decode_fp16_path(q, kh, vh, 2, inv)
    assert s16.dtype == np.float32 and o16.dtype == np.float16
    # fp16 rotated keys: scores within a few 2^-11 of the exact ones
    assert np.linalg.norm(s16 - s) / np.linalg.norm(s) < 1e-3
    assert np.linalg.norm(o16 - o) / np.linalg.norm(o) < 2e-3
    # the rotation is the reference's RoPE op (fp16 out), at an offset too
    s16b, _ = O.decode_fp16_path(q, kh, vh, 2, inv, pos0=1000)
    sb = O.key_scores(q, kh, 2, inv, 1000)
    assert np.linalg.norm(s16b - sb) / np.linalg.norm(sb) < 1e-3
    assert np.linalg.norm(s16b - s16) / np.linalg.norm(s16) > 0.1
