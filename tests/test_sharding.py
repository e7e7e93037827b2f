"""KV-head sharding of the decode step: host logic on CPU with 2 gloo ranks.

Each rank decodes its KV-head shard with the oracle (the per-head arithmetic the
GPU kernels are checked against) and the shards are all-gathered with the same
helper bench.py uses over NCCL; the gathered output must equal the single-process
decode of all heads.
"""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import kvq_oracle as O
import synth


def test_shard_heads_partition():
    from kvquant.sharding import shard_heads
    for heads, world in ((32, 1), (32, 2), (32, 8), (8, 4), (8, 8)):
        got = [shard_heads(heads, world, r) for r in range(world)]
        covered = [h for h0, n in got for h in range(h0, h0 + n)]
        assert covered == list(range(heads))
    with pytest.raises(ValueError):
        shard_heads(32, 3, 0)
    with pytest.raises(ValueError):
        shard_heads(32, 2, 2)


def test_full_heads_order():
    from kvquant.sharding import full_heads
    buf = torch.arange(2 * 3 * 4 * 5, dtype=torch.float32).reshape(2 * 3, 4, 5)  # world*B, hl, D
    out = full_heads(buf, 2)
    assert out.shape == (3, 8, 5)
    for r in range(2):
        torch.testing.assert_close(out[:, 4 * r:4 * (r + 1)], buf[3 * r:3 * (r + 1)])


def _case(seed=3, B=2, Hkv=4, G=2, T=96, bits=4, ratio=0.02):
    k, v = synth.make_kv(B, T, Hkv * 128, seed=seed)
    scale, zero = synth.key_calibration(k)
    rng = np.random.default_rng(seed)
    cbk = np.sort(rng.uniform(-1, 1, 1 << bits)).astype(np.float32)
    cbv = np.sort(rng.uniform(-1, 1, 1 << bits)).astype(np.float32)
    q = synth.make_query(B, Hkv * G, 128, seed=seed + 1)
    kq = O.quantize_k(k, cbk, scale, zero, ratio, True)
    vq = O.quantize_v(v, cbv, ratio, True)
    return q, kq["dequant"], vq["dequant"], Hkv, G


def _rank_main(rank, world, port, out_path):
    import torch.distributed as dist
    from kvquant.sharding import shard_heads, gather_buffer, gather_head_outputs, full_heads
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, kh, vh, Hkv, G = _case()
        h0, n = shard_heads(Hkv, world, rank)
        cs = slice(h0 * 128, (h0 + n) * 128)
        _, _, o = O.decode_attention(q[:, h0 * G:(h0 + n) * G], kh[:, :, cs], vh[:, :, cs], n,
                                     O.rope_inv_freq(128, 10000.0))
        local = torch.from_numpy(np.ascontiguousarray(o, dtype=np.float32))
        buf = gather_buffer(local, world)
        gather_head_outputs(local, buf)
        if rank == 0:
            np.save(out_path, full_heads(buf, world).numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_gather_matches_single_process(tmp_path):
    import torch.multiprocessing as mp
    out_path = str(tmp_path / "gathered.npy")
    mp.spawn(_rank_main, args=(2, _free_port(), out_path), nprocs=2, join=True)
    got = np.load(out_path)
    q, kh, vh, Hkv, G = _case()
    _, _, ref = O.decode_attention(q, kh, vh, Hkv, O.rope_inv_freq(128, 10000.0))
    assert got.shape == ref.shape
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-7)
