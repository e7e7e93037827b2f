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


@pytest.mark.parametrize("world", [2, 4])
def test_multi_rank_gather_matches_single_process(tmp_path, world):
    import torch.multiprocessing as mp
    out_path = str(tmp_path / "gathered.npy")
    mp.spawn(_rank_main, args=(world, _free_port(), out_path), nprocs=world, join=True)
    got = np.load(out_path)
    q, kh, vh, Hkv, G = _case()
    _, _, ref = O.decode_attention(q, kh, vh, Hkv, O.rope_inv_freq(128, 10000.0))
    assert got.shape == ref.shape
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-7)


# ---------------------------------------------------------------------------
# Token-range sharding
# ---------------------------------------------------------------------------
def test_shard_tokens_partition():
    from kvquant.sharding import shard_tokens
    for T, world in ((4096, 1), (4096, 2), (1 << 20, 8), (1000, 3), (2049, 8)):
        got = [shard_tokens(T, world, r) for r in range(world)]
        assert got[0][0] == 0 and got[-1][1] == T
        assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
        assert all(t1 > t0 and t0 % 256 == 0 for t0, t1 in got)
    with pytest.raises(ValueError):
        shard_tokens(300, 4, 0)


def test_oracle_shard_merge_is_the_whole_decode():
    q, kh, vh, Hkv, G = _case(T=200)
    inv = O.rope_inv_freq(128, 10000.0)
    _, _, ref = O.decode_attention(q, kh, vh, Hkv, inv)
    parts = [O.decode_shard(q, kh[:, a:b], vh[:, a:b], Hkv, inv, a) for a, b in ((0, 77), (77, 200))]
    got = O.merge_shards(*zip(*parts))
    np.testing.assert_allclose(got, ref, rtol=1e-10, atol=1e-12)


def _token_case_tokens(world):
    return 600 if world <= 2 else 1100  # every rank's range starts on a 256-token boundary


def _token_rank_main(rank, world, port, out_path):
    import torch.distributed as dist
    from kvquant.sharding import shard_tokens, gather_shard_partials
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, kh, vh, Hkv, G = _case(T=_token_case_tokens(world))
        t0, t1 = shard_tokens(kh.shape[1], world, rank)
        o, m, l = O.decode_shard(q, kh[:, t0:t1], vh[:, t0:t1], Hkv,
                                 O.rope_inv_freq(128, 10000.0), t0)
        B, Hq = o.shape[:2]
        o_t = torch.from_numpy(np.ascontiguousarray(o, dtype=np.float32))
        ml_t = torch.from_numpy(np.stack([m.reshape(-1), 1.0 / l.reshape(-1)], -1).astype(np.float32))
        o_buf = torch.empty((world, B, Hq, 128), dtype=torch.float32)
        ml_buf = torch.empty((world, B * Hq, 2), dtype=torch.float32)
        gather_shard_partials(o_t, ml_t, o_buf, ml_buf)
        if rank == 0:
            ms = [ml_buf[i, :, 0].numpy().astype(np.float64).reshape(B, Hq) for i in range(world)]
            ls = [1.0 / ml_buf[i, :, 1].numpy().astype(np.float64).reshape(B, Hq) for i in range(world)]
            merged = O.merge_shards([o_buf[i].numpy().astype(np.float64) for i in range(world)], ms, ls)
            np.save(out_path, merged)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_multi_rank_token_shards_match_single_process(tmp_path, world):
    """Each rank decodes its token range (positions offset), the shard outputs
    and row stats are all-gathered with the helper bench.py uses and merged."""
    import torch.multiprocessing as mp
    out_path = str(tmp_path / "merged.npy")
    mp.spawn(_token_rank_main, args=(world, _free_port(), out_path), nprocs=world, join=True)
    got = np.load(out_path)
    q, kh, vh, Hkv, G = _case(T=_token_case_tokens(world))
    _, _, ref = O.decode_attention(q, kh, vh, Hkv, O.rope_inv_freq(128, 10000.0))
    # the shard outputs and row stats travel as fp32 (as on the GPU path): a row max
    # of a few tens carries ~3e-6 absolute error into exp(m - M)
    np.testing.assert_allclose(got, ref, rtol=2e-5, atol=1e-5)


def test_bench_shard_mode():
    """bench.py keeps KV-head sharding while every rank has >= 16 heads."""
    import argparse
    import importlib.util
    from pathlib import Path
    spec = importlib.util.spec_from_file_location("bench", Path(__file__).resolve().parent.parent / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    from kvquant import synthetic as syn
    wl = syn.WORKLOADS["longctx-1m-4bit"]
    auto = argparse.Namespace(shard="auto")
    assert [bench.shard_mode(auto, wl, n) for n in (1, 2, 4, 8)] == ["heads", "heads", "tokens", "tokens"]
    assert bench.shard_mode(argparse.Namespace(shard="heads"), wl, 8) == "heads"
    cfg = bench.bench_config(wl, 32, 8, "tokens")
    assert cfg["sharding"].startswith("token ranges / 8 GPUs")
    assert not bench.flush_l2_needed(wl, 32, 8)
    assert bench.flush_l2_needed(syn.WORKLOADS["layer-4k-4bit"], 1, 1)
