#!/usr/bin/env python
"""Decode-step benchmark of the kvquant_b200 quantized-KV attention path.

Workload (default "longctx-1m-4bit"): LLaMA-2-7B shape -- batch 1, 32 KV heads
of 128 channels, 1,048,576 cached tokens in each of 32 layers, 4-bit NUQ keys
(per channel, pre-RoPE) and values (per token) with 1% fp16 outliers, RoPE
theta 10000. One step = one decode step of attention over the whole cache:
for every layer, the fused key kernel (which also leaves the softmax partials)
and the value kernel (which forms the probabilities from the raw scores). Synthetic
seeded data (the reference's wikitext-2 activations are not available); the
cache is built on the GPU by this library's quantize-on-append kernels.

Multi-GPU: one process per GPU (torchrun); KV heads are split across ranks
(strong scaling: the total cache is fixed) and each layer's per-head outputs
are all-gathered with NCCL. value = cached token positions (all heads, K and
V) scanned per second over the whole job: batch * tokens * layers / step time,
step time = max over ranks of CUDA-event time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
  python bench.py --codebook [--steps K]   (NUQ codebook fitting, offline calibration)
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "kvquant-paper-repro_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "4-bit KV decode attention: keys+values scanned/s, % of B200 HBM BW; 1–8 GPUs"
UNIT = "tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", default="longctx-1m-4bit")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count")
    ap.add_argument("--tokens", type=int, default=None, help="override the cached token count")
    ap.add_argument("--kv-heads", type=int, default=None,
                    help="override the KV head count (e.g. one rank's share of a head split)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-append", action="store_true")
    ap.add_argument("--codebook", action="store_true",
                    help="benchmark NUQ codebook fitting (offline calibration) instead of decode")
    ap.add_argument("--codebook-samples", type=int, default=1 << 24)
    ap.add_argument("--quantize", action="store_true",
                    help="measure quantize-on-append of one prefill layer on its own line")
    ap.add_argument("--config3", action="store_true",
                    help="full decode of a random-init LLaMA-2-7B through the Hugging Face "
                         "packed cache (32K-token prefill, then one-token steps)")
    ap.add_argument("--prefill", type=int, default=32768, help="--config3: prompt tokens")
    ap.add_argument("--new-tokens", type=int, default=128, help="--config3: decode steps")
    ap.add_argument("--shard", choices=["auto", "heads", "tokens"], default="auto",
                    help="multi-GPU split: KV heads, or token ranges of all heads (auto: heads "
                         "while every rank keeps at least 16 KV heads)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# the GPU arm
# ---------------------------------------------------------------------------
def setup_dist(args):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def peak_hbm():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def build_cache(wl, layers, h0, hl, dev, log, T=None, sink=True, seed=0):
    """Quantized cache of this rank's heads (and token range), every layer (built
    with our kernels). T: tokens of the range (default: the workload's); sink:
    whether its first token is the context's sink; seed: synthetic data seed."""
    import torch
    from kvquant import synthetic as syn
    from kvquant.kernels import quantize_keys, quantize_values

    B, C = wl.batch, wl.channels
    T = wl.tokens if T is None else T
    k = torch.empty((B, T, C), dtype=torch.float16, device=dev)
    v = torch.empty((B, T, C), dtype=torch.float16, device=dev)
    cache = []
    cbk = cbv = None
    t0 = time.time()
    q_ms = []  # quantize-on-append time of the whole prefill block, per layer (after the first)
    for layer in range(layers):
        syn.fill_layer(k, v, layer, seed=seed)
        ks, kz = syn.key_calibration(k, sink=sink)
        if cbk is None:  # one codebook pair for the synthetic model (same distribution per layer)
            cbk, cbv = syn.fit_codebooks(k, v, ks, kz, wl.bits)
        def quantize():
            return (quantize_keys(k, ks, kz, cbk, wl.bits, wl.outlier_ratio, sink, h0=h0,
                                  n_heads=hl, capacity=T),
                    quantize_values(v, cbv, wl.bits, wl.outlier_ratio, sink, h0=h0, n_heads=hl,
                                    capacity=T))
        if layer == 1:
            # quantize-on-append of one prefill block, kernels only: a first call
            # allocates the outputs, whose freed blocks the caching allocator hands
            # to the timed calls (no cudaMalloc inside the events)
            pk, pv = quantize()
            del pk, pv
            for _ in range(2):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                pk, pv = quantize()
                e1.record()
                e1.synchronize()
                q_ms.append(e0.elapsed_time(e1))
                del pk, pv
        pk, pv = quantize()
        cache.append((pk, pv))
        if layer == 0 or (layer + 1) % 8 == 0:
            torch.cuda.synchronize()
            log(f"layer {layer + 1}/{layers} quantized ({time.time() - t0:.1f}s, "
                f"{torch.cuda.memory_allocated(dev) / 2**30:.1f} GiB)")
    del k, v
    torch.cuda.empty_cache()
    qstat = None
    if q_ms:
        ms = min(q_ms)
        pk0, pv0 = cache[0]
        # fp16 input read once (the rank's key channels, the full value rows: per-token
        # stats span all channels); codes, outlier entries, row pointers, per-token
        # value scale/zero and the sinks written once
        in_bytes = B * T * (hl * 128 + C) * 2
        U = B * hl
        out_bytes = (2 * U * T * 16 * wl.bits + (pk0["nnz"] + pv0["nnz"]) * 4
                     + 2 * (2 * U * -(-T // 32) + 1) * 4 + B * T * 8 + 2 * B * hl * 128 * 2)
        alg = in_bytes + out_bytes
        peak, src = peak_hbm()
        qstat = {"ms_per_layer": ms, "tokens": T, "input_bytes": in_bytes,
                 "algorithmic_bytes": alg, "achieved_GBps": alg / (ms / 1e3) / 1e9,
                 "frac": alg / (ms / 1e3) / 1e9 / peak, "peak_GBps": peak, "peak_source": src,
                 "what": "quantize_keys + quantize_values of one layer's prefill block "
                         "(plan + emit, outliers, packing), kernels only (outputs come from "
                         "the caching allocator), CUDA events, best of 2"}
    return cache, qstat


def measure_decode_append(wl, h0, hl, dev, cbk, cbv, log, T0=4096, steps=32):
    """Decode-time append of one token (keys + values) into an appendable cache of
    this rank's heads: CUDA-event time per token and layer (O(1) in the length)."""
    import torch
    from kvquant import synthetic as syn
    from kvquant.kernels import (quantize_keys, quantize_values, make_appendable, append_keys,
                                 append_values, key_outlier_thresholds)

    B, C = wl.batch, wl.channels
    k = torch.empty((B, T0 + steps + 3, C), dtype=torch.float16, device=dev)
    v = torch.empty_like(k)
    syn.fill_layer(k, v, 0, seed=1)
    ks, kz = syn.key_calibration(k[:, :T0])
    pk = make_appendable(quantize_keys(k[:, :T0], ks, kz, cbk, wl.bits, wl.outlier_ratio, True,
                                       h0=h0, n_heads=hl), steps + 3)
    pv = make_appendable(quantize_values(v[:, :T0], cbv, wl.bits, wl.outlier_ratio, True,
                                         h0=h0, n_heads=hl), steps + 3)
    thr = key_outlier_thresholds(k[:, :T0], ks, kz, wl.outlier_ratio, h0=h0, n_heads=hl)
    rows = [(k[:, t:t + 1].contiguous(), v[:, t:t + 1].contiguous()) for t in range(T0, T0 + steps + 3)]
    for kt, vt in rows[:3]:
        append_keys(pk, kt, thr)
        append_values(pv, vt)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for kt, vt in rows[3:]:
        append_keys(pk, kt, thr, check=False)
        append_values(pv, vt, check=False)
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / steps
    log(f"decode append: {us:.1f} us per token and layer")
    return {"us_per_token_per_layer": us, "cached_tokens": T0, "kv_heads": hl,
            "what": "append_keys (calibrated thresholds) + append_values of one new token "
                    "into an appendable cache, CUDA events over 32 consecutive tokens"}


# DRAM bytes (ncu dram__bytes_read.sum + dram__bytes_write.sum) per algorithmic
# byte of each decode kernel, from one capture of the 4-bit 1%-outlier workload
# at 262144 tokens x 32 KV heads, fused softmax (traffic grows in proportion to
# the tokens).
DRAM_PER_ALGORITHMIC_BYTE = {"key_scores": (589057792 + 35775488) / 619708416,
                             "value_output": (618741248 + 4753664) / 620773216}


TRAFFIC_SOURCE = ("not measured on this launch: the DRAM bytes per algorithmic byte of one "
                  "ncu capture at 262144 tokens x 32 KV heads, 4-bit "
                  "(profiles/decode_kernels_longctx-4bit_262144tok.md), times this launch's "
                  "algorithmic bytes")

L2_BYTES = 126 * 2**20  # B200 L2


def flush_l2_needed(wl, layers, world) -> bool:
    """True when a rank's whole cache (about 32*bits + 18 bytes per head and token:
    codes of keys and values, outlier entries, per-token stats) could stay in L2
    between steps; the bench then writes a 256 MiB buffer between timed steps."""
    per_rank = layers * wl.batch * (wl.kv_heads // max(1, world)) * wl.tokens * (32 * wl.bits + 18)
    return per_rank < 2 * L2_BYTES


def shard_mode(args, wl, world) -> str:
    """'heads' or 'tokens'. The key kernel shares each 16-token block's RoPE
    twiddles across a work item's units, so a rank with few KV heads runs it
    below its 32-head rate; auto keeps KV-head sharding while every rank has at
    least 16 heads and splits token ranges of all heads beyond that."""
    if args.shard != "auto":
        return args.shard
    return "heads" if world == 1 or wl.kv_heads // world >= 16 else "tokens"


def bench_config(wl, layers, world, mode="heads"):
    """The workload description both arms print (identical for the same run)."""
    l2 = ("L2 flushed between timed steps (256 MiB write outside the timed region)"
          if flush_l2_needed(wl, layers, world)
          else "inputs larger than L2 (each step streams the whole cache, several GB)")
    return {"workload": wl.name, "batch": wl.batch, "kv_heads": wl.kv_heads,
            "q_per_kv": wl.q_per_kv, "tokens": wl.tokens, "layers": layers, "bits": wl.bits,
            "outlier_ratio": wl.outlier_ratio, "rope_base": wl.rope_base,
            "sharding": (f"kv heads / {world} GPUs" if mode == "heads" else
                         f"token ranges / {world} GPUs (all {wl.kv_heads} KV heads per GPU, "
                         "softmax partials all-gathered and merged)"),
            "compute": "fp16 tensor-core MMA on LUT-dequantized codes, fp32 accumulate",
            "l2": l2}


def algorithmic_bytes(wl, pk, pv, hl, T):
    """Bytes each kernel must move per layer (per launch) on this rank."""
    B, G, bits = wl.batch, wl.q_per_kv, wl.bits
    U = B * hl
    nt = -(-T // 32)
    codes = U * T * 16 * bits
    stats = B * hl * G * -(-T // 16) * 8  # softmax partials (max, sum) per 16-token block
    # key: codes, outliers, row pointers, calibration, sink, q; writes scores + partials
    key = (codes + pk["nnz"] * 4 + U * nt * 8 + 2 * hl * 128 * 4 + B * hl * 128 * 2
           + B * hl * G * 128 * 2 + B * hl * G * T * 4 + stats)
    # value: codes, outliers, row pointers, per-token scale/zero, sink, raw scores +
    # partials; writes the output
    value = (codes + pv["nnz"] * 4 + U * nt * 8 + B * T * 8 + B * hl * 128 * 2
             + B * hl * G * T * 4 + stats + B * hl * G * 128 * 2)
    return {"key_scores": key, "value_output": value}


def kernel_rates(batch, tokens, heads, key_ms, value_ms):
    """Per-rank rates of one layer's decode kernels: cached positions (all of the
    rank's KV heads) and (head, position) pairs per second, for the key kernel, the
    value path (prep + value + combine) and the two together."""
    out = {}
    for name, ms in (("key_scores", key_ms), ("value_output", value_ms),
                     ("combined", key_ms + value_ms)):
        sec = ms / 1e3
        out[name] = {"tokens_per_s": batch * tokens / sec,
                     "head_tokens_per_s": batch * tokens * heads / sec}
    return out


def run_gpu(args):
    import torch
    import torch.distributed as dist
    from kvquant import synthetic as syn
    from kvquant.kernels import qk_scores_stats, pv_out_scores, rope_inv_freq, decode_attention
    from kvquant.kernels.decode import DecodeWorkspace

    world, rank, local = setup_dist(args)
    dev = torch.device("cuda", local)
    wl = syn.WORKLOADS[args.workload]
    if args.tokens:
        import dataclasses
        wl = dataclasses.replace(wl, tokens=args.tokens, name=f"{wl.name}@{args.tokens}tok")
    if args.kv_heads:
        import dataclasses
        wl = dataclasses.replace(wl, kv_heads=args.kv_heads,
                                 name=f"{wl.name}@{args.kv_heads}kvheads")
    layers = args.layers or wl.layers
    from kvquant.sharding import (shard_heads, shard_tokens, gather_buffer, gather_head_outputs,
                                  gather_shard_partials)
    from kvquant.kernels import merge_shards, decode_attention_shard
    mode = shard_mode(args, wl, world)
    try:
        if mode == "heads":
            h0, hl = shard_heads(wl.kv_heads, world, rank)
            t0, t1 = 0, wl.tokens
        else:  # every rank: all KV heads over its range of cached positions
            h0, hl = 0, wl.kv_heads
            t0, t1 = shard_tokens(wl.tokens, world, rank)
    except ValueError as e:
        raise SystemExit(str(e))
    G = wl.q_per_kv
    T = t1 - t0  # cached tokens on this rank
    log = (lambda m: print(f"[rank {rank}] {m}", file=sys.stderr, flush=True))

    cache, qstat = build_cache(wl, layers, h0, hl, dev, log, T=T, sink=(t0 == 0),
                               seed=0 if mode == "heads" else rank)
    inv = rope_inv_freq(128, wl.rope_base).to(dev)
    qs = [syn.make_query(wl.batch, wl.kv_heads * G, l, 0, dev)[:, h0 * G:(h0 + hl) * G].contiguous()
          for l in range(layers)]
    Hq_l = hl * G
    scores = torch.empty((wl.batch, Hq_l, T), dtype=torch.float32, device=dev)
    stats = torch.empty((wl.batch * Hq_l, -(-T // 16), 2), dtype=torch.float32, device=dev)
    outs = [torch.empty((wl.batch, Hq_l, 128), dtype=torch.float16, device=dev)
            for _ in range(layers)]
    tok_split = mode == "tokens" and world > 1
    if tok_split:  # shard outputs + softmax row stats of every rank, merged per layer
        mls = [torch.empty((wl.batch * Hq_l, 2), dtype=torch.float32, device=dev)
               for _ in range(layers)]
        o_buf = [torch.empty((world, wl.batch, Hq_l, 128), dtype=torch.float16, device=dev)
                 for _ in range(layers)]
        ml_buf = [torch.empty((world, wl.batch * Hq_l, 2), dtype=torch.float32, device=dev)
                  for _ in range(layers)]
        merged = [torch.empty((wl.batch, Hq_l, 128), dtype=torch.float16, device=dev)
                  for _ in range(layers)]
        full = None
    else:
        full = [gather_buffer(outs[l], world) for l in range(layers)] if world > 1 else None
    stream = torch.cuda.current_stream(dev)
    # key (scores + softmax partials), value row max, value (softmax of the raw
    # scores fused in), combine; token ranges add the merge of the ranks' shards
    n_launch_per_layer = 5 if tok_split else 4

    def step(events=None):
        handles = []
        for l, (pk, pv) in enumerate(cache):
            if events is not None:
                events[l][0].record(stream)
            qk_scores_stats(qs[l], pk, inv, out=scores, stats_out=stats, pos0=t0)
            if events is not None:
                events[l][1].record(stream)
            if tok_split:
                pv_out_scores(scores, stats, pv, ml_out=mls[l], out=outs[l])
            else:
                outs[l] = pv_out_scores(scores, stats, pv)
            if events is not None:
                events[l][2].record(stream)
            if tok_split:
                handles.append((l, gather_shard_partials(outs[l], mls[l], o_buf[l], ml_buf[l],
                                                         async_op=True)))
            elif world > 1:
                handles.append((l, (gather_head_outputs(outs[l], full[l], async_op=True),)))
        for l, hs in handles:
            for h in hs:
                h.wait()
            if tok_split:
                merge_shards(o_buf[l], ml_buf[l], out=merged[l])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(layers)]
          for _ in range(args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    flush = (torch.empty(256 * 2**20, dtype=torch.uint8, device=dev)
             if flush_l2_needed(wl, layers, world) else None)
    if flush is None:
        t_start.record(stream)
        for s in range(args.steps):
            step(ev[s])
        t_end.record(stream)
    else:  # small caches: evict them from L2 before every step, time the steps only
        st_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
        for s in range(args.steps):
            flush.zero_()
            st_ev[s][0].record(stream)
            step(ev[s])
            st_ev[s][1].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    if flush is None:
        elapsed = t_start.elapsed_time(t_end)  # ms
    else:
        elapsed = sum(a.elapsed_time(b) for a, b in st_ev)
    key_ms = [ev[s][l][0].elapsed_time(ev[s][l][1]) for s in range(args.steps) for l in range(layers)]
    val_ms = [ev[s][l][1].elapsed_time(ev[s][l][2]) for s in range(args.steps) for l in range(layers)]
    if world > 1:
        t = torch.tensor([elapsed], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
    ms_step = elapsed / args.steps
    total_tokens = wl.batch * wl.tokens * layers  # the whole context, all ranks together
    value = total_tokens / (ms_step / 1e3)

    # e2e through the public API: pinned host q in, host output out, every step
    e2e = None
    if not args.no_e2e:
        q_host = [q.cpu().pin_memory() for q in qs]
        o_rows = wl.batch if tok_split else world * wl.batch  # token ranges: merged output
        o_host = [torch.empty((o_rows, Hq_l, 128), dtype=torch.float16).pin_memory()
                  for _ in range(layers)]
        q_dev = [torch.empty_like(q) for q in qs]
        wsp = DecodeWorkspace()

        def e2e_step():
            handles = []
            for l, (pk, pv) in enumerate(cache):
                q_dev[l].copy_(q_host[l], non_blocking=True)
                if tok_split:
                    o, ml = decode_attention_shard(q_dev[l], pk, pv, inv, pos0=t0, scores=scores,
                                                   stats=stats, out=outs[l], ml_out=mls[l],
                                                   workspace=wsp)
                    handles.append((l, gather_shard_partials(o, ml, o_buf[l], ml_buf[l],
                                                             async_op=True)))
                    continue
                o = decode_attention(q_dev[l], pk, pv, inv, workspace=wsp)
                if world > 1:
                    handles.append((l, (gather_head_outputs(o, full[l], async_op=True),)))
                else:
                    o_host[l].copy_(o, non_blocking=True)
            for l, hs in handles:
                for h in hs:
                    h.wait()
                if tok_split:
                    o_host[l].copy_(merge_shards(o_buf[l], ml_buf[l], out=merged[l]),
                                    non_blocking=True)
                else:
                    o_host[l].copy_(full[l], non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()

        for _ in range(max(1, args.warmup)):
            e2e_step()
        if world > 1:
            dist.barrier()
        e_el = 0.0
        for _ in range(args.steps):
            if flush is not None:
                flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            e2e_step()
            e1.record(stream)
            torch.cuda.synchronize()
            e_el += e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([e_el], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_el = float(t.item())
        e2e = {"value": total_tokens / (e_el / args.steps / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": sum(q.numel() * 2 for q in qs),
               "d2h_bytes_per_step": layers * o_rows * Hq_l * 128 * 2}

    append_stat = None
    if not args.no_append:
        append_stat = measure_decode_append(wl, h0, hl, dev, cache[0][0]["codebook"],
                                            cache[0][1]["codebook"], log)

    # roofline of the dominant kernel
    pk0, pv0 = cache[0]
    ab = algorithmic_bytes(wl, pk0, pv0, hl, T)
    k_avg, v_avg = statistics.mean(key_ms), statistics.mean(val_ms)
    dom, dom_ms = ("key_scores", k_avg) if k_avg >= v_avg else ("value_output", v_avg)
    peak, peak_src = peak_hbm()
    achieved = ab[dom] / (dom_ms / 1e3) / 1e9
    step_bytes = sum(ab.values()) * layers
    result = None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            cpu = cpu_baseline(wl, log)
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f16", "data": "synthetic",
            "config": bench_config(wl, layers, world, mode),
            "bytes_read_per_gpu_per_step": step_bytes,
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak,
                         "peak_source": peak_src, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": ab[dom] * DRAM_PER_ALGORITHMIC_BYTE[dom],
                         "traffic_source": TRAFFIC_SOURCE,
                         "bytes_per_launch": ab[dom], "launch_ms": dom_ms},
            "step_bandwidth_gbs": step_bytes / (ms_step / 1e3) / 1e9,
            "kernels_ms": {"key_scores": k_avg, "value_output": v_avg},
            "kernel_rates": kernel_rates(wl.batch, T, hl, k_avg, v_avg),
            "algorithmic_bytes_per_launch": ab,
            "cpu_baseline": cpu,
            "quantize_append": qstat,
            "decode_append": append_stat,
            "e2e": e2e,
            "gpu_launches": n_launch_per_layer * layers * args.steps,
            "clocks": clk,
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


# ---------------------------------------------------------------------------
# CPU baseline and the reference arm: the reference's decode path as torch ops
# on the host cores, over the reference's own cache format (one code per byte,
# CSR outliers; oracle/kvq_ref_torch.py)
# ---------------------------------------------------------------------------
CPU_SAMPLE_TOKENS = 1 << 15


def cpu_sample(wl, seed: int = 1234):
    """One layer of the workload's KV heads over a 32K-token slice of its
    context, in the reference's format."""
    from oracle import kvq_ref_torch as R
    T = min(wl.tokens, CPU_SAMPLE_TOKENS)
    return R.make_reference_cache(T, wl.kv_heads, wl.bits, wl.outlier_ratio, seed,
                                  wl.rope_base), T


def cpu_step(cache) -> float:
    """Seconds for one decode step of the sample layer (all its heads)."""
    from oracle import kvq_ref_torch as R
    t0 = time.perf_counter()
    R.decode_step(cache)
    return time.perf_counter() - t0


def cpu_threads() -> int:
    import torch
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def cpu_sample_text(wl, T, cores):
    return (f"1 layer x {wl.kv_heads} KV heads x {T} cached tokens of {wl.name} per step, "
            f"{wl.bits}-bit, {wl.outlier_ratio:g} outliers, in the reference's format (one code "
            f"per byte, CSR outliers): torch CPU port of the reference's dequant "
            f"(cb[q]+o)*s+z -> fp16, fp32 RoPE tables, q.K, softmax, p.V on {cores} threads; "
            f"value = cached positions of the slice / step time (the metric's tokens/s at "
            f"{wl.tokens} tokens assumes the linear cost in T)")


def cpu_baseline(wl, log, steps: int = 3):
    cores = cpu_threads()
    cache, T = cpu_sample(wl)
    cpu_step(cache)  # warm-up
    ts = [cpu_step(cache) for _ in range(steps)]
    val = T / statistics.median(ts)
    log(f"cpu baseline: {val:.3g} tokens/s ({statistics.median(ts):.2f} s per step)")
    return {"value": val, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": cpu_sample_text(wl, T, cores)}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from kvquant import synthetic as syn

    wl = syn.WORKLOADS[args.workload]
    cores = cpu_threads()
    cache, T = cpu_sample(wl)
    for _ in range(args.warmup):
        cpu_step(cache)
    walls = [cpu_step(cache) for _ in range(args.steps)]
    value = T / statistics.mean(walls)
    sample = cpu_sample_text(wl, T, cores)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": statistics.mean(walls) * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(wl, args.layers or wl.layers, args.gpus,
                               shard_mode(args, wl, args.gpus)),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------
# NUQ codebook fitting (offline calibration; --codebook)
# ---------------------------------------------------------------------------
CB_METRIC = "NUQ codebook fit (Fisher-weighted 1-D k-means, 16 centres): samples/s"
CB_BITS = 4
CB_REFINE = 2


def codebook_samples(n: int, seed: int = 0):
    """Normalised calibration activations in [-1, 1] (two clipped normal modes, like
    per-channel keys after min/max scaling) with Fisher-like gamma weights."""
    import numpy as np
    rng = np.random.default_rng(seed)
    half = n // 2
    x = np.concatenate([rng.normal(-0.2, 0.3, half), rng.normal(0.3, 0.25, n - half)])
    x = np.clip(x, -1.0, 1.0).astype(np.float32)
    rng.shuffle(x)
    w = rng.gamma(2.0, 1.0, n).astype(np.float32)
    return x, w


def codebook_cpu_baseline(x, w, n_cpu: int, log):
    """The reference's solver (weighted KMeans, n_init=10, max_iter=100) on the host
    cores, over the first n_cpu samples."""
    import torch
    from kvquant.quant.nuq import train_nuq_codebook
    xs, ws = torch.from_numpy(x[:n_cpu].copy()), torch.from_numpy(w[:n_cpu].copy())
    train_nuq_codebook(xs[:4096], ws[:4096], n_bits=CB_BITS)  # import / thread-pool warm-up
    t0 = time.perf_counter()
    train_nuq_codebook(xs, ws, n_bits=CB_BITS)
    wall = time.perf_counter() - t0
    cores = os.cpu_count() or 1
    log(f"codebook cpu baseline: {n_cpu / wall:.3g} samples/s ({wall:.1f}s)")
    return {"value": n_cpu / wall, "unit": "samples/s", "cores": cores, "kind": "port",
            "sample": f"{n_cpu} of the {x.size} samples; train_nuq_codebook on CPU tensors "
                      f"(scikit-learn KMeans, n_init=10, max_iter=100, the reference's solver), "
                      f"its default thread pool"}


def run_codebook(args):
    import torch
    from kvquant.kernels.cuda_ops import _ptr, get_cuda_ops
    from kvquant.quant.nuq import train_nuq_codebook

    def log(msg):
        print(msg, file=sys.stderr, flush=True)

    n = int(args.codebook_samples)
    x, w = codebook_samples(n)
    if args.impl == "reference":
        base = codebook_cpu_baseline(x, w, min(n, 1 << 18), log)
        print(json.dumps({
            "impl": "reference", "metric": CB_METRIC, "value": base["value"],
            "unit": "samples/s", "n_gpus": args.gpus, "steps": 1, "warmup": 1,
            "ms_per_step": n / base["value"] * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"codebook-fit-{n}-samples-4bit"}, "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "samples/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return
    dev = torch.device("cuda", 0)
    lib = get_cuda_ops().lib
    xd, wd = torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev)
    ws = torch.empty(int(lib.kvq_fit_codebook_workspace(n)), dtype=torch.uint8, device=dev)
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    out = torch.empty(2 ** CB_BITS, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=dev)  # inputs ~ L2 size: flush

    def fit():
        rc = lib.kvq_fit_codebook(_ptr(xd), _ptr(wd), n, CB_BITS, CB_REFINE, _ptr(out), _ptr(ws),
                                  ws.numel(), _ptr(status), stream.cuda_stream)
        if rc:
            raise RuntimeError(lib.kvq_last_error().decode())

    for _ in range(max(3, args.warmup)):
        fit()
    torch.cuda.synchronize()
    if int(status[0]):
        raise RuntimeError("codebook fit reported too few occupied bins")
    clocks = ClockSampler(0)
    clocks.start()
    time.sleep(0.3)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for a, b in evs:
        flush.zero_()
        a.record(stream)
        fit()
        b.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    value = n / (ms / 1e3)
    # end to end through the public API: pinned host samples in, centres back to the host
    xh, wh = torch.from_numpy(x).pin_memory(), torch.from_numpy(w).pin_memory()
    e2e_steps = max(2, min(args.steps, 5))
    train_nuq_codebook(xh.to(dev), wh.to(dev), n_bits=CB_BITS).cpu()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        c = train_nuq_codebook(xh.to(dev, non_blocking=True), wh.to(dev, non_blocking=True),
                               n_bits=CB_BITS).cpu()
    e2e = n * e2e_steps / (time.perf_counter() - t0)
    peak, src = peak_hbm()
    achieved = 8.0 * n / (ms / 1e3) / 1e9  # x and w read once: the algorithmic bytes
    base = None if args.no_cpu_baseline else codebook_cpu_baseline(x, w, min(n, 1 << 18), log)
    print(json.dumps({
        "metric": CB_METRIC, "value": value, "unit": "samples/s", "n_gpus": 1,
        "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"codebook-fit-{n}-samples-4bit", "refine_iters": CB_REFINE,
                   "l2": "flushed before every fit (256 MiB write)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": None, "peak_source": src,
                     "note": "whole fit (range, histogram, reduce, solve, 2 x refine + "
                             "finalize); algorithmic bytes = 8 B per sample, read once"},
        "cpu_baseline": base, "clocks": clk,
        "e2e": {"value": e2e, "unit": "samples/s", "h2d_bytes_per_step": 8 * n,
                "d2h_bytes_per_step": 4 * c.numel()},
        "gpu_launches": args.steps * (4 + 2 * CB_REFINE)}), flush=True)


# ---------------------------------------------------------------------------
# Config 3: a whole LLaMA-2-7B decoding over the packed quantized cache
# ---------------------------------------------------------------------------
C3_METRIC = "LLaMA-2-7B decode over a 4-bit packed KV cache: generated tokens/s"


def run_config3(args):
    """Random-init LLaMA-2-7B (fp16 weights ~ N(0, 0.02)), a uniform-random prompt,
    per-layer key calibration and NUQ codebooks from the first 4096 prompt tokens,
    then kvquant.hf_cache: the prefill quantized into appendable packed caches and
    one-token decode steps attending over the codes (4-bit, 1% outliers)."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM
    from kvquant.hf_cache import install, uninstall
    from kvquant.quant.kv_quantizer import KVQuantizer
    from kvquant.quant.nuq import fit_nuq_codebook_cuda

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    dev = torch.device("cuda", 0)
    log = (lambda m: print(f"[config3] {m}", file=sys.stderr, flush=True))
    S, N, bits = args.prefill, args.new_tokens, 4
    cfg = LlamaConfig(vocab_size=32000, hidden_size=4096, intermediate_size=11008,
                      num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=32,
                      max_position_embeddings=S + N + 16, rope_theta=10000.0,
                      initializer_range=0.02)
    torch.manual_seed(0)
    t0 = time.time()
    with torch.device(dev):
        torch.set_default_dtype(torch.float16)
        model = LlamaForCausalLM(cfg).eval()
        torch.set_default_dtype(torch.float32)
    model.set_attn_implementation("sdpa")
    weight_bytes = sum(p.numel() * p.element_size() for p in model.parameters())
    log(f"model built ({weight_bytes / 1e9:.1f} GB, {time.time() - t0:.0f} s)")
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg.vocab_size, (1, S), generator=g).to(dev)
    # calibration on the first 4096 prompt tokens (kvquant/calibration.py's statistics:
    # per-channel key min/max, codebooks fit to normalized values, scale^2 weights)
    L = cfg.num_hidden_layers
    kcal, vcal = {}, {}
    hooks = []
    for i, layer in enumerate(model.model.layers):
        hooks.append(layer.self_attn.k_proj.register_forward_hook(
            lambda m, inp, out, i=i: kcal.__setitem__(i, out.detach())))
        hooks.append(layer.self_attn.v_proj.register_forward_hook(
            lambda m, inp, out, i=i: vcal.__setitem__(i, out.detach())))
    with torch.no_grad():
        model(prompt[:, :4096])
    for h in hooks:
        h.remove()
    scales, zeros, cbk, cbv = [], [], [], []
    for i in range(L):
        x = kcal[i][0, 1:].float()
        lo, hi = x.amin(0), x.amax(0)
        sc, zr = (hi - lo) / 2, (hi + lo) / 2
        scales.append(sc)
        zeros.append(zr)
        kn = ((x - zr) / (sc + 1e-8)).clamp(-1, 1).reshape(-1)
        cbk.append(fit_nuq_codebook_cuda(kn, (sc ** 2).expand_as(x).reshape(-1), bits))
        v = vcal[i][0, 1:].float()
        vmin, vmax = v.amin(1, keepdim=True), v.amax(1, keepdim=True)
        vs, vz = (vmax - vmin) / 2, (vmax + vmin) / 2
        vn = ((v - vz) / (vs + 1e-8)).reshape(-1)
        cbv.append(fit_nuq_codebook_cuda(vn, (vs ** 2).expand_as(v).reshape(-1), bits))
    del kcal, vcal
    quantizer = KVQuantizer(cbk, cbv, scales, zeros, k_bits=bits, v_bits=bits,
                            outlier_ratio=0.01, sink_token=True)
    kv = install(model, quantizer, max_new_tokens=N + 1)
    try:
        with torch.no_grad():
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            out = model(prompt, past_key_values=kv, use_cache=True)
            e1.record()
            e1.synchronize()
            prefill_ms = e0.elapsed_time(e1)
            log(f"prefill {S} tokens: {prefill_ms:.0f} ms")
            tok = out.logits[:, -1:].argmax(-1)
            state = model.model.layers[0].self_attn._kvq_state
            kv_bytes = sum(sum(t.numel() * t.element_size() for t in (p["q_idx"],
                                                                      p["outlier_entries"]))
                           for p in state.pk + state.pv)
            clocks = ClockSampler(0)
            clocks.start()
            time.sleep(0.2)
            steps = []
            for n in range(N):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                out = model(tok, past_key_values=kv, use_cache=True)
                tok = out.logits[:, -1:].argmax(-1)
                tok.item()  # the generated token back on the host every step
                e1.record()
                e1.synchronize()
                steps.append(e0.elapsed_time(e1))
            clk = clocks.stop()
        assert kv.get_seq_length() == S + N
    finally:
        uninstall(model)
    ms = statistics.mean(steps[3:]) if N > 6 else statistics.mean(steps)
    print(json.dumps({
        "metric": C3_METRIC, "value": 1e3 / ms, "unit": "tokens/s", "n_gpus": 1,
        "steps": N, "warmup": 0, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "none", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"llama2-7b-{S}tok-prefill-{N}-decode-4bit",
                   "model": "LLaMA-2-7B shape, random init N(0, 0.02), fp16",
                   "prefill_tokens": S, "new_tokens": N, "bits": bits, "outlier_ratio": 0.01,
                   "attention": "kvquant.hf_cache (prefill: fake-quant keys/values through SDPA, "
                                "cache packed; decode: decode_attention on the codes, tokens "
                                "appended per step)"},
        "prefill_ms": prefill_ms,
        "decode_ms_per_token": ms, "decode_ms_first3": steps[:3],
        "kv_cache_bytes_per_step": kv_bytes, "weight_bytes_per_step": weight_bytes,
        "kv_fraction_of_step_bytes": kv_bytes / (kv_bytes + weight_bytes),
        "e2e": {"value": 1e3 / ms, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 8},
        "clocks": clk,
    }), flush=True)


def run_quantize(args):
    """Quantize-on-append of one prefill layer on its own JSON line: quantize_keys +
    quantize_values of the workload's layer (all heads, --tokens tokens), kernels
    only, best of 2 after a warm call (the same measurement as the default line's
    quantize_append)."""
    import dataclasses
    import torch
    from kvquant import synthetic as syn
    dev = torch.device("cuda", 0)
    log = (lambda m: print(f"[quantize] {m}", file=sys.stderr, flush=True))
    wl = syn.WORKLOADS[args.workload]
    if args.tokens:
        wl = dataclasses.replace(wl, tokens=args.tokens, name=f"{wl.name}@{args.tokens}tok")
    _, q = build_cache(wl, 2, 0, wl.kv_heads, dev, log)
    print(json.dumps({
        "metric": "quantize-on-append of one prefill layer (keys + values): tokens/s",
        "value": wl.tokens / (q["ms_per_layer"] / 1e3), "unit": "tokens/s", "n_gpus": 1,
        "higher_is_better": True, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"quantize-{wl.name}", "tokens": wl.tokens,
                   "kv_heads": wl.kv_heads, "bits": wl.bits, "outlier_ratio": wl.outlier_ratio},
        "ms_per_layer": q["ms_per_layer"],
        "roofline": {"bound": "hbm", "achieved": q["achieved_GBps"], "peak": q["peak_GBps"],
                     "peak_source": q["peak_source"], "unit": "GB/s", "frac": q["frac"],
                     "traffic": None, "bytes_per_launch": q["algorithmic_bytes"]},
        "what": q["what"]}), flush=True)


def main():
    args = parse()
    if args.config3:
        run_config3(args)
        return
    if args.codebook:
        if int(os.environ.get("RANK", "0")) == 0:
            run_codebook(args)
        return
    if args.quantize:
        if int(os.environ.get("RANK", "0")) == 0:
            run_quantize(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
