#!/usr/bin/env python
"""Benchmark: Qwen3-0.6B decode step at B=128 per GPU on the sm_100a kernels.

Workload (one step): the full decode step of a random-init bf16 Qwen3-0.6B
(28 layers, hidden 1024, 16/8 GQA heads, head_dim 128, SwiGLU 3072, vocab
151936, QK-RMSNorm, RoPE theta 1e6) for 128 sequences per GPU with contexts
uniform in [512, 1024] over a paged cache of 512 blocks x 256 tokens,
captured in a CUDA graph as the engine's DecodeGraph does. Synthetic data:
seeded random weights, KV pool, token ids and lengths. Every step streams
~11.6 GB of KV cache (larger than the 126 MB L2), so no L2 flush is needed.

  value        tokens/s of the device-timed graph replay (next-token argmax
               included), summed over GPUs; weak scaling (128 rows per GPU).
  e2e          the same through DecodeGraph.step(): pinned host -> device
               copy of ids/pos/block table/lengths, replay, next tokens back
               to the host, every step.
  roofline     the paged decode attention op (decode kernel + combine) timed
               alone over the 28 layer caches with CUDA events: algorithmic
               KV bytes per launch / launch duration, against the measured
               HBM copy bandwidth.
  cpu_baseline the reference's decode step in fp32 on the host cores
               (oracle.qwen3_step), all 28 layers, median of --cpu-steps.
  secondary    (N=1) one line per other workload, each timed with CUDA events
               over input sets larger than the L2 together (CUDA graph,
               back to back) and checked against the fp32 oracle on
               sampled rows (max_abs_err), beside the reference's own kernels
               on the same GPU where they run (flash-attn 2.8.3, torch SDPA)
               and its CPU attention path on the host cores: single-layer
               decode B=8 and B=128, long-context decode B=32 with 256- and
               16-token blocks, prefill of 16 packed prompts and of one
               prompt, chunked prefill, and the whole step over 16-token
               blocks.
  kv_head_sharded  (N>1) the KV-head-sharded partition per layer (NCCL and
               the fused NVLink gather), with its parity on every rank.

--impl reference times the CPU step alone (rank 0), with the same metric and
config.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

B_PER_GPU = 128
CTX_LO, CTX_HI = 512, 1024
NUM_BLOCKS, BLOCK_SIZE = 512, 256
METRIC = "decode tok/s (Qwen3-0.6B decode step, B=128/GPU, ctx U[512,1024], paged 256-token blocks, CUDA graph)"
WORKLOAD = "qwen3-0.6b decode step, B=128 per GPU, contexts U[512,1024], 512x256-token paged KV blocks"
FALLBACK_HBM_GBS = 6650.0


def env_int(name, default):
    v = os.environ.get(name)
    return int(v) if v is not None else default


def measured_peak_hbm():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        # address the GPU by UUID: CUDA's device order need not match nvidia-smi's
        try:
            self.index = f"GPU-{torch.cuda.get_device_properties(index).uuid}"
        except Exception:
            self.index = str(index)
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
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
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def bench_config(world: int) -> dict:
    """The workload description both arms print (identical for a given N)."""
    return {"workload": WORKLOAD, "global_batch": world * B_PER_GPU, "seq_len": f"U[{CTX_LO},{CTX_HI}]",
            "parallelism": f"request-sharded x{world} (no collective)",
            "l2": "inputs larger than L2 (~11.6 GB KV streamed per step)", "cuda_graph": True}


DATA = "synthetic (seeded random weights, KV pool, ids, lengths)"


def host_cores() -> dict:
    return {"cores": len(os.sched_getaffinity(0)), "threads": torch.get_num_threads()}


def synth_inputs(rank: int, seed: int = 0):
    """Seeded per-rank decode inputs: lengths, block tables, ids."""
    import __graft_entry__

    __graft_entry__.load_package()
    from lean_infer_b200 import workloads as W

    s = seed + 1000 * rank
    while True:
        L = W.seq_lengths(B_PER_GPU, CTX_LO, CTX_HI, s)
        try:
            bt, _ = W.deal_blocks(L, BLOCK_SIZE, NUM_BLOCKS, s)
            break
        except ValueError:
            s += 1
    g = torch.Generator().manual_seed(s + 3)
    ids = torch.randint(0, 151936, (B_PER_GPU, 1), generator=g)
    return ids, (L - 1).long(), bt, L.to(torch.int32)


def cpu_reference_run(steps: int, warmup: int):
    """The reference's fp32 decode step, all 28 layers, on the host cores;
    returns tok/s and a description of what was timed."""
    from oracle.qwen3_step import CpuQwen3Decode

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    m = CpuQwen3Decode()
    ids, pos, bt, ctx = synth_inputs(0)
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        m.decode_step(ids, pos, bt, ctx)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    sec = statistics.median(times)
    return {
        "value": B_PER_GPU / sec,
        "unit": "tok/s",
        "cores": cores,
        "kind": "port",
        "sample": (f"the whole fp32 decode step (28 layers, embedding, lm_head) for B=128 rows of the benchmark "
                   f"workload on {cores} host threads; median of {steps} timed steps after {warmup} warm-up"),
        "ms_per_step": sec * 1e3,
        "steps_timed": steps,
    }


# --------------------------------------------------------------------------
# timing and checking helpers for the per-kernel lines
# --------------------------------------------------------------------------
L2_BYTES = 126 << 20


def rotating_us(fns, reps: int = 5) -> float:
    """Mean device time of one call when calls over distinct input sets run
    back to back: every fn in `fns` works on its own inputs, chosen so that
    all of them together exceed the 126 MB L2 (a call never finds its inputs
    left in L2 by the previous one, as in the 28-layer decode step). The
    calls are captured in one CUDA graph; CUDA events bracket `reps` replays
    on the current stream."""
    for f in fns:
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in fns:
            f()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) * 1e3 / (reps * len(fns))
    del g
    return t


def sets_for(bytes_per_set: int, minimum: int = 1) -> int:
    """Input sets whose total exceeds the L2 (at least `minimum`)."""
    return max(minimum, L2_BYTES // max(bytes_per_set, 1) + 1)


def compact_rows(q, k_cache, v_cache, block_table, seqlens, rows):
    """CPU copies of the given rows' queries, lengths and only the pool blocks
    they read, with their block tables renumbered into the compact pool (the
    oracle then reads exactly what the kernel read)."""
    rows = torch.as_tensor(rows, dtype=torch.long)
    BS = k_cache.shape[1]
    L = seqlens.cpu()[rows].long()
    btr = block_table.cpu()[rows]
    nblk = [max(1, -(-int(n) // BS)) for n in L]
    ids = torch.cat([btr[i, :n].long() for i, n in enumerate(nblk)])
    kc = k_cache[ids.to(k_cache.device)].cpu()
    vc = v_cache[ids.to(v_cache.device)].cpu()
    bt = torch.zeros(len(rows), max(nblk), dtype=torch.int32)
    o = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = torch.arange(o, o + n, dtype=torch.int32)
        o += n
    return q.cpu()[rows], kc, vc, bt, L.to(torch.int32)


def decode_err(out, w, rows):
    """max |out - oracle| over the given rows of a decode batch."""
    from oracle import paged_attention as opa

    q, kc, vc, bt, L = compact_rows(w.q, w.k_cache, w.v_cache, w.block_table, w.cache_seqlens, rows)
    ref = opa.paged_decode(q, kc, vc, bt, L)
    return float((out.cpu()[torch.as_tensor(rows)].float() - ref).abs().max())


def cpu_decode_us(w, rows, reps: int = 3) -> float:
    """The reference's CPU decode attention (fp32: gather the rows' keys and
    values through the block table, one masked SDPA) timed on the host cores
    for `rows`, in microseconds."""
    from oracle import paged_attention as opa

    q, kc, vc, bt, L = compact_rows(w.q, w.k_cache, w.v_cache, w.block_table, w.cache_seqlens, rows)
    kc, vc = kc.float(), vc.float()
    opa.paged_decode_padded(q, kc, vc, bt, L)
    t = []
    for _ in range(reps):
        t0 = time.perf_counter()
        opa.paged_decode_padded(q, kc, vc, bt, L)
        t.append(time.perf_counter() - t0)
    return statistics.median(t) * 1e6


def flash_attn_module():
    """flash-attn 2.8.3, the reference's attention dependency, if it imports."""
    try:
        import flash_attn

        return flash_attn
    except Exception:
        return None


def secondary_metrics(pkg, dev):
    """The metric's other components on one GPU, each with its own parity
    check against the fp32 oracle and, where they run, the reference's GPU
    kernels (flash-attn 2.8.3, torch SDPA) and its CPU path on the host cores.
    Every time is a CUDA-graph mean over input sets that together exceed the
    L2 (rotating_us), the same for every implementation compared."""
    from lean_infer_b200 import workloads as W
    from oracle import paged_attention as opa

    out = {}
    fa = flash_attn_module()
    hbm, hbm_kind = measured_peak_hbm()
    peak, peak_kind = measured_peak_bf16()
    cores = host_cores()
    torch.set_num_threads(cores["cores"])
    cores = host_cores()

    def decode_line(ws, name, workload, rows, cpu_rows, fa_ok):
        w = ws[0]
        B, _, Hq, D = w.q.shape
        alg = w.kv_bytes + 2 * B * Hq * D * 2

        def ours(x):
            return pkg.flash_attn_with_kvcache(x.q, x.k_cache, x.v_cache, cache_seqlens=x.cache_seqlens,
                                               block_table=x.block_table, causal=True, num_splits=1)

        us = rotating_us([lambda x=x: ours(x) for x in ws])
        o = ours(w)
        torch.cuda.synchronize()
        line = {"workload": workload, "us": us, "gbs": alg / (us * 1e-6) / 1e9, "peak_gbs": hbm,
                "frac": alg / (us * 1e-6) / 1e9 / hbm, "peak_source": hbm_kind, "alg_bytes": alg,
                "input_sets": len(ws), "max_abs_err": decode_err(o, w, rows), "checked_rows": len(rows),
                "tolerance": 2e-2}
        if fa is not None and fa_ok:
            def theirs(x):
                return fa.flash_attn_with_kvcache(x.q, x.k_cache, x.v_cache, cache_seqlens=x.cache_seqlens,
                                                  block_table=x.block_table, causal=True, num_splits=1)

            try:
                fus = rotating_us([lambda x=x: theirs(x) for x in ws])
                line["flash_attn_us"] = fus
                line["flash_attn_max_abs_err"] = decode_err(theirs(w), w, rows)
                line["speedup_vs_flash_attn"] = fus / us
            except Exception as e:  # a kernel image missing for this GPU, say
                line["flash_attn"] = f"did not run: {type(e).__name__}: {str(e)[:120]}"
        cpu_us = cpu_decode_us(w, cpu_rows)
        frac_keys = float(w.cache_seqlens[torch.as_tensor(cpu_rows, device=w.cache_seqlens.device)].sum()) / \
            float(w.cache_seqlens.sum())
        line["cpu_reference"] = {"us": cpu_us / frac_keys, **cores,
                                 "sample": f"fp32 gather + masked SDPA over {len(cpu_rows)} of {B} rows, "
                                           f"scaled by the key count to all rows"}
        out[name] = line

    # C1: single-layer decode, B=8, 512x256 pool, contexts U[512,1024]
    ws = [W.decode_batch(8, CTX_LO, CTX_HI, num_blocks=NUM_BLOCKS, block_size=BLOCK_SIZE, seed=11 + i, device=dev)
          for i in range(sets_for(8 * 768 * 4096))]
    decode_line(ws, "decode_c1_b8", "B=8, contexts U[512,1024], pool 512x256, one layer", list(range(8)),
                list(range(8)), True)
    del ws
    # one layer of the headline step: B=128
    ws = [W.decode_batch(B_PER_GPU, CTX_LO, CTX_HI, num_blocks=NUM_BLOCKS, block_size=BLOCK_SIZE, seed=1 + i,
                         device=dev) for i in range(2)]
    decode_line(ws, "decode_b128_layer", "B=128, contexts U[512,1024], pool 512x256, one layer",
                list(range(0, 128, 8)), list(range(0, 128, 16)), True)
    del ws
    # C4: long-context split-KV decode, B=32, contexts U[8192,32768], 256- and 16-token blocks
    for bs in (256, 16):
        w = W.decode_batch(32, 8192, 32768, num_blocks=None, block_size=bs, seed=40, device=dev)
        L = w.cache_seqlens.cpu()
        rows = sorted({int(L.argmin()), int(L.argmax()), int(L.argsort()[16])})
        decode_line([w], "decode_long_b32" if bs == 256 else "decode_long_b32_bs16",
                    f"B=32, contexts U[8192,32768], {bs}-token blocks (split-KV)", rows, rows[:2], bs % 256 == 0)
        del w
    torch.cuda.synchronize()

    # C3: causal varlen prefill, 16 packed prompts of U[512,1024]
    ws = [W.prefill_batch(16, CTX_LO, CTX_HI, seed=3 + 100 * i, device=dev) for i in range(3)]
    w = ws[0]

    def ours_p(x):
        mx = int(x.lengths.max())
        return pkg.flash_attn_varlen_func(x.q, x.k, x.v, x.cu_seqlens, x.cu_seqlens, mx, mx, causal=True)

    us = rotating_us([lambda x=x: ours_p(x) for x in ws])
    flops = sum(x.causal_flops for x in ws) / len(ws)
    o = ours_p(w)
    qc, kc, vc, cu = w.q.cpu(), w.k.cpu(), w.v.cpu(), w.cu_seqlens.cpu()
    t0 = time.perf_counter()
    ref = opa.varlen_causal_prefill(qc, kc, vc, cu)
    cpu_s = time.perf_counter() - t0
    tf = flops / (us * 1e-6) / 1e12
    line = {"workload": "16 packed prompts, lengths U[512,1024], causal, 16/8 heads, D=128", "us": us, "tflops": tf,
            "peak_tflops": peak, "frac": tf / peak, "peak_source": peak_kind, "flops": flops,
            "input_sets": len(ws), "max_abs_err": float((o.float().cpu() - ref).abs().max()), "tolerance": 2e-2,
            "cpu_reference": {"us": cpu_s * 1e6 * flops / w.causal_flops, **cores,
                              "sample": "fp32 causal SDPA per prompt, all 16 prompts of one set"}}
    if fa is not None:
        def theirs_p(x):
            mx = int(x.lengths.max())
            return fa.flash_attn_varlen_func(x.q, x.k, x.v, x.cu_seqlens, x.cu_seqlens, mx, mx, causal=True)

        try:
            fus = rotating_us([lambda x=x: theirs_p(x) for x in ws])
            line["flash_attn_varlen_us"] = fus
            line["speedup_vs_flash_attn"] = fus / us
        except Exception as e:
            line["flash_attn"] = f"did not run: {type(e).__name__}: {str(e)[:120]}"
    # the reference engine prefills one prompt per step with torch SDPA
    # (model.py:56-57): the 16 prompts as 16 such calls
    views = []
    for x in ws:
        cux = x.cu_seqlens.cpu()
        vx = []
        for s_ in range(16):
            a, b = int(cux[s_]), int(cux[s_ + 1])
            vx.append((x.q[a:b].unsqueeze(0).transpose(1, 2), x.k[a:b].unsqueeze(0).transpose(1, 2),
                       x.v[a:b].unsqueeze(0).transpose(1, 2)))
        views.append(vx)

    def sdpa_all(vx):
        for q_, k_, v_ in vx:
            torch.nn.functional.scaled_dot_product_attention(q_, k_, v_, is_causal=True, enable_gqa=True)

    sus = rotating_us([lambda vx=vx: sdpa_all(vx) for vx in views])
    line["torch_sdpa_per_prompt_us"] = sus
    line["speedup_vs_torch_sdpa"] = sus / us
    out["prefill_b16"] = line
    del ws, w, o, ref, views

    # C3 at B=1: one prompt per call, the reference's own prefill call shape
    # q [1, 16, L, 128] (a transposed view of the [1, L, 16, 128] projection)
    pts = []
    g = torch.Generator(device=dev).manual_seed(31)
    for L in (512, 768, 1024):
        sets = []
        for _ in range(sets_for(L * 32 * 256 + L * 16 * 256)):
            sets.append(tuple(torch.randn(1, L, h, 128, generator=g, device=dev).to(torch.bfloat16).transpose(1, 2)
                              for h in (16, 8, 8)))

        def ours_1(x):
            return pkg.scaled_dot_product_attention(*x, is_causal=True, enable_gqa=True)

        def torch_1(x):
            return torch.nn.functional.scaled_dot_product_attention(*x, is_causal=True, enable_gqa=True)

        us = rotating_us([lambda x=x: ours_1(x) for x in sets])
        tus = rotating_us([lambda x=x: torch_1(x) for x in sets])
        o = ours_1(sets[0])
        qf, kf, vf = (t.float().cpu() for t in sets[0])
        t0 = time.perf_counter()
        ref = torch.nn.functional.scaled_dot_product_attention(qf, kf, vf, is_causal=True, enable_gqa=True)
        cpu_us = (time.perf_counter() - t0) * 1e6
        flops = 2 * 16 * 128 * L * L
        pt = {"L": L, "us": us, "tflops": flops / (us * 1e-6) / 1e12, "torch_sdpa_us": tus,
              "speedup_vs_torch_sdpa": tus / us, "max_abs_err": float((o.float().cpu() - ref).abs().max()),
              "cpu_reference_us": cpu_us, "input_sets": len(sets)}
        if fa is not None:
            cu1 = torch.tensor([0, L], dtype=torch.int32, device=dev)

            def fa_1(x, cu1=cu1, L=L):
                qv, kv, vv = (t.transpose(1, 2)[0] for t in x)
                return fa.flash_attn_varlen_func(qv, kv, vv, cu1, cu1, L, L, causal=True)

            try:
                pt["flash_attn_varlen_us"] = rotating_us([lambda x=x: fa_1(x) for x in sets])
            except Exception as e:
                pt["flash_attn"] = f"did not run: {type(e).__name__}: {str(e)[:120]}"
        pts.append(pt)
        del sets
    out["prefill_b1"] = {"workload": "one prompt per call, q [1,16,L,128] / k,v [1,8,L,128] views of [1,L,H,128] "
                                     "(model.py:56-57), L = 512 / 768 / 1024", "points": pts, "tolerance": 2e-2,
                         "cpu_reference": {**cores, "sample": "fp32 causal SDPA of the same prompt"},
                         "peak_tflops": peak, "peak_source": peak_kind}

    # chunked prefill (row f1): 16 chunks of 512 over cached prefixes U[512,1536]
    cs = [W.chunk_batch(16, 512, 512, 1536, seed=4 + 100 * i, device=dev) for i in range(2)]
    c = cs[0]

    def chunk(x):
        return pkg.flash_attn_with_kvcache(x.q, x.k_cache, x.v_cache, cache_seqlens=x.cache_seqlens,
                                           block_table=x.block_table, causal=True)

    us = rotating_us([lambda x=x: chunk(x) for x in cs])
    flops = sum(x.causal_flops for x in cs) / len(cs)
    o = chunk(c)
    rows = [0, 7, 15]
    qr, kc, vc, bt, L = compact_rows(c.q, c.k_cache, c.v_cache, c.block_table, c.cache_seqlens, rows)
    n = c.q.shape[1]
    cu = torch.arange(0, (len(rows) + 1) * n, n, dtype=torch.int32)
    ref = opa.paged_chunk_prefill(qr.reshape(-1, *qr.shape[2:]), kc, vc, bt, L, cu)
    err = float((o.cpu()[torch.as_tensor(rows)].reshape(-1, *o.shape[2:]).float() - ref).abs().max())
    tf = flops / (us * 1e-6) / 1e12
    out["chunk_prefill_b16"] = {"workload": "16 chunks of 512 tokens over cached prefixes U[512,1536] (paged, "
                                            "256-token blocks, bottom-right causal)",
                                "us": us, "tflops": tf, "peak_tflops": peak, "frac": tf / peak,
                                "peak_source": peak_kind, "flops": flops, "input_sets": len(cs),
                                "max_abs_err": err, "checked_rows": rows, "tolerance": 2e-2}
    del cs, c
    torch.cuda.synchronize()
    pkg.check_device_errors(dev.index)
    return out


def relayout_pool(cache_src, bt_src, cache_dst, bt_dst, ctx):
    """Copy every sequence's cached tokens 0..ctx-1 from one paged pool into
    another of a different block size (block tables bt_src / bt_dst)."""
    bs_s, bs_d = cache_src.block_size, cache_dst.block_size
    src, dst = [], []
    for b in range(bt_src.shape[0]):
        t = torch.arange(int(ctx[b]))
        src.append(bt_src[b, t // bs_s].long() * bs_s + t % bs_s)
        dst.append(bt_dst[b, t // bs_d].long() * bs_d + t % bs_d)
    src, dst = torch.cat(src).to(cache_src.device), torch.cat(dst).to(cache_dst.device)
    for pool_s, pool_d in ((cache_src.k, cache_dst.k), (cache_src.v, cache_dst.v)):
        for layer in range(pool_s.shape[0]):
            s = pool_s[layer].view(-1, *pool_s.shape[3:])
            d = pool_d[layer].view(-1, *pool_d.shape[3:])
            d[dst] = s[src]


def kv_head_sharded_layer(pkg, dist, world, rank, dev, reps, max_over_ranks):
    """The KV-head-sharded partition at `world` GPUs: 128*world requests, each
    rank holding 8/world kv heads of all of them; one 'layer' = the decode
    kernel on the local heads + the all-gather of the [B, 16/world, 128]
    outputs into [B, 16, 128], by NCCL or fused into the decode kernels over
    NVLink. Times are CUDA events, max over ranks. Parity: on every rank the
    fused gather must equal the NCCL gather bit for bit, and this rank's heads
    in it must match the fp32 oracle on 16 sampled rows (max over ranks)."""
    from lean_infer_b200 import sharding as S
    from lean_infer_b200 import workloads as W
    from oracle import paged_attention as opa

    sh = S.kv_head_shard(rank, world, 8, 16)
    B = B_PER_GPU * world
    L = W.seq_lengths(B, CTX_LO, CTX_HI, 500)  # identical on every rank
    bt, nb = W.deal_blocks(L, BLOCK_SIZE, None, 500)
    gen = torch.Generator(device=dev).manual_seed(900 + rank)
    pools = []
    for _ in range(4):  # rotate 4 pools (each > L2) so no layer reads cached KV
        kc = torch.randn((nb, BLOCK_SIZE, sh.num_kv_heads, 128), generator=gen, device=dev).to(torch.bfloat16)
        vc = torch.randn((nb, BLOCK_SIZE, sh.num_kv_heads, 128), generator=gen, device=dev).to(torch.bfloat16)
        pools.append((kc, vc))
    q = torch.randn((B, 1, sh.num_q_heads, 128), generator=gen, device=dev).to(torch.bfloat16)
    seq, btd = L.to(torch.int32).to(dev), bt.to(dev)
    dec = S.KVHeadShardedDecode(sh)
    o_fixed = torch.randn((B, 1, sh.num_q_heads, 128), generator=gen, device=dev).to(torch.bfloat16)

    def attn(i):
        kc, vc = pools[i % 4]
        return pkg.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=seq, block_table=btd, causal=True)

    def timed(fn):
        for i in range(4):
            fn(i)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        dist.barrier()
        return max_over_ranks(e0.elapsed_time(e1) * 1e3 / reps)

    t_layer = timed(lambda i: dec.gather(attn(i)))
    t_attn = timed(attn)
    t_ag = timed(lambda i: dec.gather(o_fixed))

    # The all-gather fused into the decode kernels: peer stores over NVLink
    # plus a per-call epoch, no NCCL call. Timed eagerly and as one captured
    # CUDA graph of `reps` layers (every rank replays the same graph).
    fused = S.NVLinkAllGatherDecode(sh, max_batch=B)

    def fused_layer(i):
        kc, vc = pools[i % 4]
        return fused(q, kc, vc, seq, btd, slot=i % 2)

    def graph_timed(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(reps):
                fn(i)
        t = timed(lambda _i: g.replay()) / reps
        torch.cuda.synchronize()
        del g
        return t

    t_fused = timed(fused_layer)
    t_fused_graph = graph_timed(fused_layer)
    t_attn_graph = graph_timed(attn)
    t_layer_graph = graph_timed(lambda i: dec.gather(attn(i)))  # NCCL all-gather captured too

    # Row f4: the layer up to o_proj's output (model.py:68-69), three ways:
    # NCCL gather + cuBLAS, fused NVLink gather + barrier + cuBLAS, and the
    # fused gather with o_proj on the GEMM that waits for each peer's heads.
    wo = (torch.randn(1024, 16 * 128, generator=torch.Generator().manual_seed(8)) / 2048 ** 0.5)
    wo = wo.to(torch.bfloat16).to(dev)

    def nccl_oproj(i):
        return torch.nn.functional.linear(dec.gather(attn(i)).view(B, 16 * 128), wo)

    def fused_barrier_oproj(i):
        return torch.nn.functional.linear(fused_layer(i).view(B, 16 * 128), wo)

    def fused_oproj(i):
        kc, vc = pools[i % 4]
        return fused.attention_o_proj(q, kc, vc, seq, btd, wo, slot=i % 2)

    t_op_nccl = graph_timed(nccl_oproj)
    t_op_barrier = graph_timed(fused_barrier_oproj)
    t_op_fused = graph_timed(fused_oproj)
    y_ref = nccl_oproj(0).clone()
    y_fused = fused_oproj(0).clone()
    torch.cuda.synchronize()
    dist.barrier()
    ys = [torch.empty_like(y_fused) for _ in range(world)]
    dist.all_gather(ys, y_fused)
    y_same = all(torch.equal(ys[0], y) for y in ys)
    y_err = max_over_ranks(float((y_fused.float() - y_ref.float()).abs().max()))
    y_scale = float(y_ref.float().abs().max())

    # parity, pool 0, both forms on every rank
    o_nccl = dec.gather(attn(0)).clone()
    o_fused = fused_layer(0).clone()
    torch.cuda.synchronize()
    dist.barrier()
    same = bool(torch.equal(o_nccl, o_fused))
    fused_vs_nccl = float((o_nccl.float() - o_fused.float()).abs().max())
    Lc = L.to(torch.int32)
    rows = sorted(set(torch.randperm(B, generator=torch.Generator().manual_seed(77))[:14].tolist())
                  | {int(Lc.argmax()), int(Lc.argmin())})
    kc, vc = pools[0]
    qr, kcr, vcr, btr, Lr = compact_rows(q, kc, vc, btd, seq, rows)
    ref = opa.paged_decode(qr, kcr, vcr, btr, Lr)  # this rank's heads only
    mine = o_fused[torch.as_tensor(rows, device=dev)][:, :, sh.q_lo:sh.q_hi].float().cpu()
    err_fused = max_over_ranks(float((mine - ref).abs().max()))
    mine = o_nccl[torch.as_tensor(rows, device=dev)][:, :, sh.q_lo:sh.q_hi].float().cpu()
    err_nccl = max_over_ranks(float((mine - ref).abs().max()))
    n_diff = max_over_ranks(0.0 if same else 1.0)
    fused.close()
    kv_total = int(L.sum()) * 8 * 128 * 2 * 2
    pkg.check_device_errors(dev.index)
    best = min(t_layer, t_layer_graph, t_fused, t_fused_graph)
    return {"requests": B, "kv_heads_per_gpu": sh.num_kv_heads, "us_per_layer": best,
            "nccl_us_per_layer": t_layer, "nccl_graph_us_per_layer": t_layer_graph,
            "decode_us": t_attn, "allgather_us": t_ag,
            "decode_graph_us": t_attn_graph,
            "fused_nvlink_us_per_layer": t_fused, "fused_nvlink_graph_us_per_layer": t_fused_graph,
            "allgather_bytes_per_gpu": B * sh.num_q_heads * 128 * 2,
            "kv_gbs_total": kv_total / (best * 1e-6) / 1e9,
            "kv_gbs_per_gpu_decode": kv_total / world / (t_attn_graph * 1e-6) / 1e9,
            "tok_per_s_attention_only": B / (best * 28 * 1e-6),
            "o_proj": {"nccl_cublas_us_per_layer": t_op_nccl, "fused_gather_barrier_cublas_us_per_layer": t_op_barrier,
                       "fused_gather_o_proj_us_per_layer": t_op_fused,
                       "max_abs_diff_vs_nccl_cublas": y_err, "y_max_abs": y_scale,
                       "identical_on_all_ranks": y_same,
                       "what": "decode + all-gather + o_proj [B,2048]x[2048,1024] per layer, graph-captured"},
            "parity": {"max_abs_err_fused": err_fused, "max_abs_err_nccl": err_nccl,
                       "fused_equals_nccl_all_ranks": n_diff == 0.0, "fused_vs_nccl_max_abs": fused_vs_nccl,
                       "checked_rows_per_rank": len(rows), "tolerance": 2e-2,
                       "oracle": "fp32 paged decode over each rank's own kv heads"}}


def measured_peak_bf16():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    return 1590.0, "fallback"


def run_reference(args):
    rank = env_int("RANK", 0)
    if rank != 0:
        return
    r = cpu_reference_run(args.steps, args.warmup)
    out = {
        "metric": METRIC, "value": r["value"], "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": DATA,
        "config": bench_config(args.gpus),
        "impl": "reference",
        "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": r["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def step_bs16(pkg, model, cache, dg, ids, pos, bt, ctx, dev, steps, order="random"):
    """Row f2 end to end: the same decode step over a pool of 16-token blocks
    (same token capacity, the same cached tokens copied into it), timed like
    the headline; parity = its logits against the 256-token-block step's.
    order: "random" deals the blocks from a seeded permutation of the pool
    (as the 256-token step does), "fifo" in allocator order (each sequence's
    blocks one after another, as a fresh BlockAllocator hands them out)."""
    from lean_infer_b200 import qwen3
    from lean_infer_b200 import workloads as W
    from lean_infer_b200.cache import BlockCache

    cfg = model.config
    nb16 = NUM_BLOCKS * BLOCK_SIZE // 16
    cache16 = BlockCache(cfg.num_hidden_layers, nb16, 16, cfg.num_key_value_heads, cfg.head_dim, dev, zero=False)
    if order == "random":
        bt16, _ = W.deal_blocks(ctx.long(), 16, nb16, 123)
    else:
        need = [-(-int(n) // 16) for n in ctx]
        bt16 = torch.zeros(len(need), max(need), dtype=torch.int32)
        o = 1
        for b, n in enumerate(need):
            bt16[b, :n] = torch.arange(o, o + n, dtype=torch.int32)
            o += n
    relayout_pool(cache, bt, cache16, bt16, ctx)
    dg16 = qwen3.DecodeGraph(model, cache16, B_PER_GPU, -(-CTX_HI // 16))
    dg16.stage(ids, pos, bt16, ctx)
    dg16.upload()
    dg16.capture()
    for _ in range(3):
        dg16.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        dg16.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    # parity: one more step of each graph on identical inputs
    dg.stage(ids, pos, bt, ctx)
    dg.upload()
    dg.replay()
    dg16.replay()
    torch.cuda.synchronize()
    a, b = dg16.logits[:, 0].detach().float(), dg.logits[:, 0].detach().float()
    err = float((a - b).abs().max())
    agree = float((dg16.next_tokens == dg.next_tokens).float().mean())
    pkg.check_device_errors(dev.index)
    dg16.release()
    del cache16
    return {"workload": WORKLOAD.replace("512x256-token", "8192x16-token") + f", blocks in {order} order",
            "ms_per_step": ms, "tok_per_s": B_PER_GPU / (ms / 1e3), "logits_max_abs_diff_vs_bs256": err,
            "next_token_agreement_vs_bs256": agree}


def run_ours(args):
    import __graft_entry__

    pkg = __graft_entry__.load_package()
    from lean_infer_b200 import qwen3
    from lean_infer_b200.cache import BlockCache

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    cfg = qwen3.ModelConfig()
    model = qwen3.random_model(cfg, dev, seed=1234)
    cache = BlockCache(cfg.num_hidden_layers, NUM_BLOCKS, BLOCK_SIZE, cfg.num_key_value_heads, cfg.head_dim, dev,
                       zero=False)
    gen = torch.Generator(device=dev).manual_seed(77 + rank)
    for t in (cache.k, cache.v):
        flat = t.view(-1)
        step = 1 << 28
        for i in range(0, flat.numel(), step):
            n = min(step, flat.numel() - i)
            flat[i:i + n] = torch.randn(n, generator=gen, device=dev)
    ids, pos, bt, ctx = synth_inputs(rank)
    max_blocks = -(-CTX_HI // BLOCK_SIZE)
    dg = qwen3.DecodeGraph(model, cache, B_PER_GPU, max_blocks)
    dg.stage(ids, pos, bt, ctx)
    dg.upload()
    dg.capture()
    torch.cuda.synchronize()
    pkg.check_device_errors(local)

    # ---------------------------------------------------------------- value
    for _ in range(args.warmup):
        dg.replay()
    torch.cuda.synchronize()
    # per layer: fused pre-attention, decode, combine, two add+RMSNorm, SiLU*mul;
    # plus the first layer's input RMSNorm and the greedy-token argmax
    launches_per_step = cfg.num_hidden_layers * 6 + 2
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            dg.replay()
        e1.record()
        torch.cuda.synchronize()
        barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    value = world * B_PER_GPU / (ms / 1e3)

    # ---------------------------------------------------------------- e2e
    for _ in range(max(1, args.warmup // 2)):
        dg.step()
    barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        dg.stage(ids, pos, bt, ctx)
        toks = dg.step()  # H2D copies, replay, D2H of the next tokens (syncs)
    t1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(t0.elapsed_time(t1) / args.steps)
    assert len(toks) == B_PER_GPU
    d2h = B_PER_GPU * 8

    # ---------------------------------------------------------------- roofline
    # The decode attention op alone over the 28 layer caches (q from the
    # workload's distribution), captured in a graph, CUDA events on its stream.
    qs = [torch.randn(B_PER_GPU, 1, cfg.num_attention_heads, cfg.head_dim, device=dev).to(torch.bfloat16)
          for _ in range(cfg.num_hidden_layers)]
    d_bt, d_ctx = dg.bt, dg.ctx

    def attn_all():
        for li in range(cfg.num_hidden_layers):
            pkg.flash_attn_with_kvcache(qs[li], cache.k[li], cache.v[li], cache_seqlens=d_ctx, block_table=d_bt,
                                        causal=True, num_splits=1)

    attn_all()
    g_attn = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_attn):
        attn_all()
    for _ in range(2):
        g_attn.replay()
    torch.cuda.synchronize()
    reps = max(2, args.steps // 2)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    for _ in range(reps):
        g_attn.replay()
    a1.record()
    torch.cuda.synchronize()
    pkg.check_device_errors(local)
    us_per_launch = max_over_ranks(a0.elapsed_time(a1) * 1e3 / (reps * cfg.num_hidden_layers))
    kv_bytes = int(ctx.long().sum()) * cfg.num_key_value_heads * cfg.head_dim * 2 * 2
    qo_bytes = 2 * B_PER_GPU * cfg.num_attention_heads * cfg.head_dim * 2
    alg_bytes = kv_bytes + qo_bytes
    achieved = alg_bytes / (us_per_launch * 1e-6) / 1e9
    peak, peak_kind = measured_peak_hbm()
    del g_attn

    bs16 = None
    if world == 1 and not args.no_secondary:
        bs16 = {o: step_bs16(pkg, model, cache, dg, ids, pos, bt, ctx, dev, max(3, args.steps), order=o)
                for o in ("random", "fifo")}
        bs16["bs256_ms_per_step"] = ms
    dg.release()

    result = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": DATA,
        "config": bench_config(world),
        "e2e": {"value": world * B_PER_GPU / (e2e_ms / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": dg.h2d_bytes, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": {"bound": "hbm", "kernel": "paged decode attention (la_paged_decode: decode + combine)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6650 GB/s",
                     "traffic": None, "alg_bytes_per_launch": alg_bytes,
                     "us_per_launch": us_per_launch},
        "clocks": clk.summary(),
    }
    del cache, model, qs
    torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not args.no_secondary:
        result["secondary"] = secondary_metrics(pkg, dev)
        result["secondary"]["step_bs16"] = bs16
    if world > 1:
        dist.barrier()
        result["kv_head_sharded"] = kv_head_sharded_layer(pkg, dist, world, rank, dev, max(8, args.steps // 10),
                                                          max_over_ranks)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = cpu_reference_run(args.cpu_steps, 1)
        result["cpu_baseline"] = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_case(args):
    """Single-kernel cases for profilers (ncu): run one op a few times on a
    small, fixed input and exit. --case decode-b128 | decode-c1 | decode-kvshard8 | o-proj | decode-long |
    prefill-b16 | prefill-b1 | prefill-long | chunk-prefill-b16 | pre-attn-b128."""
    import __graft_entry__

    pkg = __graft_entry__.load_package()
    from lean_infer_b200 import workloads as W

    dev = torch.device("cuda", 0)
    reps = 3
    if args.case in ("decode-b128", "decode-long", "decode-c1"):
        if args.case == "decode-b128":  # one layer of the benchmark step: 408 MB of KV, > L2
            w = W.decode_batch(128, CTX_LO, CTX_HI, num_blocks=NUM_BLOCKS, block_size=BLOCK_SIZE, seed=1, device=dev)
        elif args.case == "decode-c1":  # B=8, one layer, 512x256 pool
            w = W.decode_batch(8, CTX_LO, CTX_HI, num_blocks=NUM_BLOCKS, block_size=BLOCK_SIZE, seed=11, device=dev)
        else:  # B=32, contexts U[8192, 32768]
            w = W.decode_batch(32, 8192, 32768, num_blocks=None, block_size=BLOCK_SIZE, seed=40, device=dev)
        for _ in range(reps):
            pkg.flash_attn_with_kvcache(w.q, w.k_cache, w.v_cache, cache_seqlens=w.cache_seqlens,
                                        block_table=w.block_table, causal=True)
        info = {"kv_bytes": w.kv_bytes}
    elif args.case in ("prefill-b16", "prefill-b1", "prefill-long"):
        if args.case == "prefill-long":  # 4 prompts of 8192 tokens: the steady state of the kernel
            w = W.prefill_batch(4, 8192, 8192, seed=5, device=dev)
        else:
            w = W.prefill_batch(16 if args.case == "prefill-b16" else 1, CTX_LO, CTX_HI, seed=3, device=dev)
        mx = int(w.lengths.max())
        for _ in range(reps):
            pkg.flash_attn_varlen_func(w.q, w.k, w.v, w.cu_seqlens, w.cu_seqlens, mx, mx, causal=True)
        info = {"causal_flops": w.causal_flops}
    elif args.case == "chunk-prefill-b16":  # 16 chunks of 512 over cached prefixes U[512, 1536]
        c = W.chunk_batch(16, 512, 512, 1536, seed=4, device=dev)
        for _ in range(reps):
            pkg.flash_attn_with_kvcache(c.q, c.k_cache, c.v_cache, cache_seqlens=c.cache_seqlens,
                                        block_table=c.block_table, causal=True)
        info = {"causal_flops": c.causal_flops}
    elif args.case == "o-proj":  # the gathered o_proj of the KV-head-sharded layer, world = 1: B=1024 and 256
        from lean_infer_b200 import _lib
        from lean_infer_b200 import flash_attn_interface as fai

        lib = _lib.load()
        fai.ensure_init(0)
        g = torch.Generator(device=dev).manual_seed(6)
        w_o = (torch.randn(1024, 2048, generator=g, device=dev) / 45).to(torch.bfloat16)
        sig = torch.zeros(8, dtype=torch.int32, device=dev)
        err = fai.error_word(0)
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        for m in (1024, 256):
            a = torch.randn(m, 2048, generator=g, device=dev).to(torch.bfloat16)
            o = torch.empty(m, 1024, dtype=torch.bfloat16, device=dev)
            for _ in range(reps):
                rc = lib.la_o_proj_gathered(ctypes.c_void_p(a.data_ptr()), 2048, ctypes.c_void_p(w_o.data_ptr()), 2048,
                                            ctypes.c_void_p(o.data_ptr()), 1024, m, 1024, 2048,
                                            ctypes.c_void_p(sig.data_ptr()), 1, 0, ctypes.c_void_p(err.data_ptr()),
                                            stream)
                assert rc == 0
        info = {"flops": 2 * 1280 * 1024 * 2048}
    elif args.case == "decode-kvshard8":  # one rank of the KV-head-sharded partition at 8 GPUs
        L = W.seq_lengths(1024, CTX_LO, CTX_HI, 500)
        w = W.decode_batch(1024, CTX_LO, CTX_HI, num_blocks=None, block_size=BLOCK_SIZE, num_q_heads=2,
                           num_kv_heads=1, seed=500, device=dev, lengths=L)
        for _ in range(reps):
            pkg.flash_attn_with_kvcache(w.q, w.k_cache, w.v_cache, cache_seqlens=w.cache_seqlens,
                                        block_table=w.block_table, causal=True)
        info = {"kv_bytes": w.kv_bytes}
    elif args.case == "pre-attn-b128":
        from lean_infer_b200 import qwen3

        L = W.seq_lengths(128, CTX_LO, CTX_HI, 0)
        bt, nb = W.deal_blocks(L, BLOCK_SIZE, NUM_BLOCKS, 0)
        qkv = torch.randn(128, 4096, device=dev).to(torch.bfloat16)
        kc = torch.zeros(nb, BLOCK_SIZE, 8, 128, dtype=torch.bfloat16, device=dev)
        vc = torch.zeros_like(kc)
        cos, sin = pkg.rope_tables(4096, 128, 1e6, dev)
        w1 = torch.ones(128, dtype=torch.bfloat16, device=dev)
        for _ in range(reps):
            pkg.qk_norm_rope_paged_write(qkv[:, :2048].view(128, 16, 128), qkv[:, 2048:3072].view(128, 8, 128),
                                         qkv[:, 3072:].view(128, 8, 128), w1, w1, cos, sin, (L - 1).to(dev),
                                         bt.to(dev), kc, vc)
        info = {"tokens": 128}
    else:
        raise SystemExit(f"unknown case {args.case}")
    torch.cuda.synchronize()
    pkg.check_device_errors(0)
    print(json.dumps({"case": args.case, **info}), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-steps", type=int, default=5, help="timed CPU steps for cpu_baseline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="skip the per-kernel lines and the BS=16 step")
    ap.add_argument("--case", default=None, help="run one kernel case for a profiler and exit")
    args = ap.parse_args()
    if args.case:
        run_case(args)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
