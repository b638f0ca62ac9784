#!/usr/bin/env python3
"""Benchmark of the vx27 attention hot path on B200: BASELINE.json's metric
"DeltaNet+GQA decode tokens/s at 1/2/4/8 B200; % of HBM roofline" on its config 2
(batched hybrid decode step: 48 Gated DeltaNet + 16 gated GQA layers, 256 sequences per
GPU, BF16 KV cache of 4096 tokens per layer, 64 decode steps, seed 2).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1). Every rank holds its own 256 sequences (weak
scaling, no collective on the data path). Timing: W untimed steps, then K steps between a
barrier + cuda synchronize, CUDA events on the launching stream, max over ranks. The
resident working set (~84 GB per GPU) is far larger than L2, so no flush is needed.
Rank 0 prints one JSON line.

--impl reference times the reference's own CPU implementation of the same step
(oracle/_ref, compiled from the reference's sources; the oracle port if absent) on the
host cores, on a bounded sample of sequences per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "DeltaNet+GQA decode tokens/s at 1/2/4/8 B200; % of HBM roofline"
# DRAM bytes (read + write) per algorithmic byte of the split-KV GQA decode kernel, from
# ncu captures of the same kernel for one layer at 64 sequences (the full 256-sequence
# workload holds 83 GB, too much to profile): each K/V byte is read once; the last tile of
# every (sequence, KV head) fetches only the 32-row boxes it needs; the fused variant also
# writes the new K/V rows.
GQA_SPLIT_DRAM_PER_ALGO_BYTE = {True: 1.016, False: 1.010}  # keyed by the fused prologue
FALLBACK_HBM_GBS = 6650.0


def peaks() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback 6.65 TB/s"


def tensor_peak() -> tuple[float, str]:
    """Dense bf16 tensor peak for a kernel timed alone (the burst figure)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops)"
    except Exception:
        return 1590.0, "fallback 1.59 PFLOP/s"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples every 200 ms while the timed region runs. Started before the
    warm-up, with begin() / end() marking the timed region on the host clock, the summary
    keeps the samples taken inside it (or, for a region shorter than the sampling period,
    the samples within 0.5 s of it)."""
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.t_begin = self.t_end = None

    def begin(self) -> None:
        self.t_begin = time.time()

    def end(self) -> None:
        self.t_end = time.time()

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-i", str(self.idx), "-lms", "200"], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def _rows(self) -> list:
        import datetime
        rows = []
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            try:
                t = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((t, float(f[2]), float(f[3]), f[6:10]))
            except (ValueError, IndexError):
                continue
        return rows

    def summary(self) -> dict:
        rows, window = self._rows(), "timed region"
        if self.t_begin is not None and self.t_end is not None:
            inside = [r for r in rows if self.t_begin <= r[0] <= self.t_end]
            if not inside:
                inside = [r for r in rows if self.t_begin - 0.5 <= r[0] <= self.t_end + 0.5]
                window = "within 0.5 s of the timed region (shorter than the 200 ms period)"
            rows = inside
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = {n for r in rows for n, v in zip(names, r[3]) if v.lower() == "active"}
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(r[1] for r in rows),
                "sm_max_mhz": max(r[2] for r in rows), "reasons": sorted(reasons),
                "samples": len(rows), "window": window}


# ---------------------------------------------------------------- our arm
def run_ours(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch
    import torch.distributed as dist
    from vx27_b200.hybrid import HybridConfig, HybridDecoder, N_FULL, N_LIN

    torch.cuda.set_device(local_rank)
    cfg = HybridConfig(batch=args.batch, ctx=args.ctx, steps=args.warmup + args.steps + 2,
                       fused_gqa=args.fused_gqa,
                       seed=2 + rank * 1000)
    dec = HybridDecoder(cfg)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # warm-up, then the device-resident timed region; the clock sampler starts before the
    # warm-up so that it is running when the timed region begins
    clk = ClockSampler(local_rank if "CUDA_VISIBLE_DEVICES" not in os.environ
                       else int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local_rank]))
    clk.__enter__()
    for _ in range(args.warmup):
        dec.step()
    barrier()
    ev = {"dn": [], "gqa": []}
    kinds = {"gqa"}

    # Events bracket the GQA split kernel (the roofline kernel) in the timed region. The
    # DeltaNet kernels start while their predecessor drains (programmatic dependent launch),
    # which an event between them would prevent, so their per-launch time is taken from two
    # extra steps after the timed region.
    def on_layer(kind, i, phase):
        if kind not in kinds:
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        ev[kind].append(e)

    ctx0 = int(dec.pos[0].item())
    clk.begin()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    launches = 0
    for _ in range(args.steps):
        launches += dec.step(on_layer=on_layer)
    t1.record(stream)
    barrier()
    clk.end()
    clk.__exit__(None, None, None)
    ms = t0.elapsed_time(t1)
    if world > 1:
        tt = torch.tensor([ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    ms_step = ms / args.steps
    kinds.clear()
    kinds.add("dn")
    for _ in range(2):
        dec.step(on_layer=on_layer)
    barrier()

    def avg_ms(kind):
        e = ev[kind]
        return sum(e[2 * j].elapsed_time(e[2 * j + 1]) for j in range(len(e) // 2)) / (len(e) // 2)

    # attended positions per step average (positions 0..pos inclusive)
    ctx_avg = ctx0 + 1 + (args.steps - 1) / 2.0
    by = dec.bytes_per_step(ctx_avg)
    c = cfg
    if args.fused_gqa:  # the fused kernel: K/V, q/k/v in, gate, out, the new K/V rows
        gqa_bytes = (by["kv"] + by["gqa_act"]) / N_FULL
    else:  # the split kernel: K/V, the normalised fp32 q, gate and out
        gqa_bytes = by["kv"] / N_FULL + c.batch * c.nq * c.hd * (4 + 2 + 2)
    dn_bytes = (by["dn_state"] + by["dn_conv"] + by["dn_act"]) / N_LIN
    peak, peak_src = peaks()
    gqa_ms, dn_ms = avg_ms("gqa"), avg_ms("dn")
    gqa_gbs = gqa_bytes / (gqa_ms * 1e-3) / 1e9
    dn_gbs = dn_bytes / (dn_ms * 1e-3) / 1e9
    step_gbs = by["total"] / (ms_step * 1e-3) / 1e9

    # end-to-end through the public API with host buffers: every step copies its
    # activations in from pinned host memory and its attention outputs back (per layer,
    # overlapped with the other layers' kernels), all inside the timed region
    hin = [t.cpu().pin_memory() for t in dec.step_inputs()]
    hout = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in dec.step_outputs()]
    h2d = sum(t.numel() * t.element_size() for t in hin)
    d2h = sum(t.numel() * t.element_size() for t in hout)

    def e2e_step():
        return dec.step_host(hin, hout)

    dec.reset_positions()
    for _ in range(args.warmup):
        e2e_step()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        tt = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())

    from vx27_b200 import ops
    status = ops.device_status()
    if rank != 0:
        return None
    tokens = c.batch * world * args.steps
    return {
        "metric": METRIC,
        "value": round(tokens / (ms * 1e-3), 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded splitmix64 + Box-Muller, config 2 distributions)",
        "config": {
            "workload": "config 2: batched hybrid decode step, 48 Gated DeltaNet + 16 gated GQA "
                        "layers (3:1 order), hd 128 / 24Q-4KV hd 256, BF16 KV cache",
            "batch_per_gpu": c.batch, "global_batch": c.batch * world,
            "ctx_at_first_step": ctx0 + 1, "decode_steps": args.steps,
            "state": "fp32 S ~N(0,0.05); KV bf16 ~N(0,1); activations bf16 ~N(0,1)",
            "l2": "inputs larger than L2 (resident working set %.1f GB/GPU)" %
                  (sum(t.numel() * t.element_size() for t in (dec.S, dec.ring, dec.kc, dec.vc))
                   / 1e9),
            "parallelism": f"dp{world} (sequences sharded, no collective)",
            "gqa_layer": ("one fused kernel (vx27_gqa_decode_fused)" if args.fused_gqa
                          else "vx27_gqa_append + vx27_gqa_decode_batch"),
        },
        "roofline": {
            "bound": "hbm",
            "kernel": ("gqa_split_tc split-KV decode" +
                       (" with the QK norm, RoPE and K/V append fused in" if args.fused_gqa
                        else "") +
                       ", per layer (one split: it writes the gated output itself, no "
                       "combine pass)"),
            "achieved": round(gqa_gbs, 1), "peak": peak, "unit": "GB/s",
            "frac": round(gqa_gbs / peak, 4),
            "traffic": int(GQA_SPLIT_DRAM_PER_ALGO_BYTE[args.fused_gqa] * gqa_bytes),
            "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of gqa_split_tc "
                               "for one layer at B = 64 (same kernel and per-sequence context; "
                               f"{GQA_SPLIT_DRAM_PER_ALGO_BYTE[args.fused_gqa]} x its algorithmic "
                               "bytes), scaled by the sequences of this launch"),
            "peak_source": peak_src,
            "algorithmic_bytes_per_launch": int(gqa_bytes), "avg_launch_ms": round(gqa_ms, 4),
        },
        "roofline_other": {
            "deltanet_decode": {"achieved": round(dn_gbs, 1), "frac": round(dn_gbs / peak, 4),
                                "algorithmic_bytes_per_launch": int(dn_bytes),
                                "avg_launch_ms": round(dn_ms, 4)},
            "whole_step": {"achieved": round(step_gbs, 1), "frac": round(step_gbs / peak, 4),
                           "algorithmic_bytes_per_step": int(by["total"]),
                           "frac_of_nominal_8TBps": round(step_gbs / 8000.0, 4)},
        },
        "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms / args.steps, 4)},
        "gpu_launches": launches,
        "device_status": status,
        "clocks": clk.summary(),
    }


# ------------------------------------------------- single-layer workloads
def run_layer(args) -> dict:
    """One attention layer launched repeatedly (kernel rooflines in isolation and ncu
    captures at a chosen size): --workload dn_layer | gqa_layer."""
    import torch
    from vx27_b200 import ops
    torch.cuda.set_device(0)
    B = args.batch
    peak, peak_src = peaks()
    bf = torch.bfloat16
    if args.workload == "dn_layer":
        nqk = nv = 16
        C = (2 * nqk + nv) * 128
        S = torch.empty(B, nv, 128, 128, device="cuda")
        ring = torch.empty(B, 4, C, device="cuda")
        qkv = torch.empty(B, C, dtype=bf, device="cuda")
        a = torch.empty(B, nv, dtype=bf, device="cuda")
        b = torch.empty(B, nv, dtype=bf, device="cuda")
        w = torch.empty(C, 4, device="cuda")
        A = torch.empty(nv, device="cuda")
        dt = torch.empty(nv, device="cuda")
        o = torch.empty(B, nv, 128, dtype=bf, device="cuda")
        for n, t in enumerate((S, ring, qkv, a, b, w, dt)):
            ops.fill_normal(t, 2, n, 0.0, 0.05 if n == 0 else 1.0)
        ops.fill_uniform(A, 2, 9, 1.0, 16.0)
        A.log_()
        pos = torch.full((B,), args.ctx, dtype=torch.int32, device="cuda")
        run = lambda: ops.deltanet_decode_batch(S, ring, qkv, a, b, A, dt, w, pos, o, nqk, nv)
        nbytes = B * nv * 128 * 128 * 4 * 2 + B * C * (16 + 2) + B * nv * 128 * 2
        name = "dn_decode_k (fused DeltaNet decode), one layer"
    else:
        nq, nkv, hd, cap = 24, 4, 256, args.ctx + 1
        kc = torch.empty(B, nkv, cap, hd, dtype=bf, device="cuda")
        vc = torch.empty(B, nkv, cap, hd, dtype=bf, device="cuda")
        q = torch.empty(B, nq, hd, device="cuda")
        gate = torch.empty(B, nq, hd, dtype=bf, device="cuda")
        out = torch.empty(B, nq, hd, dtype=bf, device="cuda")
        for n, t in enumerate((kc, vc, q, gate)):
            ops.fill_normal(t, 3, n)
        ws = torch.empty(ops.gqa_workspace_bytes(B, nq, nkv, hd, cap) // 4 + 1, device="cuda")
        pos = torch.full((B,), args.ctx, dtype=torch.int32, device="cuda")
        if args.fused_gqa:  # the fused kernel, as the config 2 step runs it
            q_in = torch.empty(B, nq, hd, dtype=bf, device="cuda")
            k_in = torch.empty(B, nkv, hd, dtype=bf, device="cuda")
            v_in = torch.empty_like(k_in)
            for n, t in enumerate((q_in, k_in, v_in)):
                ops.fill_normal(t, 3, 10 + n)
            qw = torch.ones(hd, device="cuda")
            kw = torch.ones(hd, device="cuda")
            rope = ops.rope_table(cap)
            run = lambda: ops.gqa_decode_fused(q_in, k_in, v_in, qw, kw, rope, gate, kc, vc, pos,
                                               out, ws)
            nbytes = B * nkv * cap * hd * 2 * 2 + B * (nq * hd * 2 * 3 + 2 * nkv * hd * 2 * 2)
            name = ("gqa_split_tc with the QK norm, RoPE and K/V append fused in (one split "
                    "writes the gated output), one layer")
        else:
            run = lambda: ops.gqa_decode_batch(q, gate, kc, vc, pos, out, ws)
            nbytes = B * nkv * cap * hd * 2 * 2 + B * nq * hd * (4 + 2 + 2)
            name = "gqa_split_tc (split-KV decode; one split writes the gated output), one layer"
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"workload": args.workload, "kernel": name, "batch": B, "ctx": args.ctx,
            "ms_per_launch": round(ms, 4), "algorithmic_bytes_per_launch": nbytes,
            "achieved_GBps": round(gbs, 1), "peak": peak, "frac": round(gbs / peak, 4),
            "peak_source": peak_src}


# ------------------------------------------------- K5: projection matvecs
PMAT_SHAPES = [  # (projection, rows, cols) of one layer (src/vx27_qfwd.c:97-213, H = 5120)
    ("deltanet.in_proj_qkv", 10240, 5120), ("deltanet.in_proj_z", 6144, 5120),
    ("deltanet.in_proj_a", 48, 5120), ("deltanet.in_proj_b", 48, 5120),
    ("deltanet.out_proj", 5120, 6144), ("gqa.q_proj", 12288, 5120), ("gqa.k_proj", 1024, 5120),
    ("gqa.v_proj", 1024, 5120), ("gqa.o_proj", 5120, 6144)]


PMAT_GROUPS = {"deltanet": ["deltanet.in_proj_qkv", "deltanet.in_proj_z", "deltanet.in_proj_a",
                              "deltanet.in_proj_b"],
               "gqa": ["gqa.q_proj", "gqa.k_proj", "gqa.v_proj"]}


def bp3_weights(rows: int, cols: int, n_copy: int):
    """n_copy copies of random BP3_128 rows (3-bit codes uniform, fp16 scale 0.0200)."""
    import torch
    from vx27_b200 import ops
    rb = ops.pmat_row_bytes(ops.PMAT_BP3_128, cols)
    W = torch.randint(0, 256, (n_copy, rows * rb), dtype=torch.uint8, device="cuda")
    g = W.view(-1, 52)
    g[:, 48:50] = torch.tensor([0x1F, 0x25], dtype=torch.uint8, device="cuda")
    g[:, 50:52] = 0
    return W


def graph_us(go, reps: int, warmup: int) -> float:
    """Device time per call of go(i), i = 0..reps-1, captured as one CUDA graph and replayed
    (so the host's per-call argument checks stay out of the figure)."""
    import torch
    for i in range(max(3, warmup)):
        go(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(reps):
            go(i)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(3):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (3 * reps)
    del graph
    return us


def time_pmat_group(names, B: int, args) -> dict:
    """A layer's input projections of the same x as one launch (vx27_pmat_multi_dev), each
    weight set cycled through >= 512 MB of copies in all."""
    import torch
    from vx27_b200 import ops
    shp = {n: (r, c) for n, r, c in PMAT_SHAPES}
    rows = [shp[n][0] for n in names]
    cols = shp[names[0]][1]
    rb = ops.pmat_row_bytes(ops.PMAT_BP3_128, cols)
    wbytes = sum(rows) * rb
    n_copy = max(2, -(-512 * 2**20 // wbytes))
    Ws = [bp3_weights(r, cols, n_copy) for r in rows]
    x = torch.randn(B, cols, device="cuda")
    ys = [torch.empty(B, r, device="cuda") for r in rows]

    def go(i):
        ops.pmat_multi([W[i % n_copy] for W in Ws], ops.PMAT_BP3_128, x, ys, rows, cols)
    us = graph_us(go, max(args.steps, 2 * n_copy), args.warmup)
    return {"projections": names, "tokens": B, "us": round(us, 2), "weight_bytes": wbytes,
            "GBps": round(wbytes / (us * 1e-6) / 1e9, 1)}


def run_pmat(args) -> dict:
    """Packed BP3_128 weights (random codes, fp16 scale 0.02), the projection shapes of one
    DeltaNet and one GQA layer, B = 1 and 8 tokens. Each shape cycles through enough copies
    of its weights (>= 512 MB) that every call reads them from HBM, not L2; the calls are
    timed replayed from a CUDA graph. Per layer: the projections one launch each, and the
    input projections grouped into one launch."""
    import torch
    from vx27_b200 import ops
    peak, peak_src = peaks()
    per = []
    for B in (1, 8):
        for name, rows, cols in PMAT_SHAPES:
            rb = ops.pmat_row_bytes(ops.PMAT_BP3_128, cols)
            wbytes = rows * rb
            n_copy = max(2, -(-512 * 2**20 // wbytes))
            W = bp3_weights(rows, cols, n_copy)
            x = torch.randn(B, cols, device="cuda")
            y = torch.empty(B, rows, device="cuda")
            us = graph_us(lambda i: ops.pmat_batch(W[i % n_copy], ops.PMAT_BP3_128, x, y, rows,
                                                   cols), max(args.steps, 2 * n_copy), args.warmup)
            gbs = (wbytes + B * (rows + cols) * 4) / (us * 1e-6) / 1e9
            per.append({"projection": name, "rows": rows, "cols": cols, "tokens": B,
                        "us": round(us, 2), "weight_bytes": wbytes, "GBps": round(gbs, 1),
                        "frac": round(gbs / peak, 4),
                        "weights_per_s_T": round(rows * cols / (us * 1e-6) / 1e12, 3)})
            del W
    layer = {}
    for B in (1, 8):
        for kind in ("deltanet", "gqa"):
            sel = [r for r in per if r["tokens"] == B and r["projection"].startswith(kind)]
            us = sum(r["us"] for r in sel)
            wb = sum(r["weight_bytes"] for r in sel)
            layer[f"{kind}_B{B}"] = {"us": round(us, 1), "GBps": round(wb / (us * 1e-6) / 1e9, 1),
                                     "frac": round(wb / (us * 1e-6) / 1e9 / peak, 4)}
            grp = time_pmat_group(PMAT_GROUPS[kind], B, args)
            out = [r for r in sel if r["projection"] not in PMAT_GROUPS[kind]]
            gus = grp["us"] + sum(r["us"] for r in out)
            layer[f"{kind}_B{B}_grouped"] = {
                "us": round(gus, 1), "input_projections_us": grp["us"],
                "GBps": round(wb / (gus * 1e-6) / 1e9, 1),
                "frac": round(wb / (gus * 1e-6) / 1e9 / peak, 4)}
    cpu = None
    if not args.no_cpu_baseline:
        cpu = pmat_cpu_baseline()
    return {"metric": "projection matvec weight GB/s (BP3_128 packed weights, K5)",
            "workload": "pmat", "value": layer["deltanet_B1_grouped"]["GBps"], "unit": "GB/s",
            "n_gpus": 1, "higher_is_better": True, "dtype": "f32 (packed 3.25-bit weights)",
            "data": "synthetic (random 3-bit codes, fp16 scale 0.02; x ~N(0,1))",
            "config": {"workload": "projections of one DeltaNet and one GQA layer, H = 5120",
                       "l2": "weights cycled through >= 512 MB of copies",
                       "timing": "CUDA events around replays of a graph of the calls"},
            "roofline": {"bound": "hbm (weights) / CUDA-core unpack", "peak": peak,
                         "unit": "GB/s", "peak_source": peak_src},
            "per_layer": layer, "per_projection": per, "cpu_baseline": cpu}


def pmat_cpu_baseline() -> dict | None:
    """The reference's own vx27_pmat (oracle/_ref, AVX2, all host threads) on
    in_proj_qkv (10240 x 5120, BP3_128), one token."""
    import ctypes as C
    import time
    import numpy as np
    sys.path.insert(0, ROOT)
    import oracle.oracle as O
    if not os.path.exists(O.REF_PMAT_LIB) and not O.build_ref():
        return None
    if not os.path.exists(O.REF_PMAT_LIB):
        return None
    lib = C.CDLL(O.REF_PMAT_LIB)
    lib.tp_create.restype = C.c_void_p
    lib.tp_create.argtypes = [C.c_int, C.c_char_p, C.c_size_t]
    lib.vx27_pmat.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p,
                              C.c_int, C.c_int]
    threads = os.cpu_count() or 1
    tp = lib.tp_create(threads, None, 0)
    rows, cols = 10240, 5120
    W = O.packed_weights(O.PMAT_BP3, rows, cols, 5)
    x = np.random.default_rng(1).standard_normal(cols).astype(np.float32)
    y = np.empty(rows, np.float32)
    best = 1e9
    for _ in range(5):
        t0 = time.perf_counter()
        lib.vx27_pmat(tp, O.P(W), O.PMAT_BP3, O.P(x), O.P(y), rows, cols)
        best = min(best, time.perf_counter() - t0)
    return {"value": round(rows * 52 * (cols // 128) / best / 1e9, 2), "unit": "GB/s",
            "us": round(best * 1e6, 1), "cores": threads, "kind": "reference",
            "sample": "vx27_pmat on in_proj_qkv 10240 x 5120 BP3_128, one token, best of 5"}


# ------------------------------------------------- configs 0 and 1 (batch-1 latency)
def run_batch1(args, cpu: bool = True) -> dict:
    """Config 0: one DeltaNet layer decoding 2000 tokens of one sequence (16 heads, fp32
    activations, seed 0); config 1: one gated GQA single-query decode at context 8192
    (seed 1). Both are latency-bound at batch 1: the line reports microseconds per token,
    launched one call per token as a decode loop does, and replayed from one CUDA graph."""
    import torch
    from oracle import oracle as orc
    from vx27_b200 import ops
    torch.cuda.set_device(0)
    hbm, hbm_src = peaks()
    bf = torch.bfloat16
    if args.workload == "config0":
        n_tok, nqk, nv = 2000, 16, 16
        C = (2 * nqk + nv) * 128
        qkv = torch.empty(n_tok, C, device="cuda")
        a = torch.empty(n_tok, nv, device="cuda")
        b = torch.empty(n_tok, nv, device="cuda")
        w = torch.empty(C, 4, device="cuda")
        dt = torch.empty(nv, device="cuda")
        A = torch.empty(nv, device="cuda")
        for n, (t, sd) in enumerate(((qkv, 1.0), (a, 1.0), (b, 1.0), (w, 0.5), (dt, 0.1))):
            ops.fill_normal(t, 0, n + 1, 0.0, sd)
        ops.fill_uniform(A, 0, 6, 1.0, 16.0)
        A.log_()
        S = torch.zeros(1, nv, 128, 128, device="cuda")
        ring = torch.zeros(1, 4, C, device="cuda")
        o = torch.empty(n_tok, nv, 128, device="cuda")
        pos = torch.arange(n_tok, dtype=torch.int32, device="cuda")

        def run():
            for t in range(n_tok):
                ops.deltanet_decode_batch(S, ring, qkv[t:t + 1], a[t:t + 1], b[t:t + 1], A, dt,
                                          w, pos[t:t + 1], o[t:t + 1], nqk, nv)
        def run_tokens():  # all 2000 tokens in one call, the state resident in the kernel
            ops.deltanet_decode_tokens(S[0], ring[0], qkv, a, b, A, dt, w, pos, o, nqk, nv)
        units, unit_name = n_tok, "token"
        bytes_per_unit = 2 * nv * 128 * 128 * 4 + 4 * C * 4 + C * 4 + nv * 128 * 4
        name = "config 0: DeltaNet decode, batch 1, 16 heads, 2000 sequential tokens"
        others = {"vx27_deltanet_decode_tokens, one call for the 2000 tokens": run_tokens}
    else:
        ctx, nq, nkv, hd = 8192, 24, 4, 256
        cap = ctx
        kc = torch.empty(1, nkv, cap, hd, dtype=bf, device="cuda")
        vc = torch.empty_like(kc)
        ops.fill_normal(kc, 1, 1)
        ops.fill_normal(vc, 1, 2)
        q_in = torch.empty(1, nq, hd, device="cuda")
        k_in = torch.empty(1, nkv, hd, device="cuda")
        v_in = torch.empty(1, nkv, hd, device="cuda")
        gate = torch.empty(1, nq, hd, device="cuda")
        qw = torch.empty(hd, device="cuda")
        kw = torch.empty(hd, device="cuda")
        for n, t in enumerate((q_in, k_in, v_in, gate)):
            ops.fill_normal(t, 1, 3 + n)
        ops.fill_normal(qw, 1, 7, 1.0, 0.02)
        ops.fill_normal(kw, 1, 8, 1.0, 0.02)
        rope = ops.rope_table(ctx)
        qn = torch.empty(1, nq, hd, device="cuda")
        out = torch.empty(1, nq, hd, device="cuda")
        pos = torch.full((1,), ctx - 1, dtype=torch.int32, device="cuda")
        ws = torch.empty(ops.gqa_workspace_bytes(1, nq, nkv, hd, cap) // 4 + 1, device="cuda")

        def run():  # append + the tensor-core split-KV decode (+ combine)
            ops.gqa_append(q_in, k_in, v_in, qw, kw, rope, pos, kc, vc, qn)
            ops.gqa_decode_batch(qn, gate, kc, vc, pos, out, ws, prefetch_kv=True)

        def run_fused():  # the same in one split kernel (+ combine)
            ops.gqa_decode_fused(q_in, k_in, v_in, qw, kw, rope, gate, kc, vc, pos, out, ws,
                                 prefetch_kv=True)

        def run_cc():  # the CUDA-core split-KV kernel, prologue fused
            ops.gqa_decode_fused(q_in, k_in, v_in, qw, kw, rope, gate, kc, vc, pos, out, ws,
                                 kernel="cc", prefetch_kv=True)
        others = {"fused tensor-core decode": run_fused, "fused CUDA-core decode": run_cc}
        units, unit_name = 1, "decode"
        bytes_per_unit = nkv * ctx * hd * 2 * 2 + nq * hd * 4 * 3
        name = "config 1: gated GQA single-query decode, batch 1, context 8192"
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    reps = max(1, args.steps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        e0.record()
        for _ in range(reps):
            run()
        e1.record()
        torch.cuda.synchronize()
        us_launch = e0.elapsed_time(e1) * 1e3 / (reps * units)
        # graph replays: 10 warm, then enough timed replays (>= 200 for one decode, one
        # for the 2000 tokens) that the per-replay launch jitter averages out
        g_reps = max(reps, 200 // units, 1)

        def graph_us(fn) -> float:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            for _ in range(10 if units == 1 else 1):
                g.replay()
            torch.cuda.synchronize()
            e0.record()
            for _ in range(g_reps):
                g.replay()
            e1.record()
            torch.cuda.synchronize()
            del g
            return e0.elapsed_time(e1) * 1e3 / (g_reps * units)
        us_graph = graph_us(run)
        other_us = {}
        for label, fn in others.items():
            for _ in range(args.warmup):
                fn()
            other_us[label] = round(graph_us(fn), 3)
    if ops.device_status() != 0:
        raise RuntimeError("device status flag set during the batch-1 run")
    gbs = bytes_per_unit / (us_graph * 1e-6) / 1e9
    line = {
        "metric": f"microseconds per {unit_name} ({args.workload}, batch 1)",
        "value": round(us_graph, 3), "unit": f"us/{unit_name}", "n_gpus": 1,
        "steps": reps, "graph_replays": g_reps, "warmup": args.warmup,
        "higher_is_better": False, "dtype": "f32",
        "data": "synthetic (seeded, BASELINE.json distributions)",
        "config": {"workload": name},
        "us_per_unit_launched": round(us_launch, 3), "us_per_unit_graph": round(us_graph, 3),
        "other_forms_us_graph": other_us,
        "roofline": {"bound": "hbm (latency at batch 1)", "achieved": round(gbs, 1),
                     "peak": hbm, "unit": "GB/s", "frac": round(gbs / hbm, 4),
                     "algorithmic_bytes_per_unit": bytes_per_unit, "peak_source": hbm_src},
        "clocks": clk.summary(),
    }
    if not cpu:
        return line
    # the reference's own code on the host (oracle/_ref when built, else the port)
    import os as _os
    import time as _time
    kind = "reference" if orc.use_reference(True) else "port"
    L, P = orc.lib(), orc.P
    threads = _os.cpu_count() or 1
    if args.workload == "config0":
        n_cpu = 100
        Sh = np.zeros(nv * 128 * 128, np.float32)
        rh = np.zeros(4 * C, np.float32)
        xh = orc.normal(n_cpu * C, 0, 1)
        ah, bh = orc.normal(n_cpu * nv, 0, 2), orc.normal(n_cpu * nv, 0, 3)
        wh = orc.normal(C * 4, 0, 4, 0.0, 0.5)
        dth = orc.normal(nv, 0, 5, 0.0, 0.1)
        Ah = np.log(orc.uniform(nv, 0, 6, 1.0, 16.0)).astype(np.float32)
        oh = np.zeros(nv * 128, np.float32)
        t0 = _time.perf_counter()
        for t in range(n_cpu):
            p = np.array([t], np.int32)
            L.orc_deltanet_decode_batch_mt(P(Sh), P(rh), P(xh[t * C:]), P(ah[t * nv:]),
                                           P(bh[t * nv:]), P(Ah), P(dth), P(wh), P(p), P(oh),
                                           1, nqk, nv, 128, 0, threads)
        cpu_us = (_time.perf_counter() - t0) * 1e6 / n_cpu
        sample = f"{n_cpu} tokens x 16 heads (step_exact per head, {threads} threads)"
    else:
        from oracle.oracle import to_bf16
        kh = to_bf16(orc.normal(nkv * ctx * hd, 1, 1))
        vh = to_bf16(orc.normal(nkv * ctx * hd, 1, 2))
        qh = orc.normal(nq * hd, 1, 3)
        gh = orc.normal(nq * hd, 1, 6)
        outh = np.zeros(nq * hd, np.float32)
        p = np.array([ctx - 1], np.int32)
        t0 = _time.perf_counter()
        n_cpu = 5
        for _ in range(n_cpu):
            L.orc_gqa_attend_mt(P(qh), P(gh), P(kh), P(vh), ctx, P(p), P(outh), 1, nq, nkv, hd,
                                0, threads)
        cpu_us = (_time.perf_counter() - t0) * 1e6 / n_cpu
        sample = f"{n_cpu} decodes over 8192 positions ({threads} threads)"
    line["cpu_baseline"] = {"value": round(cpu_us, 2), "unit": f"us/{unit_name}",
                            "cores": threads, "kind": kind, "sample": sample}
    return line


# ------------------------------------------------- config 4 (prefill)
def prefill_flops(T: int) -> tuple[float, float]:
    """Algorithmic FLOPs of one config-4 layer of each kind.
    GQA: causal QK^T and PV over T(T+1)/2 (query, key) pairs, 24 heads, hd 256.
    DeltaNet (chunk 64, 16 heads, 128x128 state), per chunk and head: K K^T and Q K^T
    (2*64*64*128 each), T V and T K (2*64*64*128 each), U = W_v - W_k S and the state
    update (2*64*128*128 each), Q S (2*64*128*128) and the intra-chunk P U (2*64*64*128)."""
    pairs = T * (T + 1) / 2
    gqa = 2 * 2 * pairs * 24 * 256
    per_chunk = 5 * (2 * 64 * 64 * 128) + 3 * (2 * 64 * 128 * 128)
    dn = per_chunk * 16 * ((T + 63) // 64)
    return gqa, dn


def run_prefill(args) -> dict:
    """Config 4: a 32768-token prompt, batch 1, through one DeltaNet layer (chunked gated
    delta rule, 16 heads) and one gated GQA layer (causal 24Q/4KV hd256 on the tensor
    cores). value = prompt tokens/s through one layer of each kind."""
    import torch
    from vx27_b200 import ops
    torch.cuda.set_device(0)
    T = args.prefill_T
    bf = torch.bfloat16
    hbm, hbm_src = peaks()
    tc_peak, tc_src = tensor_peak()
    # DeltaNet layer inputs (gates as in config 0), seed 4
    nqk = nv = 16
    q = torch.empty(T, nqk, 128, dtype=bf, device="cuda")
    k = torch.empty_like(q)
    v = torch.empty(T, nv, 128, dtype=bf, device="cuda")
    a = torch.empty(T, nv, dtype=bf, device="cuda")
    b = torch.empty_like(a)
    A = torch.empty(nv, device="cuda")
    dt = torch.empty(nv, device="cuda")
    S = torch.zeros(nv, 128, 128, device="cuda")
    o = torch.empty(T, nv, 128, dtype=bf, device="cuda")
    for n, t in enumerate((q, k, v, a, b)):
        ops.fill_normal(t, 4, n + 1)
    ops.fill_normal(dt, 4, 7, 0.0, 0.1)
    ops.fill_uniform(A, 4, 6, 1.0, 16.0)
    A.log_()
    ws_dn = torch.empty(ops.load().vx27_deltanet_prefill_workspace_size(T, nqk, nv, 128) // 4 + 1,
                        device="cuda")
    run_dn = lambda: ops.deltanet_prefill_chunked(q, k, v, a, b, A, dt, S, o, ws_dn)
    # GQA layer inputs
    nq, nkv, hd = 24, 4, 256
    gq = torch.empty(T, nq, hd, dtype=bf, device="cuda")
    gk = torch.empty(T, nkv, hd, dtype=bf, device="cuda")
    gv = torch.empty_like(gk)
    gate = torch.empty_like(gq)
    qw = torch.empty(hd, device="cuda")
    kw = torch.empty(hd, device="cuda")
    for n, t in enumerate((gq, gk, gv, gate)):
        ops.fill_normal(t, 4, 10 + n)
    ops.fill_normal(qw, 4, 14, 1.0, 0.02)
    ops.fill_normal(kw, 4, 15, 1.0, 0.02)
    kc = torch.empty(nkv, T, hd, dtype=bf, device="cuda")
    vc = torch.empty_like(kc)
    out = torch.empty(T, nq, hd, dtype=bf, device="cuda")
    rope = ops.rope_table(T)
    ws_g = torch.empty(ops.load().vx27_gqa_prefill_workspace_size(T, nq, hd) // 2 + 1,
                       dtype=torch.int16, device="cuda")
    run_gqa = lambda: ops.gqa_prefill(gq, gk, gv, gate, qw, kw, rope, kc, vc, out, ws_g)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        for e0, e1 in evs:
            e0.record()
            fn()
            e1.record()
        torch.cuda.synchronize()
        return [e0.elapsed_time(e1) for e0, e1 in evs]

    with ClockSampler(0) as clk:
        t_dn = timed(run_dn)
        t_gqa = timed(run_gqa)
    if ops.device_status() != 0:
        raise RuntimeError("device status flag set during the prefill run")
    ms_dn, ms_gqa = statistics.mean(t_dn), statistics.mean(t_gqa)
    f_gqa, f_dn = prefill_flops(T)
    # HBM bytes the DeltaNet layer must move: q,k,v,a,b in (bf16), o out (bf16), S in/out
    dn_bytes = T * (2 * nqk + nv) * 128 * 2 + T * nv * 2 * 2 + T * nv * 128 * 2 + \
        2 * nv * 128 * 128 * 4
    tflops = f_gqa / (ms_gqa * 1e-3) / 1e12
    return {
        "metric": "prompt tokens/s through one DeltaNet + one gated GQA layer (config 4)",
        "value": round(T / ((ms_dn + ms_gqa) * 1e-3), 1), "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_dn + ms_gqa, 4), "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic (seed 4)",
        "config": {"workload": f"config 4: prefill of a {T}-token prompt, batch 1",
                   "l2": "inputs and workspaces larger than L2"},
        "gqa_prefill": {"ms": round(ms_gqa, 4), "tflops": round(tflops, 1),
                        "algorithmic_flops": f_gqa,
                        "roofline": {"bound": "tensor", "achieved": round(tflops, 1),
                                     "peak": tc_peak, "unit": "TFLOP/s",
                                     "frac": round(tflops / tc_peak, 4),
                                     "peak_source": tc_src}},
        "deltanet_prefill": {"ms": round(ms_dn, 4), "algorithmic_flops": f_dn,
                             "tflops": round(f_dn / (ms_dn * 1e-3) / 1e12, 2),
                             "algorithmic_bytes": dn_bytes,
                             "hbm_GBps": round(dn_bytes / (ms_dn * 1e-3) / 1e9, 1),
                             "hbm_frac": round(dn_bytes / (ms_dn * 1e-3) / 1e9 / hbm, 4),
                             "hbm_peak_source": hbm_src},
        "clocks": clk.summary(),
    }


# ------------------------------------------------- config 3 (long context)
def run_longctx(args, rank: int, world: int, local: int) -> dict | None:
    """Config 3: 16 gated GQA layers at context 262144, query at 262143.
    config3a: 16 sequences sharded across ranks (no collective); a rank whose share does
    not fit in HBM runs it in waves (the cache of the next wave is regenerated between
    waves, outside the timed region). config3b: one sequence, KV range sharded across
    ranks, one all-gather of the partial records per step."""
    import torch
    import torch.distributed as dist
    from vx27_b200.dist import shard_range
    from vx27_b200.longctx import LongContextGQA
    torch.cuda.set_device(local)
    ctx, layers = args.ctx3, 16
    seq_bytes = layers * 4 * ctx * 256 * 2 * 2
    split = args.workload == "config3b"
    if split:
        waves, total_seq = [(1, 0)], 1
    else:
        total_seq = args.seqs3
        b0, b1 = shard_range(total_seq, world, rank)
        w = max(1, min(b1 - b0, int(args.hbm_budget_gb * 1e9 // seq_bytes)))
        waves = [(min(w, b1 - s), s) for s in range(b0, b1, w)]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    step_ms, kv_bytes, launches = 0.0, 0, 0
    for bsz, off in waves:
        dec = LongContextGQA(bsz, ctx, layers, rank=rank, world=world, split_kv=split,
                             seq_offset=off)
        for _ in range(args.warmup):
            per_step = dec.step()
        graph = None
        if args.graph:  # one CUDA graph per step: no host launch overhead between kernels
            barrier()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                dec.step()
            graph.replay()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            if graph is not None:
                graph.replay()
                launches += per_step
            else:
                launches += dec.step()
        e1.record()
        barrier()
        del graph
        step_ms += e0.elapsed_time(e1) / args.steps
        kv_bytes += dec.kv_bytes()
        del dec
        torch.cuda.empty_cache()
    mx = step_ms
    if world > 1:
        t = torch.tensor([step_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        mx = float(t.item())
    peak, peak_src = peaks()
    gbs = kv_bytes / (step_ms * 1e-3) / 1e9
    if rank != 0:
        return None
    return {"metric": "long-context gated GQA decode tokens/s (config 3); % of HBM roofline",
            "workload": args.workload, "value": round(total_seq / (mx * 1e-3), 3),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(mx, 4), "higher_is_better": True,
            "scaling": "strong" if split else "weak",
            "config": {"ctx": ctx, "layers": layers, "sequences": total_seq,
                       "waves_rank0": [w[0] for w in waves],
                       "wave_note": "caches regenerated between waves, outside timing",
                       "parallelism": (f"kv-split{world} (NCCL all-gather of partial records)"
                                       if split else f"dp{world} (sequences sharded)")},
            "roofline_rank0": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak,
                               "unit": "GB/s", "frac": round(gbs / peak, 4),
                               "kv_bytes_per_step": kv_bytes, "peak_source": peak_src},
            "gpu_launches": launches, "cuda_graph": bool(args.graph)}


# ------------------------------------------------- the other configs, briefly
def other_configs(args) -> dict:
    """Configs 0, 1 and 4 on the same GPU after the config 2 timed region (its buffers
    freed): the batch-1 DeltaNet decode of 2000 tokens and the batch-1 GQA decode at context
    8192 (both replayed from a CUDA graph), and the 32768-token prefill of one layer of each
    kind, each with its own clock samples."""
    import copy
    import torch
    torch.cuda.empty_cache()
    a0 = copy.copy(args)
    a0.workload, a0.steps, a0.warmup = "config0", 3, 1
    c0 = run_batch1(a0, cpu=False)
    a1 = copy.copy(args)
    a1.workload, a1.steps, a1.warmup = "config1", 200, 10
    c1 = run_batch1(a1, cpu=False)
    a4 = copy.copy(args)
    a4.workload, a4.steps, a4.warmup = "config4", 5, 2
    c4 = run_prefill(a4)
    torch.cuda.empty_cache()
    return {
        "config0_token_us": c0["value"],
        "config0": {"us_per_token_graph": c0["us_per_unit_graph"],
                    "us_per_token_launched": c0["us_per_unit_launched"],
                    "form": "vx27_deltanet_decode_batch, one call per token",
                    "other_forms_us_graph": c0["other_forms_us_graph"],
                    "roofline": c0["roofline"], "clocks": c0["clocks"]},
        "config1_decode_us": c1["value"],
        "config1": {"us_per_decode_graph": c1["us_per_unit_graph"],
                    "us_per_decode_launched": c1["us_per_unit_launched"],
                    "form": "vx27_gqa_append + vx27_gqa_decode_batch (tensor cores)",
                    "other_forms_us_graph": c1["other_forms_us_graph"],
                    "roofline": c1["roofline"], "clocks": c1["clocks"]},
        "config4_gqa_prefill": {"ms": c4["gqa_prefill"]["ms"],
                                "tflops": c4["gqa_prefill"]["tflops"],
                                "frac": c4["gqa_prefill"]["roofline"]["frac"],
                                "peak": c4["gqa_prefill"]["roofline"]["peak"],
                                "peak_source": c4["gqa_prefill"]["roofline"]["peak_source"]},
        "config4_deltanet_prefill": {"ms": c4["deltanet_prefill"]["ms"],
                                     "tflops": c4["deltanet_prefill"]["tflops"],
                                     "hbm_frac": c4["deltanet_prefill"]["hbm_frac"]},
        "config4_prompt_tokens_per_s": c4["value"],
        "config4_clocks": c4["clocks"],
    }


# ------------------------------------------------------------ CPU reference
def cpu_reference_step_sampler(n_seq: int, ctx: int, threads: int):
    """Builds host buffers for n_seq sequences of config 2 and returns (run_step, kind).
    run_step() runs one decode step of those sequences through all 64 layers with the
    reference's step_exact/conv1d_step/gate_params/rmsnorm/rope (oracle/_ref) when built,
    else the oracle port; the attention loop is the restatement of src/vx27_qfwd.c:347-371
    over a BF16 cache (the reference has no callable long-context attention)."""
    from oracle import oracle as orc
    kind = "reference" if orc.use_reference(True) else "port"
    L = orc.lib()
    P = orc.P
    nqk = nv = 16
    hd, nq, nkv, HD = 128, 24, 4, 256
    C = (2 * nqk + nv) * hd
    cap = ctx + 1
    rng = np.random.default_rng(2)
    block = rng.standard_normal(1 << 20).astype(np.float32)

    def tiled(n, scale=1.0, dtype=np.float32):
        reps = -(-n // block.size)
        a = np.tile(block * scale, reps)[:n]
        return np.ascontiguousarray(a if dtype == np.float32 else orc.to_bf16(a))

    S = [tiled(n_seq * nv * hd * hd, 0.05) for _ in range(48)]
    ring = [tiled(n_seq * 4 * C) for _ in range(48)]
    qkv = tiled(n_seq * C, dtype=np.uint16)
    ab = tiled(n_seq * nv, dtype=np.uint16)
    conv_w = tiled(C * 4, 0.5)
    A_log = np.log(np.linspace(1, 16, nv)).astype(np.float32)
    dt_bias = tiled(nv, 0.1)
    kc = [tiled(n_seq * nkv * cap * HD, dtype=np.uint16) for _ in range(16)]
    vc = [tiled(n_seq * nkv * cap * HD, dtype=np.uint16) for _ in range(16)]
    qi = tiled(n_seq * nq * HD, dtype=np.uint16)
    ki = tiled(n_seq * nkv * HD, dtype=np.uint16)
    gate = tiled(n_seq * nq * HD, dtype=np.uint16)
    wn = np.ones(HD, np.float32)
    o = np.zeros(n_seq * nv * hd, np.float32)
    qo = np.zeros(n_seq * nq * HD, np.float32)
    att = np.zeros(n_seq * nq * HD, np.float32)
    pos = np.full(n_seq, ctx, np.int32)

    def run_step():
        for layer in range(64):
            if (layer + 1) % 4:
                i = layer - (layer + 1) // 4
                L.orc_deltanet_decode_batch_mt(P(S[i]), P(ring[i]), P(qkv), P(ab), P(ab),
                                               P(A_log), P(dt_bias), P(conv_w), P(pos), P(o),
                                               n_seq, nqk, nv, hd, orc.F_ACT_BF16, threads)
            else:
                i = layer // 4
                L.orc_gqa_append(P(qi), P(ki), P(ki), P(wn), P(wn), P(pos), P(kc[i]), P(vc[i]),
                                 cap, P(qo), n_seq, nq, nkv, HD, 64, 1e7, 1e-6, orc.F_ACT_BF16)
                L.orc_gqa_attend_mt(P(qo), P(gate), P(kc[i]), P(vc[i]), cap, P(pos), P(att),
                                    n_seq, nq, nkv, HD, orc.F_ACT_BF16, threads)
    return run_step, kind


def cpu_baseline(n_seq: int, ctx: int, min_s: float = 3.0, max_reps: int = 10) -> dict:
    threads = os.cpu_count() or 1
    run, kind = cpu_reference_step_sampler(n_seq, ctx, threads)
    run()  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        run()
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_s or reps >= max_reps:
            break
    return {"value": round(n_seq * reps / el, 3), "unit": "tokens/s", "cores": threads,
            "kind": kind,
            "sample": f"{n_seq} sequences x {reps} decode steps x 64 layers at ctx {ctx} "
                      f"({el:.1f} s wall, all host threads)"}


def run_reference(args, rank: int) -> dict | None:
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    n_seq = args.ref_seqs
    run, kind = cpu_reference_step_sampler(n_seq, args.ctx, threads)
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    el = time.perf_counter() - t0
    v = round(n_seq * args.steps / el, 3)
    return {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64-accumulate/f32",
        "data": "synthetic",
        "config": {"workload": "config 2 (bounded CPU sample of sequences per step)",
                   "sequences_per_step": n_seq, "ctx": args.ctx},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": kind,
                         "sample": f"{n_seq} sequences per step x 64 layers, {args.steps} "
                                   f"steps"},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=256, help="sequences per GPU")
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--ref-seqs", type=int, default=4)
    ap.add_argument("--cpu-seqs", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-other-configs", action="store_true",
                    help="config 2 at N = 1: skip the config 1 and config 4 figures added "
                         "after its timed region")
    ap.add_argument("--two-kernel-gqa", dest="fused_gqa", action="store_false",
                    help="config 2: GQA layers as append + split-KV decode instead of one "
                         "fused kernel (vx27_gqa_decode_fused, the default)")
    ap.add_argument("--workload", choices=["config2", "config0", "config1", "config3a",
                                           "config3b", "config4", "dn_layer", "gqa_layer", "pmat"],
                    default="config2",
                    help="config2 (the metric); config3a/3b long context; single-layer "
                         "workloads are for kernel rooflines and profiling")
    ap.add_argument("--ctx3", type=int, default=262144)
    ap.add_argument("--seqs3", type=int, default=16)
    ap.add_argument("--hbm-budget-gb", type=float, default=150.0)
    ap.add_argument("--prefill-T", type=int, default=32768, help="config4 prompt length")
    ap.add_argument("--graph", action="store_true",
                    help="config3: replay each step as one CUDA graph")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.workload in ("dn_layer", "gqa_layer"):
        print(json.dumps(run_layer(args)), flush=True)
        return
    if args.workload == "pmat":
        print(json.dumps(run_pmat(args)), flush=True)
        return
    if args.workload == "config4":
        print(json.dumps(run_prefill(args)), flush=True)
        return
    if args.workload in ("config0", "config1"):
        print(json.dumps(run_batch1(args)), flush=True)
        return

    if args.impl == "reference":
        line = run_reference(args, rank)
        if line:
            print(json.dumps(line), flush=True)
        return

    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload in ("config3a", "config3b"):
            line = run_longctx(args, rank, world, local_rank)
            if line is not None:
                print(json.dumps(line), flush=True)
            return
        line = run_ours(args, rank, world, local_rank)
        if line is not None:
            if world == 1 and not args.no_other_configs:
                line["other_configs"] = other_configs(args)
            if world == 1 and not args.no_cpu_baseline:
                line["cpu_baseline"] = cpu_baseline(args.cpu_seqs, args.ctx)
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
