#!/usr/bin/env python
"""Decode-layer benchmark: one decode step of a layer with hidden
8192, 64 query / 8 KV heads, head_dim 128, batch 128, context lengths U[1024, 8192], page 16.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl okc|reference]

N > 1 runs under torchrun, one rank per GPU, tensor parallel over the heads; after the
row-parallel O projection one kernel over NVLink peer memory (okc_tp_allreduce_residual) sums
the ranks' partials and adds the residual.  Rank 0 prints ONE JSON line.

value     = device time per step (CUDA events around K graph replays, max over ranks), µs.
e2e       = the same step through the public API (DecodeLayer.step) with the step's input
            (x and positions, one pinned buffer) copied in and its output copied back to
            pinned memory every step, copies and step in one graph, µs.
roofline  = the attention kernel (the dominant kernel) measured with CUDA events inside an
            instrumented copy of the step graph: algorithmic KV bytes / duration vs
            MEASURED_PEAKS.json hbm_gbs; stages_us = per-stage times from the same copy.
cpu_baseline / --impl reference = the oracle (the reference's PyTorch path restated, CPU
            fp32) on the host cores, a bounded sample scaled to one full step.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
METRIC = "decode-layer µs/step and attn/GEMV HBM GB/s (% of 8 TB/s) at 1/2/4/8 B200"
WORKLOAD = {"workload": "decode_layer_c4", "batch": 128, "hidden": 8192, "heads": "64q/8kv",
            "head_dim": 128, "ctx": "U[1024,8192]", "page_size": 16, "pool_pages": 131072,
            "rope_theta": 5e5, "kv": "e4m3 per-head scales",
            "l2": "no flush: every step reads >1.5 GB (KV cache + weights), 12x the 126 MB L2"}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region (rank-local GPU)."""

    def __init__(self, index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        rows = [r.split(",") for r in Path(self.f.name).read_text().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower().startswith("active"):
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------ CPU baseline
def cpu_layer_sample(B=128, seed=0, sample_seqs=8):
    """Times the oracle layer on the host: the projections at the full 128 tokens, the
    attention over `sample_seqs` of the 128 sequences (same ctx distribution), scaled to 128."""
    import torch
    from oracle import attention as oatt
    from oracle.projection import gemm, rmsnorm
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    H, Hq, Hkv, D, P = 8192, 64, 8, 128, 16
    x = torch.randn((B, H), generator=g).to(torch.bfloat16)
    nw = torch.ones(H, dtype=torch.bfloat16)
    wqkv = (torch.randn(((Hq + 2 * Hkv) * D, H), generator=g) * 0.02).to(torch.bfloat16)
    wo = (torch.randn((H, Hq * D), generator=g) * 0.02).to(torch.bfloat16)
    lens = torch.randint(1024, 8193, (sample_seqs,), generator=g)
    pages = [math.ceil((int(n) + 1) / P) for n in lens]
    table = torch.full((sample_seqs, max(pages)), -1, dtype=torch.int32)
    off = 0
    for b, n in enumerate(pages):
        table[b, :n] = torch.arange(off, off + n, dtype=torch.int32)
        off += n
    kc = torch.randn((off, P, Hkv, D), generator=g).to(torch.float8_e4m3fn)
    vc = torch.randn((off, P, Hkv, D), generator=g).to(torch.float8_e4m3fn)
    ks = torch.ones(Hkv)
    vs = torch.ones(Hkv)
    pos = lens.long()
    t0 = time.perf_counter()
    xn = rmsnorm(x, nw, 1e-6)
    qkv = gemm(xn, wqkv)
    t1 = time.perf_counter()
    q, _ = oatt.kv_append(qkv[:sample_seqs], pos, table, kc, vc, ks, vs, Hq, Hkv, D, 5e5)
    o = oatt.attend(q.to(torch.bfloat16), kc, vc, table, pos + 1, ks, vs, D ** -0.5).to(torch.bfloat16)
    t2 = time.perf_counter()
    o_full = o.reshape(sample_seqs, Hq * D).repeat(B // sample_seqs, 1)
    gemm(o_full, wo, residual=x)
    t3 = time.perf_counter()
    step_s = (t1 - t0) + (t2 - t1) * (B / sample_seqs) + (t3 - t2)
    return step_s * 1e6, torch.get_num_threads(), (
        f"oracle layer on host: RMSNorm+QKV and O-proj at 128 tokens, attention over {sample_seqs} "
        f"of 128 sequences (ctx U[1024,8192]) scaled x{B // sample_seqs}")


def run_reference(args):
    """--impl reference: the reference's own (PyTorch, CPU) path restated as the oracle."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    for _ in range(args.warmup):
        cpu_layer_sample(seed=1)
    vals = []
    cores = 1
    sample = ""
    for i in range(args.steps):
        v, cores, sample = cpu_layer_sample(seed=2 + i)
        vals.append(v)
    val = statistics.mean(vals)
    line = {"impl": "reference", "metric": METRIC, "value": round(val, 1), "unit": "us/step",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(val / 1000, 3), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp32 (CPU oracle)", "data": "synthetic",
            "config": dict(WORKLOAD, parallelism=f"tp{args.gpus}", reference_runs_on="host cores (rank 0)"),
            "cpu_baseline": {"value": round(val, 1), "unit": "us/step", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(val, 1), "unit": "us/step", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------- GPU arm
def run_okc(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        group = dist.group.WORLD

    from okc_b200 import ops, synth
    from okc_b200.layer import DecodeLayer, LayerConfig

    cfg = LayerConfig()
    B = 128
    lq, lkv = cfg.num_q_heads // world, cfg.num_kv_heads // world
    # identical page tables / lengths / weights on every rank (same seeds, same device type)
    att = synth.attention_case(B, lq, lkv, cfg.head_dim, (1024, 8192), cfg.page_size, 1 << 17, seed=0,
                               device=dev, extra_tokens=1)
    g = torch.Generator(device=dev).manual_seed(1)
    H = cfg.hidden
    x = torch.randn((B, H), generator=g, device=dev).to(torch.bfloat16)
    norm_w = (1.0 + 0.02 * torch.randn((H,), generator=g, device=dev)).to(torch.bfloat16)
    d, hq, hkv = cfg.head_dim, cfg.num_q_heads, cfg.num_kv_heads
    wqkv = (torch.randn(((hq + 2 * hkv) * d, H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wo = (torch.randn((H, hq * d), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    # per-rank scales for the rank's KV heads (the generated cache holds only those heads)
    ks_full = torch.ones(hkv, device=dev)
    vs_full = torch.ones(hkv, device=dev)
    ks_full[rank * lkv:(rank + 1) * lkv] = att["k_scale"]
    vs_full[rank * lkv:(rank + 1) * lkv] = att["v_scale"]
    layer = DecodeLayer(cfg, norm_w, wqkv, wo, ks_full, vs_full, rank, world, group)
    del wqkv, wo
    positions = att["seq_lens"].long().clone()
    table, kc, vc = att["page_table"], att["k_cache"], att["v_cache"]
    lens = (positions + 1).to(torch.int32)
    out = torch.empty((B, H), dtype=torch.bfloat16, device=dev)

    def step():
        # at TP > 1 the result is the exchange group's replicated output buffer (no extra copy)
        return layer.step(x, positions, table, kc, vc, lens=lens, out=out if world == 1 else None)

    # warm-up (eager), then capture one step; in-graph external events bracket attention
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    ev_a0 = torch.cuda.Event(enable_timing=True, external=True)
    ev_a1 = torch.cuda.Event(enable_timing=True, external=True)
    # stage boundaries inside the graph (external events): norm, QKV + RoPE/append,
    # attention, O projection, exchange + residual
    ev_s = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(4)]
    xn_buf = {}
    fused = world > 1 and layer.comm_for(B).fused

    def step_instrumented():
        cfgl, dd = layer.cfg, layer.cfg.head_dim
        ev_s[0].record()
        xn = ops.rmsnorm(x, layer.norm_w, cfgl.eps)
        ev_s[1].record()
        q = ops.gemm_rope_kv_append(xn, layer.wqkv, positions, table, kc, vc, layer.k_scale, layer.v_scale,
                                    layer.lq, layer.lkv, dd, layer.inv_freq)
        ev_a0.record()
        o = ops.attn_decode(q, kc, vc, table, lens, layer.k_scale, layer.v_scale, layer.sm_scale)
        ev_a1.record()
        o2 = o.view(B, layer.lq * dd)
        if world == 1:
            ops.gemm(o2, layer.wo, residual=x, out=out)
            ev_s[2].record()
        elif fused:  # O projection + exchange in one kernel
            layer.comm_for(B).oproj_allreduce_residual(o2, layer.wo, x)
            ev_s[2].record()
        else:
            comm = layer.comm_for(B)
            ops.gemm(o2, layer.wo, out_fp32=True, out=comm.partial)
            ev_s[2].record()
            comm.allreduce_residual(x)
        ev_s[3].record()
        xn_buf["q"] = q
        return out

    # Two graphs of the same step: `graph` is the public API call (DecodeLayer.step) with no
    # event inside, so programmatic dependent launch chains every kernel to the next; it is
    # what `value` and `e2e` time.  `graph_i` adds external events between the stages (an event
    # node breaks the programmatic chain there) for the attention roofline and `stages_us`.
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step_instrumented()
        step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph_i = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_i):
        step_instrumented()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(args.warmup, 3)):
        graph_i.replay()
        graph.replay()
    torch.cuda.synchronize()

    # ------------------------------------------------------------- timed region
    sampler = ClockSampler(local) if rank == 0 else None
    time.sleep(0.3 if sampler else 0)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    us = e0.elapsed_time(e1) * 1000.0 / args.steps
    t = torch.tensor([us], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us = float(t.item())

    # attention and stage durations from the instrumented graph (one replay per sample)
    att_us = []
    stage_us = {"norm": [], "qkv_rope_append": [], "attention": [], "o_proj": [], "allreduce_residual": []}
    for _ in range(args.steps):
        graph_i.replay()
        torch.cuda.synchronize()
        att_us.append(ev_a0.elapsed_time(ev_a1) * 1000.0)
        stage_us["norm"].append(ev_s[0].elapsed_time(ev_s[1]) * 1000.0)
        stage_us["qkv_rope_append"].append(ev_s[1].elapsed_time(ev_a0) * 1000.0)
        stage_us["attention"].append(ev_a0.elapsed_time(ev_a1) * 1000.0)
        stage_us["o_proj"].append(ev_a1.elapsed_time(ev_s[2]) * 1000.0)
        stage_us["allreduce_residual"].append(ev_s[2].elapsed_time(ev_s[3]) * 1000.0)
    att_avg = statistics.mean(att_us)
    stages = {k: round(statistics.median(v), 2) for k, v in stage_us.items()}
    if fused:  # one kernel does both: report it under one name
        stages["o_proj_allreduce_residual_fused"] = stages.pop("o_proj")
        stages.pop("allreduce_residual")
    kv_bytes = sum((n + 1) for n in att["lens"]) * lkv * d * 2
    act_bytes = B * lq * d * 2 * 2 + B * table.shape[1] * 4
    alg_bytes = kv_bytes + act_bytes
    peak, peak_kind = peaks()
    achieved = alg_bytes / (att_avg * 1e-6) / 1e9

    # e2e: through the public API with host buffers in and out every step.  The step's inputs
    # (x and the positions) travel as ONE pinned host buffer into one device buffer that x and
    # positions are views of, and the output comes back into pinned memory; the two copies and
    # the step are captured in one graph, so every replay moves 2 MB in and 2 MB out over PCIe.
    xb = B * H * 2
    io_dev = torch.empty(xb + B * 8, dtype=torch.uint8, device=dev)
    x_io = io_dev[:xb].view(torch.bfloat16).view(B, H)
    pos_io = io_dev[xb:].view(torch.int64)
    x_io.copy_(x)
    pos_io.copy_(positions)
    io_host = io_dev.cpu().pin_memory()
    out_host = torch.empty((B, H), dtype=torch.bfloat16).pin_memory()

    def step_e2e():
        io_dev.copy_(io_host, non_blocking=True)
        r = layer.step(x_io, pos_io, table, kc, vc, lens=lens, out=out if world == 1 else None)
        out_host.copy_(r, non_blocking=True)

    with torch.cuda.stream(s):
        step_e2e()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph_e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_e):
        step_e2e()
    for _ in range(3):
        graph_e.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        graph_e.replay()
    f1.record()
    torch.cuda.synchronize()
    e2e_us = f0.elapsed_time(f1) * 1000.0 / args.steps
    t = torch.tensor([e2e_us], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_us = float(t.item())

    traffic = None
    tp = ROOT / "profiles" / "traffic.json"
    if tp.exists():
        try:
            tr = json.loads(tp.read_text()).get("attn_decode_c4_per_kv_byte")
            if tr:
                traffic = round(tr * alg_bytes)
        except Exception:
            traffic = None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, cores, sample = cpu_layer_sample()
        cpu = {"value": round(v, 1), "unit": "us/step", "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(us, 2), "unit": "us/step", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1000, 4),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; decode-layer workload shapes)",
            "config": dict(WORKLOAD, parallelism=f"tp{world}"),
            "e2e": {"value": round(e2e_us, 2), "unit": "us/step", "h2d_bytes_per_step": B * H * 2 + B * 8,
                    "d2h_bytes_per_step": B * H * 2},
            "roofline": {"kernel": "okc::attn_decode_kernel<128,%d> + merge" % lkv, "bound": "hbm",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "alg_bytes_per_launch": alg_bytes, "launch_us": round(att_avg, 2),
                         "peak_source": peak_kind},
            "gpu_launches": layer.kernels_per_step(B) * args.steps,
            "stages_us": stages,
            "clocks": clocks, "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    del graph, graph_i, graph_e
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        layer.close()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="okc", choices=["okc", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    args = ap.parse_args(argv)
    sys.path.insert(0, str(ROOT))
    if args.impl == "reference":
        return run_reference(args)
    return run_okc(args)


if __name__ == "__main__":
    sys.exit(main())
