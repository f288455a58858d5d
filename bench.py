#!/usr/bin/env python
"""Decode-layer benchmark: one decode step of a layer with hidden
8192, 64 query / 8 KV heads, head_dim 128, batch 128, context lengths U[1024, 8192], page 16.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl okc|reference]

N > 1 runs under torchrun, one rank per GPU, tensor parallel over the heads; the row-parallel O
projection and the sum of the ranks' partials + residual run as one kernel over NVLink peer
memory (okc_tp_oproj_allreduce_residual).  Rank 0 prints ONE JSON line.

value     = device time per step (CUDA events around K graph replays, max over ranks), µs.  Where
            one rank's working set (weights + its KV heads) is under 4x the 126 MB L2 (N >= 4),
            the replays rotate over several independent sets of weights and caches.
e2e       = the same step through the public API (DecodeLayer.step driven by
            okc_b200.pipeline.HostPipeline) with the step's input copied in from pinned host
            memory and its output copied back every step, µs per step over K steps: step k's
            copy-in and step k-1's copy-out overlap step k's compute (double-buffered, three
            streams).  serial_value: the same with copy in, step and copy out in series (one
            graph).  At N > 1 each rank copies out the 1/N of the output rows it owns; it copies
            in the whole x when pipelined (the copy overlaps the previous step), and its 1/N of
            the x rows, gathered over NVLink by an NCCL all-gather in the step, when serial.
roofline  = the attention kernel (the dominant kernel) measured with CUDA events inside an
            instrumented copy of the step graph: algorithmic KV bytes / duration vs
            MEASURED_PEAKS.json hbm_gbs; stages_us = per-stage times from the same copy.
rooflines = (N = 1) standalone records of the other workloads: paged attention decode (batch 64,
            ctx U[512, 32768]), the projection at M = 1 and M = 128 (K 8192, N 10240), the
            W4A16 MoE at T = 8 and T = 256 and the Muse decode-layer drop-in at 33 tokens (page 1),
            each µs, algorithmic bytes and fraction of HBM.
cpu_baseline / --impl reference = the oracle (the reference's PyTorch path restated, CPU
            fp32) on the host cores: one warm-up, then the median of 5 samples; a sample runs
            the projections at all 128 tokens and the attention of 8 of the 128 sequences,
            scaled by the ratio of the tokens of all 128 sequences to those of the 8.
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
            "l2": "no flush: inputs larger than L2 every step (1 GPU: 1.5 GB of KV cache + weights; where a "
                  "rank's share is under 4x the 126 MB L2, replays rotate over several input sets)"}
L2_BYTES = 126 << 20


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
    """Times the oracle layer on the host: RMSNorm + QKV and the O projection at all B tokens,
    RoPE/append + attention over the first `sample_seqs` sequences of a batch whose context
    lengths are drawn like the GPU arm's (U[1024, 8192]); the attention time is scaled by
    sum(len + 1) over all B sequences / the same sum over the sample.  The cache is laid out
    as on the GPU: a seeded random permutation of the pool's pages, per-KV-head scales
    U[0.5, 2], e4m3(N(0, 1) / scale) codes.  Returns (us per step, threads, description)."""
    import torch
    from oracle import attention as oatt
    from oracle.projection import gemm, rmsnorm
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    H, Hq, Hkv, D, P = 8192, 64, 8, 128, 16
    x = torch.randn((B, H), generator=g).to(torch.bfloat16)
    nw = (1.0 + 0.02 * torch.randn((H,), generator=g)).to(torch.bfloat16)
    wqkv = (torch.randn(((Hq + 2 * Hkv) * D, H), generator=g) * 0.02).to(torch.bfloat16)
    wo = (torch.randn((H, Hq * D), generator=g) * 0.02).to(torch.bfloat16)
    lens_all = torch.randint(1024, 8193, (B,), generator=g)
    lens = lens_all[:sample_seqs]
    pages = [math.ceil((int(n) + 1) / P) for n in lens]
    pool = sum(pages) + 64
    perm = torch.randperm(pool, generator=g).to(torch.int32)
    table = torch.full((sample_seqs, max(pages)), -1, dtype=torch.int32)
    off = 0
    for b, n in enumerate(pages):
        table[b, :n] = perm[off:off + n]
        off += n
    ks = torch.rand(Hkv, generator=g) * 1.5 + 0.5
    vs = torch.rand(Hkv, generator=g) * 1.5 + 0.5
    kc = (torch.randn((pool, P, Hkv, D), generator=g) / ks[None, None, :, None]).to(torch.float8_e4m3fn)
    vc = (torch.randn((pool, P, Hkv, D), generator=g) / vs[None, None, :, None]).to(torch.float8_e4m3fn)
    pos = lens.long()
    factor = float((lens_all + 1).sum()) / float((lens + 1).sum())
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
    step_s = (t1 - t0) + (t2 - t1) * factor + (t3 - t2)
    return step_s * 1e6, torch.get_num_threads(), (
        f"oracle layer (torch fp32 on the host): RMSNorm+QKV and O-proj at 128 tokens; RoPE/append + "
        f"attention over {sample_seqs} of 128 sequences (ctx U[1024,8192], permuted page table, per-head "
        f"scales) scaled by their token ratio x{factor:.2f}")


def cpu_baseline(runs=5):
    """One warm-up sample, then the median of `runs` samples."""
    cpu_layer_sample(seed=1)
    vals = []
    for i in range(runs):
        v, cores, sample = cpu_layer_sample(seed=2 + i)
        vals.append(v)
    return statistics.median(vals), cores, f"median of {runs} after 1 warm-up; " + sample


def run_reference(args):
    """--impl reference: the reference's own (PyTorch, CPU) path restated as the oracle."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    for i in range(max(args.warmup, 1)):
        cpu_layer_sample(seed=100 + i)
    vals = []
    cores = 1
    sample = ""
    for i in range(args.steps):
        v, cores, sample = cpu_layer_sample(seed=2 + i)
        vals.append(v)
    val = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": round(val, 1), "unit": "us/step",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(val / 1000, 3), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded; decode-layer workload shapes)",
            "config": dict(WORKLOAD, parallelism=f"tp{args.gpus}"),
            "cpu_baseline": {"value": round(val, 1), "unit": "us/step", "cores": cores, "kind": "port",
                             "sample": f"median of {args.steps} samples, rank 0 only, on the host cores; " + sample},
            "e2e": {"value": round(val, 1), "unit": "us/step", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------- GPU arm
def _graph_us(calls, reps=7):
    """Captures `calls` (a list of callables, each one operator call on the current stream) in
    one CUDA graph, replays it `reps` times after 3 warm-up replays and returns the median
    device time per call in µs (CUDA events on the replaying stream)."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for c in calls:
            c()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for c in calls:
            c()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    per = []
    for _ in range(reps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        per.append(e0.elapsed_time(e1) * 1000.0 / len(calls))
    del g
    return statistics.median(per)


def _record(us, alg_bytes, peak, peak_kind, kernel, config):
    gbs = alg_bytes / (us * 1e-6) / 1e9
    return {"kernel": kernel, "config": config, "us": round(us, 2), "alg_bytes": int(alg_bytes),
            "achieved_gbs": round(gbs, 1), "peak_gbs": peak, "frac": round(gbs / peak, 4), "bound": "hbm",
            "peak_source": peak_kind}


def extra_rooflines(dev, peak, peak_kind):
    """Standalone roofline records of the path's other workloads (1 GPU).  Inputs are larger
    than L2 on every call: the attention cache is 4 GB, and the projection weights and expert
    banks rotate over several copies (>= 500 MB between two uses of one copy)."""
    import torch
    from okc_b200 import ops, synth
    recs = {}
    # paged FP8 attention decode: batch 64, 64q/8kv, D 128, ctx U[512, 32768], P 16, pool 2^17 pages
    a = synth.attention_case(64, 64, 8, 128, (512, 32768), 16, 1 << 17, seed=7, device=dev)
    kv = sum(a["lens"]) * 8 * 128 * 2
    act = 64 * 64 * 128 * 2 * 2 + a["page_table"].numel() * 4 + 64 * 4
    us = _graph_us([lambda: ops.attn_decode(a["q"], a["k_cache"], a["v_cache"], a["page_table"], a["seq_lens"],
                                            a["k_scale"], a["v_scale"], a["sm_scale"])] * 8)
    recs["attn_decode_b64_ctx512-32k"] = _record(us, kv + act, peak, peak_kind, "okc::attn_decode_kernel<128,8> + merge",
                                                 "batch 64, 64q/8kv, D128, ctx U[512,32768], P16, pool 2^17 pages")
    del a
    torch.cuda.empty_cache()
    # BF16 projection (K 8192, N 10240) at M = 1 and M = 128, three weight copies in rotation
    K, N = 8192, 10240
    ws = [synth.projection_case(1, K, N, seed=20 + i, device=dev)[1] for i in range(3)]
    for M in (1, 128):
        x = torch.randn((M, K), device=dev).to(torch.bfloat16)
        outs = [torch.empty((M, N), dtype=torch.bfloat16, device=dev) for _ in ws]
        calls = [(lambda w=w, o=o: ops.gemm(x, w, out=o)) for w, o in zip(ws, outs)] * 4
        us = _graph_us(calls)
        kern = "okc::skinny_gemm_kernel<1>" if M == 1 else "okc::tc_gemm (tcgen05 stream-K) + tc_reduce"
        recs[f"gemm_bf16_m{M}_k8192_n10240"] = _record(us, 2 * N * K + 2 * M * K + 2 * M * N, peak, peak_kind, kern,
                                                       f"x [{M},8192] bf16, W [10240,8192] bf16, 3 weight copies")
    del ws
    torch.cuda.empty_cache()
    # W4A16 MoE (route + permute + experts + combine): E 64, top-8, H 4096, I 1536, two banks in rotation
    banks = [synth.moe_case(T=256, seed=30 + i, device=dev) for i in range(2)]
    per_expert = 2 * 1536 * 4096 // 2 + 2 * 1536 * 4096 // 16 + 4096 * 1536 // 2 + 4096 * 1536 // 16
    for T in (8, 256):
        calls, hit = [], []
        for bk in banks:
            x = bk["x"][:T]

            def moe(bk=bk, x=x):
                ids, wts = ops.moe_route(x, bk["router"], 8)
                perm = ops.moe_permute(ids, 0, 64)
                return ops.moe_experts(x, ids, wts, perm, bk["w13"], bk["w13_sf"], bk["w13_gs"], bk["w2"],
                                       bk["w2_sf"], bk["w2_gs"], 0)
            ids, _ = ops.moe_route(x, bk["router"], 8)
            hit.append(int(torch.unique(ids).numel()))
            calls.append(moe)
        us = _graph_us(calls * 3)
        alg = statistics.mean(hit) * per_expert + T * 4096 * 2 * 2 + 64 * 4096 * 2
        recs[f"moe_w4a16_t{T}"] = _record(us, alg, peak, peak_kind, "okc::route/permute/moe experts/combine",
                                          f"T {T}, E 64 top-8 softmax, H 4096, I 1536, NVFP4 weights; "
                                          f"{statistics.mean(hit):.1f} distinct experts hit")
    del banks
    torch.cuda.empty_cache()
    # Muse TP8/EP8 decode layer drop-in (problems/muse_decode_layer.py): 33 requests x 1 token,
    # ctx U[10000, 20000], page 1, no local routing preference; 1.1 GB of weights per step
    from okc_b200.problems import muse_decode_layer as muse
    w, d = synth.muse_layer_case(B=33, L=1, ctx=(10000, 20000), page=1, local_bias=0.0, seed=40, device=dev)
    st = muse.prepare(w)
    _, _, ids = muse.kernel_fn(d, st)
    lids = torch.remainder(ids.long() - 32, 256)
    hit = int(torch.unique(lids[lids < 32]).numel())
    us = _graph_us([lambda: muse.kernel_fn(d, st)] * 4)
    dense = 2 * (2304 * 8192 + 8192 * 1024 + 4096 * 8192 + 8192 * 4096 + 2 * 256 * 8192)
    per_exp = 8192 * 2048 + 8192 * 256 + 4096 * 2048 + 4096 * 256
    kv = int((d["seq_lens"].long() + 1).sum()) * 2 * 2 * 64
    recs["muse_decode_layer_t33_page1"] = _record(us, dense + hit * per_exp + kv, peak, peak_kind,
                                                  "problems/muse_decode_layer.py (23 okc kernels per step)",
                                                  f"33 x 1 token, ctx U[10000,20000], page 1, 16q/2kv D64, "
                                                  f"32 local NVFP4 experts (H = I = 4096), {hit} hit")
    del w, d, st
    torch.cuda.empty_cache()
    return recs


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
    H, d, hq, hkv = cfg.hidden, cfg.head_dim, cfg.num_q_heads, cfg.num_kv_heads
    lq, lkv = hq // world, hkv // world

    def make_set(i):
        """One independent input set (identical on every rank: same seeds, same device type):
        this rank's paged cache, the layer weights (sharded by DecodeLayer) and x."""
        att = synth.attention_case(B, lq, lkv, d, (1024, 8192), cfg.page_size, 1 << 17, seed=i, device=dev,
                                   extra_tokens=1)
        g = torch.Generator(device=dev).manual_seed(1 + 1000 * i)
        x = torch.randn((B, H), generator=g, device=dev).to(torch.bfloat16)
        norm_w = (1.0 + 0.02 * torch.randn((H,), generator=g, device=dev)).to(torch.bfloat16)
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
        return {"att": att, "layer": layer, "x": x, "positions": positions, "table": att["page_table"],
                "kc": att["k_cache"], "vc": att["v_cache"], "lens": (positions + 1).to(torch.int32)}

    sets = [make_set(0)]
    L0 = sets[0]["layer"]
    kv_bytes = sum((n + 1) for n in sets[0]["att"]["lens"]) * lkv * d * 2
    rank_bytes = (L0.wqkv.numel() + L0.wo.numel()) * 2 + kv_bytes
    nsets = 1 if rank_bytes >= 4 * L2_BYTES else math.ceil(4 * L2_BYTES / rank_bytes)
    for i in range(1, nsets):
        st = make_set(i)
        st["layer"]._comms = L0._comms  # one exchange group serves every set (used in stream order)
        sets.append(st)
    out = torch.empty((B, H), dtype=torch.bfloat16, device=dev)

    def step(st):
        # at TP > 1 the result is the exchange group's replicated output buffer (no extra copy)
        return st["layer"].step(st["x"], st["positions"], st["table"], st["kc"], st["vc"], lens=st["lens"],
                                out=out if world == 1 else None)

    # warm-up (eager), then capture one step per set; in-graph external events bracket attention
    for _ in range(max(args.warmup, 3)):
        for st in sets:
            step(st)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    s0 = sets[0]
    x, positions, table, kc, vc, lens = s0["x"], s0["positions"], s0["table"], s0["kc"], s0["vc"], s0["lens"]
    layer = L0
    ev_a0 = torch.cuda.Event(enable_timing=True, external=True)
    ev_a1 = torch.cuda.Event(enable_timing=True, external=True)
    # stage boundaries inside the graph (external events): norm, QKV + RoPE/append,
    # attention, O projection, exchange + residual
    ev_s = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(4)]
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
        return out

    # Graphs of the same step: `graphs[i]` is the public API call (DecodeLayer.step) on input set
    # i with no event inside, so programmatic dependent launch chains every kernel to the next;
    # they are what `value` times.  `graph_i` adds external events between the stages (an event
    # node breaks the programmatic chain there) for the attention roofline and `stages_us`.
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step_instrumented()
        for st in sets:
            step(st)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph_i = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_i):
        step_instrumented()
    graphs = []
    for st in sets:
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            step(st)
        graphs.append(gr)
    for _ in range(max(args.warmup, 3)):
        graph_i.replay()
        for gr in graphs:
            gr.replay()
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
    for k in range(args.steps):
        graphs[k % nsets].replay()
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

    # attention and stage durations from the instrumented graph (one replay per sample; the other
    # sets are replayed in between so that set 0 is not served from L2)
    att_us = []
    stage_us = {"norm": [], "qkv_rope_append": [], "attention": [], "o_proj": [], "allreduce_residual": []}
    for _ in range(args.steps):
        for gr in graphs[1:]:
            gr.replay()
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
    act_bytes = B * lq * d * 2 * 2 + B * table.shape[1] * 4
    alg_bytes = kv_bytes + act_bytes
    peak, peak_kind = peaks()
    achieved = alg_bytes / (att_avg * 1e-6) / 1e9

    # e2e: through the public API with host buffers in and out every step, on input set 0.  The
    # step's input travels as ONE pinned host buffer into one device buffer (x rows, positions);
    # the output comes back into pinned memory.  At N > 1 rank r copies in only its 1/N of the x
    # rows (gathered over NVLink into the full x by an NCCL all-gather in the step) and copies out
    # only the 1/N of the output rows it owns.  Two forms, each K steps timed with CUDA events,
    # max over ranks: serial (copy in, step, copy out as one graph, one step after another) and
    # the headline, okc_b200.pipeline.HostPipeline (step k's copy-in and step k-1's copy-out run
    # on their own streams while step k computes; every step still copies its input in and its
    # output out).
    rows = B // world
    r0 = rank * rows
    xb = rows * H * 2
    io_dev = torch.empty(xb + B * 8, dtype=torch.uint8, device=dev)
    x_loc = io_dev[:xb].view(torch.bfloat16).view(rows, H)
    pos_io = io_dev[xb:].view(torch.int64)
    x_loc.copy_(x[r0:r0 + rows])
    pos_io.copy_(positions)
    io_host = io_dev.cpu().pin_memory()
    out_host = torch.empty((rows, H), dtype=torch.bfloat16).pin_memory()
    x_full = torch.empty((B, H), dtype=torch.bfloat16, device=dev) if world > 1 else x_loc

    def step_e2e():
        io_dev.copy_(io_host, non_blocking=True)
        if world > 1:
            dist.all_gather_into_tensor(x_full, x_loc, group=group)
        r = layer.step(x_full, pos_io, table, kc, vc, lens=lens, out=out if world == 1 else None)
        out_host.copy_(r[r0:r0 + rows], non_blocking=True)

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
    e2e_serial_us = f0.elapsed_time(f1) * 1000.0 / args.steps

    from okc_b200.pipeline import HostPipeline

    # Pipelined, every rank copies in the whole x: the tensor-parallel step needs all rows on
    # every rank, and the copy overlaps the previous step, where an all-gather would sit inside
    # the step (measured at 2 GPUs: 247 us/step with the 1/N copy + all-gather vs 207 device).
    xfb = B * H * 2
    io_full_host = torch.cat([x.contiguous().view(torch.uint8).reshape(-1).cpu(),
                              positions.contiguous().view(torch.uint8).reshape(-1).cpu()]).pin_memory()

    def step_io(inp):
        x_in = inp[:xfb].view(torch.bfloat16).view(B, H)
        pos_in = inp[xfb:].view(torch.int64)
        r = layer.step(x_in, pos_in, table, kc, vc, lens=lens)
        # at N > 1 the step's result is the exchange's shared buffer: copy the owned rows out of
        # it, so that the next step cannot overwrite them while they travel to the host
        return r[r0:r0 + rows].clone() if world > 1 else r

    pipe = HostPipeline(step_io, xfb + B * 8, dev)
    for _ in range(max(3, args.warmup)):
        pipe.submit(io_full_host, out_host)
    pipe.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    p0 = torch.cuda.Event(enable_timing=True)
    p1 = torch.cuda.Event(enable_timing=True)
    p0.record(pipe.s_in)
    for _ in range(args.steps):
        pipe.submit(io_full_host, out_host)
    p1.record(pipe.s_out)
    torch.cuda.synchronize()
    e2e_us = p0.elapsed_time(p1) * 1000.0 / args.steps
    pipe.close()
    del pipe
    t = torch.tensor([e2e_us, e2e_serial_us], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_us, e2e_serial_us = (float(v) for v in t.tolist())

    traffic = None
    tp = ROOT / "profiles" / "traffic.json"
    if tp.exists():
        try:
            tr = json.loads(tp.read_text()).get("attn_decode_c4_per_kv_byte")
            if tr:
                traffic = round(tr * alg_bytes)
        except Exception:
            traffic = None

    extra = None
    if rank == 0 and world == 1 and not args.no_extra:
        graph_e = None
        extra = extra_rooflines(dev, peak, peak_kind)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, cores, sample = cpu_baseline()
        cpu = {"value": round(v, 1), "unit": "us/step", "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(us, 2), "unit": "us/step", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1000, 4),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; decode-layer workload shapes)",
            "config": dict(WORKLOAD, parallelism=f"tp{world}"),
            "input_sets": nsets,
            "e2e": {"value": round(e2e_us, 2), "unit": "us/step", "h2d_bytes_per_step": xfb + B * 8,
                    "d2h_bytes_per_step": rows * H * 2,
                    "io": "whole batch" if world == 1 else f"whole x in per rank, 1/{world} of the output rows out",
                    "overlap": "HostPipeline: copy-in of step k and copy-out of step k-1 overlap step k",
                    "serial_value": round(e2e_serial_us, 2),
                    "serial_io": "whole batch" if world == 1 else
                    f"1/{world} of the x rows in per rank + NCCL all-gather, 1/{world} of the output rows out"},
            "roofline": {"kernel": "okc::attn_decode_kernel<128,%d> + merge" % lkv, "bound": "hbm",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "alg_bytes_per_launch": alg_bytes, "launch_us": round(att_avg, 2),
                         "peak_source": peak_kind},
            "rooflines": extra,
            "gpu_launches": layer.kernels_per_step(B) * args.steps,
            "stages_us": stages,
            "clocks": clocks, "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    del graphs, graph_i, graph_e  # graphs holding NCCL calls go before the process group
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
    ap.add_argument("--no-extra", action="store_true", help="skip the standalone roofline records")
    args = ap.parse_args(argv)
    sys.path.insert(0, str(ROOT))
    if args.impl == "reference":
        return run_reference(args)
    return run_okc(args)


if __name__ == "__main__":
    sys.exit(main())
