"""Small, self-contained cases of each kernel for Nsight Compute captures and quick timing.

Each case holds a few hundred MB on the device (more than the 126 MB L2, so DRAM counters
mean something) and runs `--warmup` untimed launches, then `--launches` timed ones, then
prints one JSON line with the CUDA-event time per launch and the algorithmic bytes.

    python -m okc_b200.profile_cases attn   [--warmup 2 --launches 3]
    python -m okc_b200.profile_cases gemv   --m 1 --k 8192 --n 10240
    python -m okc_b200.profile_cases moe    --t 8
    python -m okc_b200.profile_cases layer

The `tp` case runs on W ranks (one process per GPU, under torchrun) and times the O projection
+ tensor-parallel exchange variants at T = 128 tokens, H = 8192 per call (graphs of 20
back-to-back calls, the max over ranks); with OKC_TP_TRACE=1 it adds the %globaltimer phase
trace of CTA 0 of each kernel (ns from its griddepcontrol.wait) for its last three calls:

    OKC_TP_TRACE=1 python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 \
        --master-addr 127.0.0.1 --master-port 29513 -m okc_b200.profile_cases tp --kk 4096,1024

The `muse_layer` case times one Muse TP8/EP8 decode-layer step (problems/muse_decode_layer.py,
`--b` requests of `--l` new tokens, context ~U[ctx-lo, ctx-hi], `--window`, page `--page`) as
a CUDA graph of 10 steps, with the algorithmic bytes (dense weights, router, the local experts
the step routed to, the KV rows read):

    python -m okc_b200.profile_cases muse_layer --b 33 --l 1 --ctx-lo 10000 --ctx-hi 20000 --page 1

The `moe_ep` case (also under torchrun) times the expert-parallel MoE with `--t` tokens of its
own per rank (ExpertParallelMoE.forward_local: all-gather dispatch, local experts, NVLink
combine), and on rank 0 the single-GPU MoE over the same world * t tokens:

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \
        --master-port 29514 -m okc_b200.profile_cases moe_ep --t 32
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

from . import ops, synth


def _time(fn, warmup, launches):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(launches):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / launches


def case_attn(a):
    page = a.page or 16
    pool = max(a.pool, (a.b * (a.ctx_hi + page)) // page + 8)
    c = synth.attention_case(B=a.b, Hq=a.hq, Hkv=a.hkv, D=a.d, ctx=(a.ctx_lo, a.ctx_hi), page=page, pool_pages=pool,
                             device="cuda", seed=0)
    fn = lambda: ops.attn_decode(c["q"], c["k_cache"], c["v_cache"], c["page_table"], c["seq_lens"],  # noqa
                                 c["k_scale"], c["v_scale"], c["sm_scale"])
    us = _time(fn, a.warmup, a.launches)
    by = sum(c["lens"]) * a.hkv * a.d * 2
    return {"case": "attn", "B": a.b, "hq": a.hq, "hkv": a.hkv, "d": a.d, "page": page, "ctx": [a.ctx_lo, a.ctx_hi],
            "us": us, "kv_bytes": by,
            "gbs": by / us / 1e3}


def case_gemv(a):
    x, w = synth.projection_case(a.m, a.k, a.n, device="cuda")
    fn = lambda: ops.gemm(x, w, family=a.family)  # noqa: E731
    us = _time(fn, a.warmup, a.launches)
    by = 2 * a.n * a.k + 2 * a.m * a.k + 2 * a.m * a.n
    return {"case": "gemv", "m": a.m, "k": a.k, "n": a.n, "us": us, "bytes": by, "gbs": by / us / 1e3}


def case_moe(a):
    m = synth.moe_case(T=a.t, device="cuda", seed=0)
    ids, wts = ops.moe_route(m["x"], m["router"], 8)
    perm = ops.moe_permute(ids, 0, 64)

    def fn():
        i, w_ = ops.moe_route(m["x"], m["router"], 8)
        p = ops.moe_permute(i, 0, 64)
        return ops.moe_experts(m["x"], i, w_, p, m["w13"], m["w13_sf"], m["w13_gs"], m["w2"], m["w2_sf"],
                               m["w2_gs"], 0)
    us = _time(fn, a.warmup, a.launches)
    hit = int((perm["counts"] > 0).sum())
    per_expert = 3072 * 2048 + 3072 * 256 + 4096 * 768 + 4096 * 96
    by = hit * per_expert + a.t * 4096 * 4 + 64 * 4096 * 2
    return {"case": "moe", "t": a.t, "experts_hit": hit, "us": us, "bytes": by, "gbs": by / us / 1e3}


def case_muse_layer(a):
    from .problems import muse_decode_layer as prob
    w, d = synth.muse_layer_case(B=a.b, L=a.l, ctx=(a.ctx_lo, a.ctx_hi), page=a.page or 1, window=a.window,
                                 local_bias=0.0, seed=0, device="cuda")
    state = prob.prepare(w)
    T = a.b * a.l
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            _, _, ids = prob.kernel_fn(d, state)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    R = 10
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for _ in range(R):
            prob.kernel_fn(d, state)
    us = _time(gr.replay, 3, max(1, a.launches)) / R
    lids = torch.remainder(ids.long() - 32, 256)
    hit = int(torch.unique(lids[lids < 32]).numel())
    per_expert = 8192 * 2048 + 8192 * 256 + 4096 * 2048 + 4096 * 256
    dense = 2 * (2304 * 8192 + 8192 * 1024 + 4096 * 8192 + (1024 if T <= 8 else 8192) * 4096 + 2 * 256 * 8192)
    lens = d["seq_lens"].long() + a.l
    kv = int((lens.clamp(max=a.window + a.l - 1) if a.window else lens).sum()) * 2 * 2 * 64
    by = dense + hit * per_expert + kv
    return {"case": "muse_layer", "B": a.b, "L": a.l, "T": T, "ctx": [a.ctx_lo, a.ctx_hi], "page": a.page or 1,
            "window": a.window, "experts_hit": hit, "us": round(us, 2), "bytes": by, "gbs": round(by / us / 1e3, 1)}


def case_tp(a):
    import datetime

    import torch.distributed as dist

    from .comm import TPComm
    world, rank = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"])
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    T, H, R = 128, 8192, 20
    res = {"case": "tp", "world": world, "T": T, "H": H}
    for K in [int(k) for k in a.kk.split(",")]:
        comm = TPComm(T, H, oproj_k=K)
        g = torch.Generator(device="cuda").manual_seed(rank)
        x = torch.randn((T, K), generator=g, device="cuda").to(torch.bfloat16)
        w = (torch.randn((H, K), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        r = torch.randn((T, H), generator=g, device="cuda").to(torch.bfloat16)
        variants = {
            "fused": lambda: comm.oproj_allreduce_residual(x, w, r),
            "gemm+exchange": lambda: (ops.gemm(x, w, out_fp32=True, out=comm.partial), comm.allreduce_residual(r)),
            "gemm_fp32": lambda: ops.gemm(x, w, out_fp32=True, out=comm.partial),
            "exchange": lambda: comm.allreduce_residual(r),
        }
        for name, fn in variants.items():
            if name == "fused" and not comm.fused:
                continue
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for _ in range(3):
                    fn()
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            dist.barrier()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                for _ in range(R):
                    fn()
            for _ in range(3):
                gr.replay()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(5):
                gr.replay()
            e1.record()
            torch.cuda.synchronize()
            us = torch.tensor([e0.elapsed_time(e1) * 1000 / (5 * R)], device="cuda")
            dist.all_reduce(us, op=dist.ReduceOp.MAX)
            res[f"K{K}/{name}_us"] = round(float(us), 2)
            if name in ("fused", "exchange") and rank == 0:
                st = comm.trace_stamps()[1 if name == "fused" else 0]
                ep = int(comm.state[512 if name == "fused" else 0].item())
                if int(st[ep & 3][1]):
                    res[f"K{K}/{name}_trace_ns"] = [[int(v) - int(st[e & 3][1]) if int(v) else None
                                                     for v in st[e & 3].tolist()[:11]] for e in (ep - 2, ep - 1, ep)]
            del gr
            torch.cuda.synchronize()
            dist.barrier()
        res[f"K{K}/device_error"] = ops.read_device_error("tp", rank)
        comm.close()
    dist.barrier()
    dist.destroy_process_group()
    return res if rank == 0 else None


def case_moe_ep(a):
    """Expert-parallel MoE with each rank's own T tokens (forward_local) under torchrun: us per
    step (graph replays, max over ranks) and, on rank 0, the single-GPU MoE over the same W*T
    tokens for comparison."""
    import datetime

    import torch.distributed as dist

    from .comm import ExpertParallelMoE
    world, rank = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    T, R = a.t, 10
    m = synth.moe_case(T=world * T, device="cuda", seed=0)
    E = m["w13"].shape[0]
    el = E // world
    sl = slice(rank * el, (rank + 1) * el)
    ep = ExpertParallelMoE(m["router"], m["w13"][sl].contiguous(), m["w13_sf"][sl].contiguous(),
                           m["w13_gs"][sl].contiguous(), m["w2"][sl].contiguous(), m["w2_sf"][sl].contiguous(),
                           m["w2_gs"][sl].contiguous(), rank * el, 8)
    mine = m["x"][rank * T:(rank + 1) * T].contiguous()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            ep.forward_local(mine)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    dist.barrier()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for _ in range(R):
            ep.forward_local(mine)
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    us = torch.tensor([e0.elapsed_time(e1) * 1000 / (5 * R)], device="cuda")
    dist.all_reduce(us, op=dist.ReduceOp.MAX)
    res = {"case": "moe_ep", "world": world, "tokens_per_rank": T, "experts_per_rank": el,
           "ep_us": round(float(us), 2), "tokens_per_s": round(world * T / float(us) * 1e6),
           "device_error": ops.read_device_error("tp", rank)}
    del gr
    torch.cuda.synchronize()
    dist.barrier()
    if rank == 0:
        def one():
            i, w_ = ops.moe_route(m["x"], m["router"], 8)
            p_ = ops.moe_permute(i, 0, E)
            return ops.moe_experts(m["x"], i, w_, p_, m["w13"], m["w13_sf"], m["w13_gs"], m["w2"], m["w2_sf"],
                                   m["w2_gs"], 0)
        res["one_gpu_same_batch_us"] = round(_time(one, 3, 10), 2)
    dist.barrier()
    ep.close()
    dist.destroy_process_group()
    return res if rank == 0 else None


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["attn", "gemv", "moe", "tp", "moe_ep", "muse_layer"])
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--b", type=int, default=64)
    ap.add_argument("--ctx-lo", type=int, default=512)
    ap.add_argument("--ctx-hi", type=int, default=4096)
    ap.add_argument("--pool", type=int, default=1 << 14)
    ap.add_argument("--hq", type=int, default=64)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--k", type=int, default=8192)
    ap.add_argument("--n", type=int, default=10240)
    ap.add_argument("--family", type=int, default=0)
    ap.add_argument("--t", type=int, default=8)
    ap.add_argument("--l", type=int, default=1, help="muse_layer: new tokens per request")
    ap.add_argument("--page", type=int, default=0, help="page size (attn: 16, muse_layer: 1 when 0)")
    ap.add_argument("--d", type=int, default=128, help="attn: head dim")
    ap.add_argument("--window", type=int, default=0, help="muse_layer: sliding window (0: full)")
    ap.add_argument("--kk", default="1024", help="tp: comma-separated O-projection K per rank")
    a = ap.parse_args(argv)
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    res = {"attn": case_attn, "gemv": case_gemv, "moe": case_moe, "tp": case_tp, "moe_ep": case_moe_ep,
           "muse_layer": case_muse_layer}[a.case](a)
    if res is not None:
        print(json.dumps(res), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
