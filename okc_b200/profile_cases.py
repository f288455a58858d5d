"""Small, self-contained cases of each kernel for Nsight Compute captures and quick timing.

Each case holds a few hundred MB on the device (more than the 126 MB L2, so DRAM counters
mean something) and runs `--warmup` untimed launches, then `--launches` timed ones, then
prints one JSON line with the CUDA-event time per launch and the algorithmic bytes.

    python -m okc_b200.profile_cases attn   [--warmup 2 --launches 3]
    python -m okc_b200.profile_cases gemv   --m 1 --k 8192 --n 10240
    python -m okc_b200.profile_cases moe    --t 8
    python -m okc_b200.profile_cases layer
"""

from __future__ import annotations

import argparse
import json
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
    c = synth.attention_case(B=a.b, Hq=a.hq, Hkv=a.hkv, ctx=(a.ctx_lo, a.ctx_hi), pool_pages=a.pool, device="cuda",
                             seed=0)
    fn = lambda: ops.attn_decode(c["q"], c["k_cache"], c["v_cache"], c["page_table"], c["seq_lens"],  # noqa
                                 c["k_scale"], c["v_scale"], c["sm_scale"])
    us = _time(fn, a.warmup, a.launches)
    by = sum(c["lens"]) * a.hkv * 128 * 2
    return {"case": "attn", "B": a.b, "hq": a.hq, "hkv": a.hkv, "ctx": [a.ctx_lo, a.ctx_hi], "us": us, "kv_bytes": by,
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


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["attn", "gemv", "moe"])
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
    a = ap.parse_args(argv)
    torch.cuda.set_device(0)
    res = {"attn": case_attn, "gemv": case_gemv, "moe": case_moe}[a.case](a)
    print(json.dumps(res), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
