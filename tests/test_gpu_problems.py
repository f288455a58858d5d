"""GPU parity of the drop-in problem modules (okc_b200/problems) on the reference's own data
formats: the gated attention decode against the reference's own `attention()` output
(tests/golden/prefill_ops.pt) and against the oracle on reference-shaped inputs (16 q / 2 kv
heads, head_dim 64, page 1/16/64, kv_scale 1 and 1/64, RoPE on/off), the projection operator
on the reference's layer shapes, and the MoE operator with global ids and a local expert slice.
Tolerance: rtol 2e-2 / atol 2e-2 on bf16 outputs; untouched cache rows bit-exact."""

import math
from pathlib import Path

import pytest
import torch

from oracle import attention as oatt
from oracle import moe as omoe
from oracle import projection as oproj

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


def _close(out, exp, what, rel=1e-2):
    o, e = out.float().cpu(), exp.float().cpu()
    torch.testing.assert_close(o, e, rtol=2e-2, atol=2e-2, msg=what)
    assert (o - e).norm() / e.norm().clamp_min(1e-30) < rel, what


@pytest.mark.parametrize("i", range(6))
def test_attention_problem_matches_reference_output(i):
    """Cases 0-2: decode steps; 3: a sliding-window layer; 4-5: 8-token verify blocks (full and
    sliding window), each against the reference's own attention() output."""
    from okc_b200.problems import muse_attention_decode as prob
    c = torch.load(GOLD / "prefill_ops.pt", weights_only=False)["attention_cases"][i]
    cfg = dict(c["cfg"])
    L = cfg["q_len"]
    qkv = (c["x"] @ c["wqkv"].T).cuda()          # the reference computes qkv the same way
    s = torch.tensor(c["kv_scale"], dtype=torch.float32)
    seq = c.get("seq_lens", c["positions"].to(torch.int32))
    data = {"qkv": qkv.view(cfg["batch"], L, -1), "positions": c["positions"].cuda(),
            "cache_loc": c["cache_loc"].cuda(), "k_cache": c["k_cache_in"].clone().cuda(),
            "v_cache": c["v_cache_in"].clone().cuda(), "k_scale": s.cuda(), "v_scale": s.cuda(),
            "page_table": c["table"].cuda(), "seq_lens": seq.cuda(), "config": cfg}
    out = prob.kernel_fn(data)
    _close(out.view(cfg["batch"] * L, -1), c["out"], f"golden case {i}")
    # the cache rows the reference wrote: v exactly, k within one e4m3 step (RoPE'd fp32 values)
    ref_v = c["v_cache_out"].view(torch.uint8).view(-1, 2 * 64)
    got_v = data["v_cache"].cpu().view(torch.uint8).view(-1, 2 * 64)
    assert torch.equal(got_v, ref_v)
    torch.testing.assert_close(data["k_cache"].cpu().float(), c["k_cache_out"].float(), rtol=0.07, atol=2e-2)


def _muse_data(B, ctx, page, kv_scale, theta, seed, L=1, window=0):
    from okc_b200 import synth
    hq, hkv, d = 16, 2, 64
    g = torch.Generator(device="cuda").manual_seed(seed)
    lens = torch.randint(max(1, ctx // 2), ctx + 1, (B,), generator=g, device="cuda")
    lens_l = [int(v) for v in lens.tolist()]
    pool = sum(math.ceil((n + L) / page) for n in lens_l) + 3
    table = synth.paged_layout(lens_l, page, pool, g, "cuda", extra_tokens=L)
    kc = torch.empty((pool, page, hkv, d), dtype=torch.float8_e4m3fn, device="cuda")
    vc = torch.empty_like(kc)
    synth.fill_e4m3_normal(kc, g, torch.full((hkv,), kv_scale, device="cuda"))
    synth.fill_e4m3_normal(vc, g, torch.full((hkv,), kv_scale, device="cuda"))
    qkv = torch.randn((B * L, (2 * hq + 2 * hkv) * d), generator=g, device="cuda")
    qkv[:, :hq * d] *= 2
    qkv = qkv.to(torch.bfloat16)
    pos = (lens.long()[:, None] + torch.arange(L, device="cuda")).reshape(-1)  # the block's positions
    cfg = {"batch": B, "q_len": L, "num_q_heads": hq, "num_kv_heads": hkv, "head_dim": d, "page_size": page,
           "window": window, "rope_theta": theta, "qk_scale_factor": 5.4730064863875, "sm_scale": 0.125,
           "kv_scale": kv_scale}
    s = torch.tensor(kv_scale, dtype=torch.float32, device="cuda")
    return {"qkv": qkv.view(B, L, -1), "positions": pos, "k_cache": kc, "v_cache": vc, "k_scale": s, "v_scale": s,
            "page_table": table, "seq_lens": lens.to(torch.int32), "config": cfg}


@pytest.mark.parametrize("B,ctx,page,kv_scale,theta,L,window",
                         [(1, 10, 1, 1.0, 5e5, 1, 0), (3, 2047, 16, 1.0, 0.0, 1, 0), (4, 3000, 64, 1.0, 5e5, 1, 0),
                          (2, 9000, 64, 1 / 64, 0.0, 1, 0), (16, 5000, 1, 1.0, 0.0, 1, 0), (5, 700, 16, 0.5, 1e4, 1, 0),
                          # the reference's scored workload: sliding-window (2048) layers, verify blocks of 8
                          (8, 6000, 1, 1.0, 5e5, 1, 2048), (3, 4000, 1, 1 / 64, 5e5, 8, 2048),
                          (2, 20000, 64, 1.0, 0.0, 8, 0), (5, 5000, 16, 1.0, 5e5, 8, 2048)])
def test_attention_problem_reference_shapes(B, ctx, page, kv_scale, theta, L, window):
    from okc_b200.problems import muse_attention_decode as prob
    data = _muse_data(B, ctx, page, kv_scale, theta, seed=B + ctx, L=L, window=window)
    kc_ref, vc_ref = data["k_cache"].cpu().clone(), data["v_cache"].cpu().clone()
    cpu = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in data.items()}
    exp = oatt.muse_attention(cpu["qkv"].view(B * L, -1), cpu["positions"], cpu["page_table"], kc_ref, vc_ref,
                              cpu["k_scale"], cpu["v_scale"], data["config"])
    out = prob.kernel_fn(data)
    _close(out.view(B * L, -1), exp, f"B{B} ctx{ctx} P{page} s{kv_scale} theta{theta} L{L} window{window}")


@pytest.mark.parametrize("layer,n,k", [("qkv_gate", 2304, 8192), ("o", 8192, 1024), ("pooler", 4096, 8192),
                                       ("unpooler", 8192, 4096)])
@pytest.mark.parametrize("m", [1, 8, 16, 32, 128, 256])
def test_projection_problem(layer, n, k, m):
    from okc_b200.problems import muse_bf16_proj as prob
    g = torch.Generator(device="cuda").manual_seed(m + n)
    w = (torch.randn((n, k), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    state = prob.prepare({layer: w})
    nn = 1024 if layer == "unpooler" and m <= 8 else n   # muse_bf16_proj/projection/shapes.py:16-20
    x = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    y = prob.kernel_fn({"x": x, "config": {"layer": layer, "m": m, "n": nn, "k": k}}, state)
    assert y.shape == (m, nn)
    _close(y, oproj.gemm(x.cpu(), w[:nn].cpu()), f"{layer} m{m}", rel=5e-3)


def test_moe_problem_global_ids_local_slice():
    from okc_b200 import synth
    from okc_b200.problems import muse_moe_w4a16 as prob
    bank = synth.moe_case(T=4, E=64, H=4096, I=1536, device="cuda", seed=5)
    state = prob.prepare({k: bank[k] for k in ("w13", "w13_sf", "w13_gs", "w2", "w2_sf", "w2_gs")})
    g = torch.Generator(device="cuda").manual_seed(1)
    ids = torch.stack([torch.randperm(64, generator=g, device="cuda")[:8] for _ in range(4)]).to(torch.int32)
    wts = torch.rand((4, 8), generator=g, device="cuda")
    wts = wts / wts.sum(1, keepdim=True)
    cfg = {"bs": 4, "d_hidden": 4096, "d_expert": 1536, "n_experts": 64, "local_start": 16, "local_count": 32,
           "top_k": 8, "sharding": "ep2"}
    out = prob.kernel_fn({"hidden_states": bank["x"], "topk_ids": ids, "topk_weights": wts, "config": cfg}, state)
    c = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in bank.items()}
    sl = slice(16, 48)
    exp = omoe.experts(c["x"], ids.cpu(), wts.cpu(), c["w13"][sl], c["w13_sf"][sl], c["w13_gs"][sl], c["w2"][sl],
                       c["w2_sf"][sl], c["w2_gs"][sl], expert_lo=16)
    _close(out, exp, "moe problem")


@pytest.mark.parametrize("M", [4, 64])
def test_moe_problem_post_norm(M):
    """The problem module with the bank's post_norm_w: Muse's `_finalize` applied (prepare keeps
    1 + w in fp32 as the reference does)."""
    from okc_b200 import synth
    from okc_b200.problems import muse_moe_w4a16 as prob
    bank = synth.moe_case(T=M, E=64, H=4096, I=1536, device="cuda", seed=6)
    g = torch.Generator(device="cuda").manual_seed(2)
    post = (torch.randn(4096, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    weights = {k: bank[k] for k in ("w13", "w13_sf", "w13_gs", "w2", "w2_sf", "w2_gs")}
    weights["post_norm_w"] = post
    state = prob.prepare(weights)
    ids = torch.stack([torch.randperm(64, generator=g, device="cuda")[:8] for _ in range(M)]).to(torch.int32)
    wts = torch.rand((M, 8), generator=g, device="cuda")
    wts = wts / wts.sum(1, keepdim=True)
    cfg = {"bs": M, "d_hidden": 4096, "d_expert": 1536, "n_experts": 64, "local_start": 0, "local_count": 32,
           "top_k": 8, "sharding": "ep2"}
    out = prob.kernel_fn({"hidden_states": bank["x"], "topk_ids": ids, "topk_weights": wts, "config": cfg}, state)
    c = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in bank.items()}
    sl = slice(0, 32)
    exp = omoe.experts(c["x"], ids.cpu(), wts.cpu(), c["w13"][sl], c["w13_sf"][sl], c["w13_gs"][sl], c["w2"][sl],
                       c["w2_sf"][sl], c["w2_gs"][sl], expert_lo=0, post_gain=post.cpu().float() + 1.0)
    _close(out, exp, "moe problem post-norm")
