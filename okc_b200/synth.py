"""Seeded synthetic workloads with the shapes and value distributions of the decode-path
workloads (there is no public dataset on this path; every input is synthetic).

All generators take a torch device and a seed and use a generator on that device, so the
large paged caches are produced directly in HBM.  The same seed gives the same tensors
on the same device type.
"""

from __future__ import annotations

import math

import torch

E4M3 = torch.float8_e4m3fn


def _gen(device, seed: int) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(seed)


def fill_e4m3_normal(t: torch.Tensor, g: torch.Generator, scale: torch.Tensor | None = None,
                     chunk_rows: int = 1 << 16) -> None:
    """t: e4m3 [rows, ..., Hkv, D]; fills with e4m3(N(0,1) / scale[h]) chunk by chunk."""
    flat = t.view(t.shape[0], -1)
    per_row = flat.shape[1]
    for r0 in range(0, flat.shape[0], chunk_rows):
        r1 = min(flat.shape[0], r0 + chunk_rows)
        v = torch.randn((r1 - r0, per_row), generator=g, device=t.device)
        if scale is not None:
            hkv, d = t.shape[-2], t.shape[-1]
            v = (v.view(r1 - r0, -1, hkv, d) / scale.view(1, 1, hkv, 1)).view(r1 - r0, per_row)
        flat[r0:r1] = v.to(E4M3)


def paged_layout(seq_lens: list[int], page: int, pool_pages: int, g: torch.Generator, device,
                 extra_tokens: int = 0):
    """Seeded random permutation of the page pool; sequence b owns the next
    ceil((len_b + extra) / page) pages of it (no sharing), unused table entries are -1
    (muse_attention_decode/tools/bench_tail.py:34-39 builds its tables the same way)."""
    need = [math.ceil((n + extra_tokens) / page) for n in seq_lens]
    if sum(need) > pool_pages:
        raise ValueError(f"pool of {pool_pages} pages too small for {sum(need)}")
    perm = torch.randperm(pool_pages, generator=g, device=device).to(torch.int32)
    max_pages = max(1, max(need))
    table = torch.full((len(seq_lens), max_pages), -1, dtype=torch.int32, device=device)
    off = 0
    for b, n in enumerate(need):
        table[b, :n] = perm[off:off + n]
        off += n
    return table


def attention_case(B=64, Hq=64, Hkv=8, D=128, ctx=(512, 32768), page=16, pool_pages=1 << 17,
                   seed=0, device="cuda", scale_range=(0.5, 2.0), extra_tokens=0, fill=True):
    """Attention-decode workload: q bf16 ~N(0,1) [B, Hq, D]; ctx ~U[lo, hi]; e4m3 caches
    [pool, P, Hkv, D] of N(0,1)/scale_h codes; per-head scales ~U[0.5, 2]; sm_scale 1/sqrt(D)."""
    g = _gen(device, seed)
    lo, hi = ctx
    seq = torch.randint(lo, hi + 1, (B,), generator=g, device=device)
    seq_lens = [int(v) for v in seq.tolist()]
    table = paged_layout(seq_lens, page, pool_pages, g, device, extra_tokens)
    k_scale = (torch.rand((Hkv,), generator=g, device=device) * (scale_range[1] - scale_range[0])
               + scale_range[0]).float()
    v_scale = (torch.rand((Hkv,), generator=g, device=device) * (scale_range[1] - scale_range[0])
               + scale_range[0]).float()
    k_cache = torch.empty((pool_pages, page, Hkv, D), dtype=E4M3, device=device)
    v_cache = torch.empty_like(k_cache)
    if fill:
        fill_e4m3_normal(k_cache, g)
        fill_e4m3_normal(v_cache, g)
    q = torch.randn((B, Hq, D), generator=g, device=device).to(torch.bfloat16)
    return {"q": q, "k_cache": k_cache, "v_cache": v_cache, "page_table": table,
            "seq_lens": torch.tensor(seq_lens, dtype=torch.int32, device=device),
            "k_scale": k_scale, "v_scale": v_scale, "sm_scale": 1.0 / math.sqrt(D),
            "lens": seq_lens}


def projection_case(M, K, N, seed=0, device="cuda"):
    """Projection workload: x [M,K] ~N(0,1), W [N,K] ~N(0, 0.02), bf16."""
    g = _gen(device, seed)
    x = torch.randn((M, K), generator=g, device=device).to(torch.bfloat16)
    w = (torch.randn((N, K), generator=g, device=device) * 0.02).to(torch.bfloat16)
    return x, w


def moe_case(T, E=64, H=4096, I=1536, topk=8, seed=0, device="cuda", gs13=(0.006, 0.010),
             gs2=(0.02, 0.03)):
    """W4A16 MoE workload: router Wr [E,H] ~N(0,0.02) bf16; uniformly random E2M1 codes
    (random bytes) for W13 [E, 2I, H/2] and W2 [E, H, I/2]; e4m3 block scales ~U[0.25, 1]
    per 16-element K-group; one fp32 global scale per expert (its value is not given by the
    config: W13 ~U[0.006, 0.010], W2 ~U[0.02, 0.03], which keep h, inter and y O(1) at
    H=4096, I=1536, so the absolute tolerance of the parity tests stays meaningful);
    x [T, H] ~N(0,1) bf16."""
    g = _gen(device, seed)
    wr = (torch.randn((E, H), generator=g, device=device) * 0.02).to(torch.bfloat16)
    w13 = torch.randint(0, 256, (E, 2 * I, H // 2), generator=g, device=device, dtype=torch.uint8)
    w13_sf = (torch.rand((E, 2 * I, H // 16), generator=g, device=device) * 0.75 + 0.25).to(E4M3)
    w2 = torch.randint(0, 256, (E, H, I // 2), generator=g, device=device, dtype=torch.uint8)
    w2_sf = (torch.rand((E, H, I // 16), generator=g, device=device) * 0.75 + 0.25).to(E4M3)
    w13_gs = (torch.rand((E,), generator=g, device=device) * (gs13[1] - gs13[0]) + gs13[0]).float()
    w2_gs = (torch.rand((E,), generator=g, device=device) * (gs2[1] - gs2[0]) + gs2[0]).float()
    x = torch.randn((T, H), generator=g, device=device).to(torch.bfloat16)
    return {"x": x, "router": wr, "w13": w13, "w13_sf": w13_sf, "w13_gs": w13_gs,
            "w2": w2, "w2_sf": w2_sf, "w2_gs": w2_gs, "topk": topk}


def layer_case(B=128, H=8192, Hq=64, Hkv=8, D=128, ctx=(1024, 8192), page=16, pool_pages=1 << 17,
               theta=5e5, eps=1e-6, seed=0, device="cuda", fill=True):
    """Decode-layer workload: one decode step of a layer: x [B, H] ~N(0,1) bf16; RMSNorm weight
    (plain, ~1 + N(0, 0.02)); Wqkv [(Hq + 2Hkv) D, H] and Wo [H, Hq D] ~N(0, 0.02) bf16; paged
    FP8 cache holding ctx ~U[1024, 8192] tokens per sequence (+1 page of room for the append)."""
    att = attention_case(B, Hq, Hkv, D, ctx, page, pool_pages, seed, device, extra_tokens=1, fill=fill)
    g = _gen(device, seed + 1)
    x = torch.randn((B, H), generator=g, device=device).to(torch.bfloat16)
    norm_w = (1.0 + 0.02 * torch.randn((H,), generator=g, device=device)).to(torch.bfloat16)
    wqkv = (torch.randn(((Hq + 2 * Hkv) * D, H), generator=g, device=device) * 0.02).to(torch.bfloat16)
    wo = (torch.randn((H, Hq * D), generator=g, device=device) * 0.02).to(torch.bfloat16)
    positions = att["seq_lens"].long().clone()
    return {"x": x, "norm_w": norm_w, "wqkv": wqkv, "wo": wo, "positions": positions,
            "k_cache": att["k_cache"], "v_cache": att["v_cache"], "page_table": att["page_table"],
            "seq_lens": att["seq_lens"], "k_scale": att["k_scale"], "v_scale": att["v_scale"],
            "lens": att["lens"], "theta": theta, "eps": eps, "Hq": Hq, "Hkv": Hkv, "D": D,
            "sm_scale": 1.0 / math.sqrt(D)}


def muse_layer_case(B=1, L=1, ctx=(1000, 3000), page=1, window=0, theta=5e5, kv_scale=1.0, local_start=32,
                    local_bias=0.08, seed=0, device="cuda", weights=None):
    """One Muse TP8/EP8 decode-layer step in the reference problem's data formats
    (muse_decode_layer/decode/spec.py): weights (random init: dense ~N(0, 0.02) bf16, norm and
    gate weights ~N(0, 0.05)/N(0, 0.3), router fp32 ~N(0, 0.02), router_bias ~N(0, 0.01) plus
    `local_bias` on this GPU's 32 experts so that a step routes some tokens here, the 32 local
    experts' NVFP4 banks as moe_case makes them at H = I = 4096) and inputs (stream fp32
    ~N(0,1), attn_input bf16 ~N(0,1), B requests of ctx ~U[lo, hi] cached tokens each plus a
    block of L new ones, e4m3 caches of N(0,1)/kv_scale codes, page table and cache rows).
    Pass `weights` from an earlier call to reuse them.  Returns (weights, data)."""
    g = _gen(device, seed)
    if weights is None:
        def dense(n, k):
            return (torch.randn((n, k), generator=g, device=device) * 0.02).to(torch.bfloat16)

        def vec(n, s):
            return (torch.randn((n,), generator=g, device=device) * s).to(torch.bfloat16)
        bank = moe_case(T=1, E=32, H=4096, I=4096, seed=seed + 1, device=device, gs2=(0.015, 0.025))
        bias = torch.randn((256,), generator=g, device=device) * 0.01
        bias[local_start:local_start + 32] += local_bias
        weights = {"qkv_gate": dense(2304, 8192), "o": dense(8192, 1024), "attn_residual_gate": vec(8192, 0.3),
                   "pre_ffn_norm": vec(8192, 0.05),
                   "router": torch.randn((256, 8192), generator=g, device=device) * 0.02, "router_bias": bias,
                   "pooler": dense(4096, 8192), "pre_expert_norm": vec(4096, 0.05),
                   "post_expert_norm": vec(4096, 0.05), "unpooler": dense(8192, 4096), "post_ffn_norm": vec(8192, 0.05),
                   "ffn_residual_gate": vec(8192, 0.3), "next_pre_attn_norm": vec(8192, 0.05)}
        weights.update({k: bank[k] for k in ("w13", "w13_sf", "w13_gs", "w2", "w2_sf", "w2_gs")})
    T = B * L
    lens = torch.randint(ctx[0], ctx[1] + 1, (B,), generator=g, device=device)
    lens_l = [int(v) for v in lens.tolist()]
    pool = sum(math.ceil((n + L) / page) for n in lens_l) + 3
    table = paged_layout(lens_l, page, pool, g, device, extra_tokens=L)
    kc = torch.empty((pool, page, 2, 64), dtype=E4M3, device=device)
    vc = torch.empty_like(kc)
    fill_e4m3_normal(kc, g, torch.full((2,), kv_scale, device=device))
    fill_e4m3_normal(vc, g, torch.full((2,), kv_scale, device=device))
    pos = (lens.long()[:, None] + torch.arange(L, device=device)).reshape(-1)
    rows = table.long().repeat_interleave(L, dim=0)
    loc = rows.gather(1, (pos // page)[:, None]).reshape(-1) * page + pos % page
    cfg = {"batch": B, "q_len": L, "tokens": T, "hidden": 8192, "num_q_heads": 16, "num_kv_heads": 2, "head_dim": 64,
           "page_size": page, "window": window, "rope_theta": theta, "qk_scale_factor": 5.4730064863875,
           "sm_scale": 0.125, "kv_scale": kv_scale, "n_experts": 256, "top_k": 8, "local_experts": 32}
    s = torch.tensor(kv_scale, dtype=torch.float32, device=device)
    data = {"stream": torch.randn((T, 8192), generator=g, device=device),
            "attn_input": torch.randn((T, 8192), generator=g, device=device).to(torch.bfloat16),
            "k_cache": kc, "v_cache": vc, "positions": pos, "cache_loc": loc,
            "cache_seqlens": (lens + L).to(torch.int32),
            "cu_seqlens_q": torch.arange(0, T + 1, L, device=device, dtype=torch.int32),
            "scheduler_metadata": None, "k_scale": s, "v_scale": s, "page_table": table,
            "seq_lens": lens.to(torch.int32),
            "local_start": torch.tensor([local_start], dtype=torch.int32, device=device), "config": cfg}
    return weights, data
