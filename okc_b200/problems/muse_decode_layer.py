# okc: problem=muse_decode_layer
"""One Muse TP8/EP8 decoder layer with the reference problem's surface
(muse_decode_layer/decode/runtime.py:13-75, spec.py:6-66): `prepare(weights)` does the
constant-only preparation, `kernel_fn(data, state)` runs the layer on this GPU's slice and
returns (hidden bf16 [T, 8192], stream fp32 [T, 8192], ids int32 [T, 8]).

Stages, each on this library's kernels:
  * qkv_gate projection of attn_input, per-head QK RMSNorm, interleaved RoPE (frequencies of
    theta 500000, applied when config rope_theta != 0), the FP8 append of the new tokens' K/V,
    gated paged attention (sliding window config "window", verify blocks of q_len tokens), the
    per-head output RMSNorm x sigmoid(gate) (decode/attention.py:13-37, 88-129, 184-198);
  * O projection, then the attention residual boundary (decode/boundaries.py:17-52): stream
    update with alpha/beta of attn_residual_gate, next RMSNorm with 1 + pre_ffn_norm;
  * pooler projection + RMSNorm with 1 + pre_expert_norm (runtime.py:52-54);
  * router logits in fp32 and Muse's sigmoid + bias routing (runtime.py:55-63): up to 8 tokens
    the reference multiplies the unrounded fp32 boundary output by the fp32 router; here that
    input is split into bf16 halves x = hi + lo and each half goes through the bf16 hi/lo
    router kernel (four bf16 products summed in fp32, about 2^-16 of |x||w| from the fp32
    product); from 9 tokens on, the bf16 hidden times the hi/lo halves, as the reference does;
  * local experts (global id - local_start) mod 256 < 32, their SwiGLU NVFP4 MLPs and the
    post-expert RMSNorm finalize with the bf16 gain 1 + post_expert_norm (decode/experts.py:
    66-106);
  * unpooler projection (rows 0-1023 only for up to 8 tokens, the rest of the branch zero,
    decode/projections.py:54-57) and the final boundary (post_ffn_norm scaling, ffn gate,
    next_pre_attn_norm).

Token counts: decode steps and verify blocks (q_len 1 / 8), and prefill blocks (q_len 200-16384,
muse_prefill_layer/submission.py:201-218, the same layer): projections beyond 256 tokens run as
256-row tcgen05 blocks, the append of a long block runs per request with its table row shared,
the experts run in passes of 2048 tokens, and attention runs on the prefill kernel
(okc_attn_prefill_fp8: 8 tokens x the query heads of one KV head per CTA, the request's keys
streamed once for them).

Queries: the reference's window-0 path hands FA3 an e4m3-rounded query
(decode/attention.py:150-165); here every layer keeps the bf16 query of its split-attention
path (q x qk_scale_factor rounded to bf16), the more precise of the two."""

from __future__ import annotations

import torch

from okc_b200 import ops

HIDDEN = 8192
N_EXPERTS = 256
TOP_K = 8
LOCAL_EXPERTS = 32
RMS_EPS = 1e-5          # decode/attention.py:22, boundaries.py:13
POST_NORM_EPS = 1e-8    # decode/spec.py:76
ROPE_BASE = 500000.0    # decode/runtime.py:33
ROUTE_SCALE = 0.1767766952966369   # decode/runtime.py:31 (router_output_multiplier)
ROUTE_EPS = 1e-15
MOE_CHUNK = 2048        # tokens per expert pass (okc_moe_permute: T * top_k <= 16384)


def _gate_coeffs(w: torch.Tensor):
    """alpha, beta of a residual gate (decode/runtime.py:39-43)."""
    gate = w.float() / 0.3
    beta = torch.sigmoid(gate)
    alpha = torch.sqrt(torch.clamp(torch.sigmoid(-gate) * (1.0 + beta), min=1e-3))
    return alpha.contiguous(), beta.contiguous()


def prepare(weights: dict) -> dict:
    router = weights["router"].float()
    hi = router.to(torch.bfloat16)
    lo = (router - hi.float()).to(torch.bfloat16)
    device = weights["qkv_gate"].device
    state = {k: weights[k].contiguous() for k in
             ("qkv_gate", "o", "pooler", "unpooler", "pre_ffn_norm", "pre_expert_norm", "post_ffn_norm",
              "next_pre_attn_norm", "w13", "w13_sf", "w13_gs", "w2", "w2_sf", "w2_gs")}
    state["router_hilo"] = torch.cat([hi, lo], 0).contiguous()
    state["router_bias"] = weights["router_bias"].float().contiguous()
    # the reference keeps 1 + post_expert_norm rounded to bf16 (runtime.py:34)
    state["post_expert_gain"] = (1.0 + weights["post_expert_norm"].float()).to(torch.bfloat16).float().contiguous()
    state["inv_freq"] = ops.rope_inv_freq(ROPE_BASE, 64, device)
    for name, key in (("attn", "attn_residual_gate"), ("ffn", "ffn_residual_gate")):
        state[name + "_alpha"], state[name + "_beta"] = _gate_coeffs(weights[key])
    return state


def _attention(data: dict, state: dict) -> torch.Tensor:
    cfg = data["config"]
    B, L = cfg["batch"], cfg["q_len"]
    hq, hkv, d = cfg["num_q_heads"], cfg["num_kv_heads"], cfg["head_dim"]
    qkv = ops.gemm(data["attn_input"], state["qkv_gate"])
    ks = data["k_scale"].float().reshape(-1).expand(hkv).contiguous()
    vs = data["v_scale"].float().reshape(-1).expand(hkv).contiguous()
    positions = data["positions"].reshape(-1).long()
    table = data["page_table"]
    inv = state["inv_freq"] if cfg.get("rope_theta", 0) else None
    if L <= 8:
        table_rows = table.repeat_interleave(L, dim=0) if L > 1 else table
        q = ops.rope_kv_append(qkv, positions, table_rows, data["k_cache"], data["v_cache"], ks, vs, hq, hkv, d, inv,
                               q_scale=cfg["qk_scale_factor"], qk_norm=True, norm_eps=RMS_EPS)
    else:  # prefill blocks: one append per request, its table row shared by its L tokens (row stride 0)
        q = torch.empty((B * L, hq, d), dtype=torch.bfloat16, device=qkv.device)
        for b in range(B):
            r = slice(b * L, (b + 1) * L)
            ops.rope_kv_append(qkv[r], positions[r], table[b:b + 1].expand(L, -1), data["k_cache"], data["v_cache"],
                               ks, vs, hq, hkv, d, inv, q_out=q[r], q_scale=cfg["qk_scale_factor"], qk_norm=True,
                               norm_eps=RMS_EPS)
    cs = data.get("cache_seqlens")
    if L == 1 and cs is not None and cs.dtype == torch.int32 and cs.is_contiguous():
        lens = cs  # seq_lens + 1: each token's own position + 1 (spec.py:64)
    else:
        lens = (positions + 1).to(torch.int32)
    gate = qkv[:, (hq + 2 * hkv) * d:(2 * hq + 2 * hkv) * d]
    window = int(cfg.get("window", 0) or 0)
    if L <= 8:
        out = ops.attn_decode(q, data["k_cache"], data["v_cache"], table, lens, ks, vs, cfg["sm_scale"], gate=gate,
                              out_eps=RMS_EPS, window=window, q_per_seq=L)
        return out.view(B * L, hq * d)
    # prefill blocks: the prefill kernel (8 tokens x the query heads of a KV head per CTA, the
    # request's keys streamed once for them)
    out = ops.attn_prefill(q, data["k_cache"], data["v_cache"], table, positions, ks, vs, cfg["sm_scale"], B, L,
                           gate=gate, out_eps=RMS_EPS, window=window)
    return out.view(B * L, hq * d)


def kernel_fn(data: dict, state: dict):
    T = data["config"]["tokens"]
    attn = _attention(data, state)
    branch = ops.gemm(attn, state["o"])
    small = T <= 8
    h, stream, router_in = ops.residual_boundary(data["stream"], branch, state["attn_alpha"], state["attn_beta"],
                                                 None, state["pre_ffn_norm"], post_eps=POST_NORM_EPS,
                                                 pre_eps=RMS_EPS, router=small)
    x = ops.rmsnorm(ops.gemm(h, state["pooler"]), state["pre_expert_norm"], RMS_EPS, unit_offset=True)
    if small:
        hl = torch.empty((2 * T, HIDDEN), dtype=torch.bfloat16, device=h.device)  # [hi; lo] of router_in
        hl[:T].copy_(router_in)
        torch.sub(router_in, hl[:T], out=hl[T:])  # fp32 difference, rounded once to bf16
        logits = ops.router_logits(hl, state["router_hilo"])
        ids, wts = ops.route_sigmoid(logits[:T], state["router_bias"], TOP_K, logits_lo=logits[T:],
                                     scale=ROUTE_SCALE, eps=ROUTE_EPS)
    else:
        logits = ops.router_logits(h, state["router_hilo"])
        ids, wts = ops.route_sigmoid(logits, state["router_bias"], TOP_K, scale=ROUTE_SCALE, eps=ROUTE_EPS)
    # this GPU's experts are global ids local_start .. local_start + 31 (decode/runtime.py:71)
    lids = torch.remainder(ids - data["local_start"].to(torch.int32), N_EXPERTS).to(torch.int32)
    ex = torch.empty_like(x)
    for c0 in range(0, T, MOE_CHUNK):  # the permutation takes up to 2048 tokens x 8 slots
        c = slice(c0, min(T, c0 + MOE_CHUNK))
        perm = ops.moe_permute(lids[c], 0, LOCAL_EXPERTS)
        ops.moe_experts(x[c], lids[c], wts[c], perm, state["w13"], state["w13_sf"], state["w13_gs"], state["w2"],
                        state["w2_sf"], state["w2_gs"], 0, out=ex[c], post_gain=state["post_expert_gain"],
                        post_eps=POST_NORM_EPS)
    if small:  # only this GPU's 1024 rows of the unpooler; the boundary sees zeros beyond them
        bufs = state.setdefault("_ffn_small", {})
        if T not in bufs:  # columns 1024.. are zero once and never written
            bufs[T] = torch.zeros((T, HIDDEN), dtype=torch.bfloat16, device=ex.device)
        ffn = bufs[T]
        ops.gemm(ex, state["unpooler"][:1024], out=ffn[:, :1024])
    else:
        ffn = ops.gemm(ex, state["unpooler"])
    hidden, stream, _ = ops.residual_boundary(stream, ffn, state["ffn_alpha"], state["ffn_beta"],
                                              state["post_ffn_norm"], state["next_pre_attn_norm"],
                                              post_eps=POST_NORM_EPS, pre_eps=RMS_EPS)
    return hidden, stream, ids


custom_kernel = kernel_fn
