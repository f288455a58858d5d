"""Decode-layer oracle for the small and the full decode-layer workloads (test infrastructure only).

RMSNorm -> QKV projection -> RoPE -> FP8 KV-append -> paged attention -> O projection ->
residual add, with the bf16 boundaries of the reference layer
(muse_prefill_layer/submission.py:137-176, 201-207; muse_decode_layer/decode/runtime.py:47-50),
without Muse's QK-norm, output gate and gated residual (the plain layer is RMSNorm,
eps 1e-6, and x + O).
"""

from __future__ import annotations

import torch

from . import attention as att
from .numerics import bf16_round
from .projection import gemm, rmsnorm


def decode_layer(x, norm_w, wqkv, wo, positions, page_table, k_cache, v_cache, k_scale, v_scale,
                 Hq, Hkv, D, theta, eps, sm_scale):
    """Mutates the caches (the new token's K/V); returns (out bf16 [B, H], slots int64 [B])."""
    xn = rmsnorm(x, norm_w, eps)
    qkv = gemm(xn, wqkv)
    q, slots = att.kv_append(qkv, positions, page_table, k_cache, v_cache, k_scale, v_scale, Hq, Hkv, D, theta)
    qb = q.to(torch.bfloat16)
    lens = positions.long() + 1
    o = att.attend(qb, k_cache, v_cache, page_table, lens, k_scale, v_scale, sm_scale).to(torch.bfloat16)
    out = gemm(o.reshape(x.shape[0], Hq * D), wo, residual=x)
    return out, slots


def residual_boundary(stream: torch.Tensor, branch: torch.Tensor, alpha: torch.Tensor, beta: torch.Tensor,
                      post_w: torch.Tensor | None, pre_w: torch.Tensor, post_eps: float = 1e-8,
                      pre_eps: float = 1e-5, rounding: str = "rne"):
    """Muse's gated residual boundary (muse_decode_layer/decode/boundaries.py:17-37; the stream
    update of muse_prefill_layer/submission.py:205-215): the branch (bf16 [T, W]; with
    `post_w`, first scaled by 1 + post_w and rounded to bf16) is RMS-normalised (eps 1e-8),
    stream' = alpha * stream + beta * branch (fp32, products rounded separately), and the next
    layer's input hidden = bf16(stream' * rsqrt(mean(stream'^2) + 1e-5) * (1 + pre_w)).
    Returns (hidden bf16, stream' fp32, the unrounded hidden fp32 the router reads); `rounding`
    picks the bf16 rounding (see numerics.bf16_round)."""
    b = branch.float()
    if post_w is not None:
        b = bf16_round(b * (1.0 + post_w.float()), rounding)
    b = b * torch.rsqrt(b.pow(2).sum(-1, keepdim=True) / b.shape[-1] + post_eps)
    st = alpha.float() * stream.float() + beta.float() * b
    h = st * torch.rsqrt(st.pow(2).sum(-1, keepdim=True) / st.shape[-1] + pre_eps) * (1.0 + pre_w.float())
    return bf16_round(h, rounding).to(torch.bfloat16), st, h


def _gate_coeffs(w: torch.Tensor):
    """alpha, beta of a Muse residual gate (muse_decode_layer/decode/runtime.py:39-43)."""
    gate = w.float() / 0.3
    beta = torch.sigmoid(gate)
    return torch.sqrt(torch.clamp(torch.sigmoid(-gate) * (1.0 + beta), min=1e-3)), beta


def muse_decode_layer(data: dict, weights: dict, ids_in: torch.Tensor | None = None):
    """One Muse decode layer on this GPU's slice (muse_decode_layer/decode/runtime.py:47-75):
    gated attention (decode/attention.py:13-37, 88-129 with the bf16 query of its split path,
    RoPE frequencies of theta 500000 when config rope_theta != 0), O projection, attention
    boundary (router input: the unrounded fp32 hidden for up to 8 tokens), pooler + RMSNorm
    with 1 + pre_expert_norm, fp32 router logits (fp64 product here) and the sigmoid + bias
    routing (runtime.py:30-32, 55-63), the local experts (global id - local_start) mod 256 < 32
    with the post-expert finalize (gain bf16(1 + post_expert_norm), decode/experts.py:66-106),
    the unpooler (only rows 0-1023 up to 8 tokens, decode/projections.py:54-57; the boundary
    divides by 8192 whatever the branch width) and the final boundary.  Mutates the caches.
    `ids_in` (the device's routing) replaces the top-8 choice, with the weights taken from this
    oracle's own scores, so that a near-tie the two sides break differently does not swap an
    expert.  Returns (hidden bf16, stream fp32, ids int32, scores fp32 [T, 256] incl. bias)."""
    from . import moe as omoe
    cfg = data["config"]
    T = cfg["tokens"]
    qkv = gemm(data["attn_input"], weights["qkv_gate"])
    acfg = dict(cfg, rope_theta=500000.0 if cfg.get("rope_theta", 0) else 0.0)
    attn = att.muse_attention(qkv, data["positions"], data["page_table"], data["k_cache"], data["v_cache"],
                              data["k_scale"].reshape(-1).expand(cfg["num_kv_heads"]),
                              data["v_scale"].reshape(-1).expand(cfg["num_kv_heads"]), acfg)
    branch = gemm(attn, weights["o"])
    a, b = _gate_coeffs(weights["attn_residual_gate"])
    h, stream, router_in = residual_boundary(data["stream"], branch, a, b, None, weights["pre_ffn_norm"])
    x = rmsnorm(gemm(h, weights["pooler"]), weights["pre_expert_norm"], 1e-5, unit_offset=True)
    xr = router_in if T <= 8 else h.float()
    logits = (xr.double() @ weights["router"].double().T).float()
    scores = torch.sigmoid(logits * 0.1767766952966369)
    bias = weights["router_bias"].float()
    if ids_in is None:
        ids, wts = omoe.route_sigmoid(logits, bias, 8)
    else:
        ids = ids_in.to(torch.int32)
        picked = scores.gather(1, ids.long())
        wts = picked / (picked.sum(-1, keepdim=True) + 1e-15)
    lids = torch.remainder(ids.long() - int(data["local_start"].reshape(-1)[0]), 256).to(torch.int32)
    gain = (1.0 + weights["post_expert_norm"].float()).to(torch.bfloat16).float()
    ex = omoe.experts(x, lids, wts, weights["w13"], weights["w13_sf"], weights["w13_gs"], weights["w2"],
                      weights["w2_sf"], weights["w2_gs"], expert_lo=0, post_gain=gain)
    if T <= 8:
        ffn = torch.zeros((T, weights["unpooler"].shape[0]), dtype=torch.bfloat16)
        ffn[:, :1024] = gemm(ex, weights["unpooler"][:1024])
    else:
        ffn = gemm(ex, weights["unpooler"])
    a, b = _gate_coeffs(weights["ffn_residual_gate"])
    hidden, stream, _ = residual_boundary(stream, ffn, a, b, weights["post_ffn_norm"], weights["next_pre_attn_norm"])
    return hidden, stream, ids, scores + bias[None, :]
