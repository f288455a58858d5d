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
