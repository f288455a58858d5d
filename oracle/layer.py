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
