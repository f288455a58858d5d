# okc: problem=muse_moe_w4a16
"""Routed NVFP4 (W4A16) experts with the reference problem's surface
(muse_moe_w4a16/submission.py:22-49, 352-398): `prepare(weights)` keeps the bank as stored
(no repack), `kernel_fn(data, state)` takes hidden_states [M, H] bf16, topk_ids [M, k] int32
(global ids) and topk_weights [M, k] fp32 and returns bf16 [M, H]: the routing-weighted sum of
the local experts' SwiGLU MLP outputs.  The plain W4A16 MoE contract has no post-expert RMSNorm, so the Muse
`post_norm_w` is not applied (it is the reference's `_finalize` extra, submission.py:295-308)."""

from __future__ import annotations

import torch

from okc_b200 import ops


def prepare(weights: dict) -> dict:
    return {k: v.contiguous() for k, v in weights.items()}


def kernel_fn(data: dict, state: dict) -> torch.Tensor:
    cfg = data["config"]
    lo, n = cfg["local_start"], cfg["local_count"]
    x = data["hidden_states"].contiguous()
    ids = data["topk_ids"].to(torch.int32).contiguous()
    wts = data["topk_weights"].float().contiguous()
    sl = slice(lo, lo + n)
    perm = ops.moe_permute(ids, lo, n)
    return ops.moe_experts(x, ids, wts, perm, state["w13"][sl], state["w13_sf"][sl], state["w13_gs"][sl],
                           state["w2"][sl], state["w2_sf"][sl], state["w2_gs"][sl], lo)


custom_kernel = kernel_fn
