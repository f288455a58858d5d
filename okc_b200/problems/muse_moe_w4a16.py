# okc: problem=muse_moe_w4a16
"""Routed NVFP4 (W4A16) experts with the reference problem's surface
(muse_moe_w4a16/submission.py:22-49, 352-398): `prepare(weights)` keeps the bank as stored
(no repack), `kernel_fn(data, state)` takes hidden_states [M, H] bf16, topk_ids [M, k] int32
(global ids) and topk_weights [M, k] fp32 and returns bf16 [M, H]: the routing-weighted sum over
the local experts of their SwiGLU MLP outputs, each first passed through the post-expert
RMSNorm with weight 1 + post_norm_w (`_finalize`, submission.py:295-308) when the bank carries
`post_norm_w` (a bank without it gives the plain W4A16 sum)."""

from __future__ import annotations

import torch

from okc_b200 import ops


def prepare(weights: dict) -> dict:
    state = {k: v.contiguous() for k, v in weights.items()}
    if "post_norm_w" in weights:  # the reference's prepare keeps 1 + w in fp32 (submission.py:364)
        state["norm_w"] = (weights["post_norm_w"].float() + 1.0).contiguous()
    return state


def kernel_fn(data: dict, state: dict) -> torch.Tensor:
    cfg = data["config"]
    lo, n = cfg["local_start"], cfg["local_count"]
    x = data["hidden_states"].contiguous()
    ids = data["topk_ids"].to(torch.int32).contiguous()
    wts = data["topk_weights"].float().contiguous()
    sl = slice(lo, lo + n)
    perm = ops.moe_permute(ids, lo, n)
    return ops.moe_experts(x, ids, wts, perm, state["w13"][sl], state["w13_sf"][sl], state["w13_gs"][sl],
                           state["w2"][sl], state["w2_sf"][sl], state["w2_gs"][sl], lo,
                           post_gain=state.get("norm_w"))


custom_kernel = kernel_fn
