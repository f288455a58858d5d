# okc: problem=muse_bf16_proj
"""BF16 projection operator with the reference problem's surface
(muse_bf16_proj/projection/runtime.py:50, 223): `prepare(weights)` keeps the bf16 weight
matrices, `kernel_fn(data, state)` returns y = x @ W[:n]^T for data = {"x": [m, k] bf16,
"config": {"layer", "m", "n", "k"}} through okc_gemm_bf16 (split-K skinny kernel for m <= 32,
tcgen05 for larger m).  The FP32 router layer returns fp32 logits through its bf16 hi/lo halves
(prepare splits it as the reference does, runtime.py:42-47; okc_router_logits)."""

from __future__ import annotations

import torch

from okc_b200 import ops


def prepare(weights: dict) -> dict:
    state = {"weights": {k: w.contiguous() for k, w in weights.items()}}
    r = weights.get("router")
    if r is not None and r.dtype == torch.float32:
        hi = r.to(torch.bfloat16)
        lo = (r - hi.float()).to(torch.bfloat16)
        state["router_hilo"] = torch.cat([hi, lo], 0).contiguous()
    return state


def kernel_fn(data: dict, state: dict) -> torch.Tensor:
    x, cfg = data["x"], data["config"]
    if cfg["layer"] == "router" and "router_hilo" in state:
        return ops.router_logits(x, state["router_hilo"])[:, :cfg["n"]]
    w = state["weights"][cfg["layer"]]
    if w.dtype != torch.bfloat16:
        raise ValueError(f"layer {cfg['layer']!r} has {w.dtype} weights; okc_b200 projects bf16 only")
    n = cfg["n"]
    return ops.gemm(x, w[:n])


custom_kernel = kernel_fn
