"""Projection oracle (test infrastructure only).

y = x · W^T with fp32 accumulation and one rounding to bf16 — inputs are not rounded
before the product (muse_bf16_proj/projection/kernels/gemv.py:37) and partial sums are
fp32 (muse_decode_layer/decode/projections.py:13-15, 33-39, 42-48).
"""

from __future__ import annotations

import torch


def gemm(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None,
         out_fp32: bool = False) -> torch.Tensor:
    y = x.float() @ w.float().T
    if residual is not None:
        y = y + residual.float()
    return y if out_fp32 else y.to(torch.bfloat16)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, unit_offset: bool = False) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) * g in fp32, rounded to bf16 once
    (muse_prefill_layer/submission.py:89-96: `rms`, `gain`)."""
    xf = x.float()
    g = w.float() + (1.0 if unit_offset else 0.0)
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * g).to(torch.bfloat16)
