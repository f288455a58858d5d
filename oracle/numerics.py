"""Bit-level helpers shared by the oracle (CPU, numpy/torch).  Test infrastructure only."""

from __future__ import annotations

import numpy as np
import torch


def bf16_round_np(v: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 round-to-nearest-even, returned as fp32 (finite inputs), the same rule
    as muse_decode_layer/tests/test_nvfp4_gemv.py:17-20."""
    v = np.ascontiguousarray(v, dtype=np.float32)
    bits = v.view(np.uint32).astype(np.uint64)
    r = ((bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def to_bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16)


def e4m3(t: torch.Tensor) -> torch.Tensor:
    """fp32 -> float8_e4m3fn exactly as torch does (RNE, overflow -> NaN), the conversion
    of muse_prefill_layer/submission.py:155-156."""
    return t.float().to(torch.float8_e4m3fn)


def bf16_round(t: torch.Tensor, mode: str = "rne") -> torch.Tensor:
    """fp32 -> bf16 -> fp32.  "rne": round to nearest even (torch, and Triton on the GPU);
    "trunc": round toward zero, which is what Triton's CPU interpreter does for .to(tl.bfloat16)
    and for stores into bf16 tensors (it is how the interpreter-run golden fixtures of the
    reference's kernels were rounded)."""
    t = t.float().contiguous()
    if mode == "rne":
        return t.to(torch.bfloat16).float()
    return (t.view(torch.int32) & -65536).view(torch.float32)
