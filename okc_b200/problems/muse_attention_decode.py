# okc: problem=muse_attention_decode
"""Gated paged-FP8 attention decode with the reference problem's inputs and semantics
(muse_attention_decode/submission.py:22-49, 442-478): per-head QK RMSNorm, interleaved RoPE
when rope_theta != 0, queries scaled by qk_scale_factor and rounded to bf16, FP8 append of the
new K/V into the paged cache (written in place), attention over every cached position up to
and including the new token, then a per-head RMSNorm of the output times sigmoid(gate).

Runs on okc_rope_kv_append_ex + okc_attn_decode_fp8_gated.  Supported here: q_len 1 (decode)
and window 0 (full attention); head_dim 64 or 128 (config "head_dim", default 64 as in the
reference), up to 8 query heads per KV head."""

from __future__ import annotations

import torch

from okc_b200 import ops

RMS_EPS = 1e-5  # muse_attention_decode/submission.py:53
_FREQ: dict = {}


def _inv_freq(theta: float, d: int, device):
    key = (theta, d, device)
    if key not in _FREQ:
        _FREQ[key] = ops.rope_inv_freq(theta, d, device)
    return _FREQ[key]


def kernel_fn(data: dict) -> torch.Tensor:
    cfg = data["config"]
    B, L = cfg["batch"], cfg["q_len"]
    hq, hkv = cfg["num_q_heads"], cfg["num_kv_heads"]
    d = cfg.get("head_dim", 64)
    if L != 1:
        raise ValueError("okc_b200 muse_attention_decode: q_len must be 1 (verify blocks are not supported)")
    if cfg.get("window", 0):
        raise ValueError("okc_b200 muse_attention_decode: sliding-window attention is not supported")
    qkv = data["qkv"].reshape(B, -1)
    device = qkv.device
    theta = cfg.get("rope_theta", 0.0)
    inv = _inv_freq(theta, d, device) if theta else None
    ks = data["k_scale"].float().reshape(-1).expand(hkv).contiguous()
    vs = data["v_scale"].float().reshape(-1).expand(hkv).contiguous()
    positions = data["positions"].reshape(-1).long()
    q = ops.rope_kv_append(qkv, positions, data["page_table"], data["k_cache"], data["v_cache"], ks, vs,
                           hq, hkv, d, inv, q_scale=cfg["qk_scale_factor"], qk_norm=True, norm_eps=RMS_EPS)
    lens = (data["seq_lens"].reshape(-1) + 1).to(torch.int32)
    gate = qkv[:, (hq + 2 * hkv) * d:(2 * hq + 2 * hkv) * d]
    out = ops.attn_decode(q, data["k_cache"], data["v_cache"], data["page_table"], lens, ks, vs, cfg["sm_scale"],
                          gate=gate, out_eps=RMS_EPS)
    return out.view(B, L, hq * d)


custom_kernel = kernel_fn
