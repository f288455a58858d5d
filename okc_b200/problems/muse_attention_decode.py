# okc: problem=muse_attention_decode
"""Gated paged-FP8 attention decode with the reference problem's inputs and semantics
(muse_attention_decode/submission.py:22-49, 442-478): per-head QK RMSNorm, interleaved RoPE
when rope_theta != 0, queries scaled by qk_scale_factor and rounded to bf16, FP8 append of the
new tokens' K/V into the paged cache (written in place), attention over the cached positions
(pos - window, pos] of each query token (window 0: every position up to and including its own),
then a per-head RMSNorm of the output times sigmoid(gate).

q_len 1 is a decode step; q_len > 1 a speculative-verify block (request r's tokens are rows
r*q_len .. r*q_len + q_len - 1 of qkv / positions, causal within the block, the whole block
appended first, muse_prefill_layer/submission.py:155-171).  Runs on okc_rope_kv_append_ex +
okc_attn_decode_fp8_ex; head_dim 64 or 128 (config "head_dim", default 64 as in the
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
    window = int(cfg.get("window", 0) or 0)
    qkv = data["qkv"].reshape(B * L, -1)
    device = qkv.device
    theta = cfg.get("rope_theta", 0.0)
    inv = _inv_freq(theta, d, device) if theta else None
    ks = data["k_scale"].float().reshape(-1).expand(hkv).contiguous()
    vs = data["v_scale"].float().reshape(-1).expand(hkv).contiguous()
    positions = data["positions"].reshape(-1).long()
    table = data["page_table"]
    # the append addresses one page-table row per token: request r's row for its L tokens
    table_rows = table.repeat_interleave(L, dim=0) if L > 1 else table
    q = ops.rope_kv_append(qkv, positions, table_rows, data["k_cache"], data["v_cache"], ks, vs,
                           hq, hkv, d, inv, q_scale=cfg["qk_scale_factor"], qk_norm=True, norm_eps=RMS_EPS)
    lens = (positions + 1).to(torch.int32)  # each token sees the cache up to its own position
    gate = qkv[:, (hq + 2 * hkv) * d:(2 * hq + 2 * hkv) * d]
    out = ops.attn_decode(q, data["k_cache"], data["v_cache"], table, lens, ks, vs, cfg["sm_scale"],
                          gate=gate, out_eps=RMS_EPS, window=window, q_per_seq=L)
    return out.view(B, L, hq * d)


custom_kernel = kernel_fn
