"""Attention oracle: RoPE, FP8 KV-append and paged attention decode (test infrastructure only).

Follows muse_prefill_layer/submission.py:89-176 (`rms`, `rope`, `round_queries`,
`attention`) and muse_attention_decode/tools/bench_tail.py:79-108 (`_ref`), generalised
to the decode-path shapes: per-KV-head scales k_scale[h] / v_scale[h], any head_dim, page size
and GQA ratio.  The Muse-only pieces (per-head QK RMSNorm, query scale factor, RMSNorm x
sigmoid output gate) are kept behind `muse=True` so the reference's own shapes stay
checkable against its code.
"""

from __future__ import annotations

import torch

RMS_EPS = 1e-5  # muse_prefill_layer/submission.py:80


def rms(x: torch.Tensor, eps: float = RMS_EPS) -> torch.Tensor:
    """muse_prefill_layer/submission.py:89-91."""
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)


def inv_freq(theta: float, d: int) -> torch.Tensor:
    """muse_prefill_layer/submission.py:102."""
    return 1.0 / (theta ** (torch.arange(0, d, 2).float() / d))


def rope(x: torch.Tensor, pos: torch.Tensor, theta: float) -> torch.Tensor:
    """Interleaved RoPE on pairs (2i, 2i+1); x [T, heads, d], pos [T]
    (muse_prefill_layer/submission.py:99-105)."""
    d = x.shape[-1]
    ang = pos.float()[:, None, None] * inv_freq(theta, d).to(x.device)
    even, odd = x[..., 0::2], x[..., 1::2]
    return torch.stack([even * ang.cos() - odd * ang.sin(), even * ang.sin() + odd * ang.cos()], -1).flatten(-2)


def cache_slots(page_table: torch.Tensor, positions: torch.Tensor, page: int) -> torch.Tensor:
    """Flat cache row of each new token: table[b][pos // P] * P + pos % P
    (muse_attention_decode/tools/bench_tail.py:53; muse_prefill_layer/submission.py:165).
    page_table int32 [B, max_pages]; positions int64 [B] (q_len 1). Exact int64."""
    pos = positions.long()
    b = torch.arange(pos.shape[0])
    return page_table.long()[b, pos // page] * page + pos % page


def split_qkv(qkv: torch.Tensor, hq: int, hkv: int, d: int):
    """q | k | v (| Muse's output gate) columns of the fused projection output."""
    f = qkv.float()
    q = f[..., :hq * d]
    k = f[..., hq * d:(hq + hkv) * d]
    v = f[..., (hq + hkv) * d:(hq + 2 * hkv) * d]
    return q.reshape(-1, hq, d), k.reshape(-1, hkv, d), v.reshape(-1, hkv, d)


def kv_append(qkv: torch.Tensor, positions: torch.Tensor, page_table: torch.Tensor,
              k_cache: torch.Tensor, v_cache: torch.Tensor, k_scale: torch.Tensor,
              v_scale: torch.Tensor, hq: int, hkv: int, d: int, theta: float,
              muse: bool = False):
    """RoPE (+ Muse QK-norm) of the new token, then the FP8 cache write
    k_cache[slot] = e4m3(k / k_scale), v likewise (muse_prefill_layer/submission.py:141-156).
    Mutates the caches; returns (q rotated fp32 [B, hq, d], slots int64 [B])."""
    q, k, v = split_qkv(qkv, hq, hkv, d)
    if muse:
        q, k = rms(q), rms(k)
    if theta:
        q, k = rope(q, positions, theta), rope(k, positions, theta)
    page = k_cache.shape[1]
    slots = cache_slots(page_table, positions, page)
    kf = k_cache.view(-1, hkv, d)
    vf = v_cache.view(-1, hkv, d)
    ks = k_scale.float().reshape(-1)[None, :, None].expand(1, hkv, 1)
    vs = v_scale.float().reshape(-1)[None, :, None].expand(1, hkv, 1)
    kf[slots] = (k / ks).to(torch.float8_e4m3fn)
    vf[slots] = (v / vs).to(torch.float8_e4m3fn)
    return q, slots


def attend(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, page_table: torch.Tensor,
           seq_lens: torch.Tensor, k_scale: torch.Tensor, v_scale: torch.Tensor,
           sm_scale: float, window: int = 0, q_per_seq: int = 1) -> torch.Tensor:
    """Decode attention of one query token per row over its visible cached keys: positions
    [n - window, n) for n = seq_lens[b] (all of [0, n) when window = 0: the causal / sliding-
    window mask `t <= pos` and `t > pos - window` of muse_prefill_layer/submission.py:168-171,
    with n = pos + 1), rows = table[b // q_per_seq][t // P] * P + t % P (q_per_seq query tokens
    of a verify block share their request's table row), K = e4m3 * k_scale[h],
    V = e4m3 * v_scale[h], softmax(q K^T * sm_scale) V with GQA grouping q.view(Hkv, G, D)
    (muse_prefill_layer/submission.py:158-175; bench_tail.py:97-105).
    q [B, Hq, D] (any float dtype, used as given); returns fp32 [B, Hq, D]."""
    B, hq, d = q.shape
    pages, page, hkv, _ = k_cache.shape
    g = hq // hkv
    kf = k_cache.view(-1, hkv, d)
    vf = v_cache.view(-1, hkv, d)
    ks = k_scale.float().reshape(-1).expand(hkv)[None, :, None]
    vs = v_scale.float().reshape(-1).expand(hkv)[None, :, None]
    out = torch.zeros((B, hq, d), dtype=torch.float32)
    for b in range(B):
        n = int(seq_lens[b])
        lo = max(0, n - window) if window else 0
        if n <= lo:
            continue
        t = torch.arange(lo, n)
        rows = page_table[b // q_per_seq].long()[t // page] * page + t % page
        keys = kf[rows].float() * ks
        vals = vf[rows].float() * vs
        att = torch.einsum("kgd,tkd->kgt", q[b].float().view(hkv, g, d), keys) * sm_scale
        out[b] = torch.einsum("kgt,tkd->kgd", att.softmax(-1), vals).reshape(hq, d)
    return out


def decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, page_table: torch.Tensor,
           seq_lens: torch.Tensor, k_scale: torch.Tensor, v_scale: torch.Tensor,
           sm_scale: float, window: int = 0, q_per_seq: int = 1) -> torch.Tensor:
    """attend() rounded to the bf16 output boundary."""
    return attend(q, k_cache, v_cache, page_table, seq_lens, k_scale, v_scale, sm_scale, window,
                  q_per_seq).to(torch.bfloat16)


def muse_attention(qkv: torch.Tensor, positions: torch.Tensor, page_table: torch.Tensor,
                   k_cache: torch.Tensor, v_cache: torch.Tensor, k_scale: torch.Tensor,
                   v_scale: torch.Tensor, cfg: dict) -> torch.Tensor:
    """The reference's gated decode attention (muse_prefill_layer/submission.py:137-176) for
    q_len L tokens per request (1: decode, 8: a verify block) and sliding window cfg["window"]
    (0: full): QK-RMSNorm, RoPE, queries rounded to bf16 after the scale factor, FP8 append of
    every block token (request r's tokens are rows r*L .. r*L + L - 1, its table row r), then each
    token attends positions (pos - window, pos], then RMSNorm(out) * sigmoid(gate).
    qkv [B*L, (2hq + 2hkv) d] holds q | k | v | gate.  Mutates the caches; returns bf16
    [B*L, hq*d]."""
    hq, hkv, d = cfg["num_q_heads"], cfg["num_kv_heads"], cfg["head_dim"]
    L = cfg.get("q_len", 1)
    table_rows = page_table.repeat_interleave(L, dim=0) if L > 1 else page_table
    q, _ = kv_append(qkv, positions, table_rows, k_cache, v_cache, k_scale, v_scale, hq, hkv, d,
                     cfg["rope_theta"], muse=True)
    q = (q * cfg["qk_scale_factor"]).to(torch.bfloat16)
    gate = qkv.float()[:, (hq + 2 * hkv) * d:]
    lens = positions.long() + 1
    o = attend(q, k_cache, v_cache, page_table, lens, k_scale, v_scale, cfg["sm_scale"],
               window=cfg.get("window", 0), q_per_seq=L)
    return (rms(o).reshape(-1, hq * d) * torch.sigmoid(gate)).to(torch.bfloat16)
