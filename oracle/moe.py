"""W4A16 MoE oracle: NVFP4 decode, routing, permutation, experts, combine (test infrastructure only).

* NVFP4 decode: E2M1 magnitude grid {0, .5, 1, 1.5, 2, 3, 4, 6}, bit 3 = sign, low nibble =
  even element (muse_moe_w4a16/submission.py:311-313), value * f32(sf * gs) rounded to bf16
  (muse_decode_layer/decode/nvfp4_gemv.py:9-18; pinned by muse_decode_layer/tests/
  test_nvfp4_gemv.py:56-69).
* Experts: h = bf16(x @ W13^T), inter = bf16(silu(h_gate) * h_up), y = bf16(inter @ W2^T)
  with bf16 boundaries as muse_moe_w4a16/submission.py:236-242 and
  muse_prefill_layer/submission.py:187-198 (bf16 weights, fp32 accumulate).
* Routing (the contract: softmax top-k of bf16 router logits): logits summed in the
  fixed order the CUDA kernel uses (so ids are reproduced exactly), ties -> lower id.
* Permutation: per local expert the pair ids t*topk + slot in ascending order, counts and
  (expert << 16 | first) tiles of `bm` pairs (muse_moe_w4a16/submission.py:274-291).
"""

from __future__ import annotations

import numpy as np
import torch

from .numerics import bf16_round, bf16_round_np

E2M1_GRID = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def e2m1_codes(packed: torch.Tensor) -> torch.Tensor:
    """uint8 [R, K/2] -> codes uint8 [R, K], low nibble first (muse_moe_w4a16/submission.py:311-313)."""
    return torch.stack((packed & 15, packed >> 4), -1).reshape(packed.shape[0], -1)


def e2m1_values(codes: torch.Tensor) -> torch.Tensor:
    grid = torch.tensor(E2M1_GRID, dtype=torch.float32)
    v = grid[(codes & 7).long()]
    return torch.where((codes & 8) != 0, -v, v)


def dequantize(packed: torch.Tensor, sf: torch.Tensor, gs: float | torch.Tensor) -> torch.Tensor:
    """bf16 [R, K] = bf16(e2m1 * f32(sf * gs)) (muse_decode_layer/decode/nvfp4_gemv.py:9-18)."""
    codes = e2m1_codes(packed)
    r, k = codes.shape
    scale = (sf.float() * torch.as_tensor(gs, dtype=torch.float32)).repeat_interleave(16, dim=1)
    return (e2m1_values(codes) * scale[:, :k]).to(torch.bfloat16)


# ------------------------------------------------------------------------------ routing
def router_logits(x: torch.Tensor, wr: torch.Tensor) -> np.ndarray:
    """bf16-rounded fp32 logits [T, E] in the CUDA kernel's summation order: lane l sums
    x[256j + 8l + i] * w[256j + 8l + i] over j (outer) and i (inner) from 0, then an xor
    butterfly over the 32 lanes (16, 8, 4, 2, 1).  Products of bf16 values are exact in fp32,
    so fused and unfused multiply-adds agree and the result is bit-exact."""
    xf = x.float().numpy().astype(np.float32)
    wf = wr.float().numpy().astype(np.float32)
    T, H = xf.shape
    E = wf.shape[0]
    assert H % 256 == 0
    xr = xf.reshape(T, H // 256, 32, 8)
    wrr = wf.reshape(E, H // 256, 32, 8)
    acc = np.zeros((T, E, 32), np.float32)
    for j in range(H // 256):
        for i in range(8):
            acc = (acc + xr[:, None, j, :, i] * wrr[None, :, j, :, i]).astype(np.float32)
    lanes = np.arange(32)
    for o in (16, 8, 4, 2, 1):
        acc = (acc + acc[:, :, lanes ^ o]).astype(np.float32)
    return bf16_round_np(acc[:, :, 0])


def route(x: torch.Tensor, wr: torch.Tensor, topk: int, renormalize: bool = True):
    """ids int32 [T, topk] (descending logit, ties -> lower id) and fp32 weights: softmax over
    the chosen logits (renormalize) or the full-softmax probability of each chosen expert."""
    lg = router_logits(x, wr)
    T, E = lg.shape
    ids = np.zeros((T, topk), np.int32)
    wts = np.zeros((T, topk), np.float32)
    for t in range(T):
        order = sorted(range(E), key=lambda e: (-float(lg[t, e]), e))[:topk]
        ids[t] = order
        chosen = lg[t, order].astype(np.float64)
        if renormalize:
            ex = np.exp(chosen - chosen[0])
            wts[t] = ex / ex.sum()
        else:
            m = float(lg[t].max())
            wts[t] = np.exp(chosen - m) / np.exp(lg[t].astype(np.float64) - m).sum()
    return torch.from_numpy(ids), torch.from_numpy(wts), torch.from_numpy(lg)


def route_sigmoid(logits: torch.Tensor, bias: torch.Tensor | None, topk: int,
                  scale: float = 0.1767766952966369, eps: float = 1e-15, route_scale: float = 1.0):
    """Muse's routing from fp32 logits (muse_prefill_layer/submission.py:179-184): sigmoid
    scores, the bias only chooses, the chosen scores renormalised (ties: the lower id, which is
    what a stable descending sort gives)."""
    scores = torch.sigmoid(logits.float() * scale)
    key = scores + bias.float() if bias is not None else scores
    ids = torch.sort(key, dim=-1, descending=True, stable=True).indices[:, :topk]
    picked = scores.gather(1, ids)
    return ids.to(torch.int32), picked / (picked.sum(-1, keepdim=True) + eps) * route_scale


def muse_route(h: torch.Tensor, router: torch.Tensor, bias: torch.Tensor, topk: int):
    """Muse's routing: sigmoid scores, bias only to choose, chosen scores renormalised
    (muse_prefill_layer/submission.py:179-184)."""
    return route_sigmoid(h.float() @ router.float().T, bias, topk)


def router_hilo(router: torch.Tensor) -> torch.Tensor:
    """The reference's split of the fp32 router into bf16 halves, stacked [hi; lo]
    (muse_bf16_proj/projection/runtime.py:42-47)."""
    hi = router.to(torch.bfloat16)
    lo = (router - hi.float()).to(torch.bfloat16)
    return torch.cat([hi, lo], 0)


# -------------------------------------------------------------------------- permutation
def permute(ids: torch.Tensor, expert_lo: int, e_local: int, bm: int):
    """(counts [E], offsets [E+1], pairs [n] expert-major ascending, tiles list) as
    muse_moe_w4a16/submission.py:274-291 orders them."""
    flat = ids.reshape(-1).long().numpy() - expert_lo
    n = flat.shape[0]
    counts = np.zeros(e_local, np.int32)
    pairs = []
    tiles = []
    for e in range(e_local):
        p = [i for i in range(n) if flat[i] == e]
        counts[e] = len(p)
        pairs.extend(p)
        for j in range((len(p) + bm - 1) // bm):
            tiles.append((e << 16) | (j * bm))
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    return (torch.from_numpy(counts), torch.from_numpy(offsets),
            torch.tensor(pairs, dtype=torch.int32), torch.tensor([len(tiles)] + tiles, dtype=torch.int32))


# ------------------------------------------------------------------------------ experts
def finalize(y: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor, gain: torch.Tensor,
             expert_lo: int, e_local: int, eps: float = 1e-8, out_fp32: bool = False,
             rounding: str = "rne") -> torch.Tensor:
    """Muse's post-expert RMSNorm and routing-weighted sum (muse_moe_w4a16/submission.py:295-308,
    `post_expert_norm` of muse_prefill_layer/submission.py:114-116): for each slot
    scaled = bf16(y * gain) with gain = 1 + post_norm_w in fp32, normed = scaled *
    rsqrt(mean(scaled^2) + eps), out[t] = bf16(sum over local slots of w * normed); slots routed
    to other ranks are masked.  y bf16 [T*topk, H].  `rounding` picks the bf16 rounding (see
    numerics.bf16_round)."""
    T, topk = ids.shape
    H = y.shape[1]
    scaled = bf16_round(y.float() * gain.float()[None, :], rounding).view(T, topk, H)
    inv = torch.rsqrt(scaled.pow(2).sum(-1) / H + eps)
    e = ids.long() - expert_lo
    local = (e >= 0) & (e < e_local)
    route = torch.where(local, wts.float(), torch.zeros_like(wts.float()))
    scaled = torch.where(local[:, :, None], scaled, torch.zeros_like(scaled))
    out = (scaled * (inv * route)[:, :, None]).sum(1)
    return out if out_fp32 else bf16_round(out, rounding).to(torch.bfloat16)


def experts(x: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor, w13: torch.Tensor,
            w13_sf: torch.Tensor, w13_gs: torch.Tensor, w2: torch.Tensor, w2_sf: torch.Tensor,
            w2_gs: torch.Tensor, expert_lo: int = 0, return_y: bool = False,
            post_gain: torch.Tensor | None = None, post_eps: float = 1e-8):
    """out[t] = bf16(sum_slot w[t,slot] * y[t*topk + slot]) over local slots, with
    y = bf16(bf16(silu(bf16(x W_g^T)) * bf16(x W_u^T)) W2^T) per routed expert; with
    `post_gain` (fp32 [H] = 1 + post_norm_w) the slots are post-normed first (finalize)."""
    T, H = x.shape
    topk = ids.shape[1]
    e_local, two_i, _ = w13.shape
    inter_dim = two_i // 2
    flat = ids.reshape(-1).long() - expert_lo
    y = torch.zeros((T * topk, H), dtype=torch.bfloat16)
    xb = x.to(torch.bfloat16).float()
    for e in range(e_local):
        p = torch.nonzero(flat == e).reshape(-1)
        if p.numel() == 0:
            continue
        w13d = dequantize(w13[e], w13_sf[e], w13_gs[e]).float()
        h = (xb[p // topk] @ w13d.T).to(torch.bfloat16).float()
        g, u = h[:, :inter_dim], h[:, inter_dim:]
        inter = (torch.nn.functional.silu(g) * u).to(torch.bfloat16).float()
        w2d = dequantize(w2[e], w2_sf[e], w2_gs[e]).float()
        y[p] = (inter @ w2d.T).to(torch.bfloat16)
    if post_gain is not None:
        out = finalize(y, ids, wts, post_gain, expert_lo, e_local, post_eps)
        return (out, y) if return_y else out
    local = ((flat >= 0) & (flat < e_local)).reshape(T, topk)
    wl = torch.where(local, wts.float(), torch.zeros_like(wts.float()))
    out = torch.zeros((T, H), dtype=torch.float32)
    for s in range(topk):
        out += wl[:, s:s + 1] * y.view(T, topk, H)[:, s].float()
    out = out.to(torch.bfloat16)
    return (out, y) if return_y else out
