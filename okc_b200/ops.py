"""Torch-facing wrappers of the okc_b200 C ABI.

Each function validates dtypes/devices, allocates its outputs, passes raw pointers and
``torch.cuda.current_stream()`` to libokc_b200.so and returns at once (no host sync), so
every call can be captured in a CUDA graph.  Scratch memory comes from a per-device,
zero-initialised workspace cache (the reference's `_counters` pattern,
muse_attention_decode/submission.py:386-397).  There is no CPU path: a tensor that is
not on a CUDA device raises.
"""

from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import check

_lib.load()  # fail loudly at import if the native library is absent

_WS: dict[tuple[int, str], torch.Tensor] = {}


def _dev_index(t: torch.Tensor) -> int:
    if not t.is_cuda:
        raise _lib.OkcError("okc_b200 operators run on CUDA tensors only (no CPU fallback)")
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def workspace(device: torch.device | int, tag: str, nbytes: int) -> torch.Tensor:
    """Zero-filled scratch of at least `nbytes`, cached per (device, tag).  Grows (and is
    re-zeroed) only when a larger size is asked for; allocate before graph capture."""
    idx = device if isinstance(device, int) else (device.index or 0)
    key = (idx, tag)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        size = max(int(nbytes), 4096)
        buf = torch.zeros(size, dtype=torch.uint8, device=f"cuda:{idx}")
        _WS[key] = buf
    return buf


def read_device_error(tag: str, device: int = 0) -> int:
    """Reads and clears the device error word of workspace `tag` (synchronises)."""
    buf = _WS.get((device, tag))
    if buf is None:
        return 0
    with torch.cuda.device(device):
        return int(_lib.load().okc_read_device_error(buf.data_ptr(), torch.cuda.current_stream(device).cuda_stream))


def _stream(dev: int) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _need(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if t.dtype != dtype:
        raise _lib.OkcError(f"{name}: expected {dtype}, got {t.dtype}")
    if t.dim() >= 1 and t.stride(-1) != 1:
        raise _lib.OkcError(f"{name}: innermost dimension must be contiguous")


# ------------------------------------------------------------------------- projection
def gemm(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None,
         out: torch.Tensor | None = None, out_fp32: bool = False, family: int = 0,
         splits: int = 0) -> torch.Tensor:
    """y[M,N] = x[M,K] @ w[N,K]^T (+ residual), fp32 accumulate, one rounding."""
    dev = _dev_index(x)
    _need(x, torch.bfloat16, "x")
    _need(w, torch.bfloat16, "w")
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise _lib.OkcError(f"shape mismatch x {tuple(x.shape)} w {tuple(w.shape)}")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32 if out_fp32 else torch.bfloat16, device=x.device)
    if residual is not None:
        _need(residual, torch.bfloat16, "residual")
        if residual.stride(0) != out.stride(0):
            raise _lib.OkcError("residual must have the output's row stride")
    lib = _lib.load()
    ws = workspace(dev, "gemm", lib.okc_gemm_bf16_workspace_bytes(M, N, K))
    st = lib.okc_gemm_bf16_ex(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(),
                              out.stride(0), _ptr(residual), M, N, K, int(out_fp32), family, splits,
                              ws.data_ptr(), ws.numel(), _stream(dev))
    check(st, "okc_gemm_bf16")
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, unit_offset: bool = False,
            out: torch.Tensor | None = None) -> torch.Tensor:
    dev = _dev_index(x)
    _need(x, torch.bfloat16, "x")
    _need(w, torch.bfloat16, "w")
    T, H = x.shape
    if out is None:
        out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
    st = _lib.load().okc_rmsnorm_bf16(x.data_ptr(), x.stride(0), w.data_ptr(), out.data_ptr(), out.stride(0),
                                      T, H, float(eps), int(unit_offset), _stream(dev))
    check(st, "okc_rmsnorm_bf16")
    return out


def residual_boundary(stream: torch.Tensor, branch: torch.Tensor, alpha: torch.Tensor, beta: torch.Tensor,
                      post_w: torch.Tensor | None, pre_w: torch.Tensor, post_eps: float = 1e-8,
                      pre_eps: float = 1e-5, stream_out: torch.Tensor | None = None,
                      router: bool = False):
    """Muse's gated residual boundary (okc_residual_boundary): returns (hidden bf16 [T, H],
    stream' fp32 [T, H], router fp32 [T, H] or None).  `stream_out` may be `stream` (in place)."""
    dev = _dev_index(stream)
    _need(stream, torch.float32, "stream")
    _need(branch, torch.bfloat16, "branch")
    _need(alpha, torch.float32, "alpha")
    _need(beta, torch.float32, "beta")
    _need(pre_w, torch.bfloat16, "pre_w")
    if post_w is not None:
        _need(post_w, torch.bfloat16, "post_w")
    T, H = stream.shape
    if not stream.is_contiguous():
        raise _lib.OkcError("stream: must be contiguous")
    hidden = torch.empty((T, H), dtype=torch.bfloat16, device=stream.device)
    if stream_out is None:
        stream_out = torch.empty_like(stream)
    r = torch.empty((T, H), dtype=torch.float32, device=stream.device) if router else None
    st = _lib.load().okc_residual_boundary(stream.data_ptr(), branch.data_ptr(), branch.stride(0), alpha.data_ptr(),
                                           beta.data_ptr(), post_w.data_ptr() if post_w is not None else None,
                                           pre_w.data_ptr(), hidden.data_ptr(), stream_out.data_ptr(),
                                           r.data_ptr() if r is not None else None, T, H, float(post_eps),
                                           float(pre_eps), _stream(dev))
    check(st, "okc_residual_boundary")
    return hidden, stream_out, r


# ------------------------------------------------------------------------- attention
def rope_inv_freq(theta: float, D: int, device) -> torch.Tensor:
    """inv_freq[i] = 1 / theta^(2i/D) in fp32, computed exactly as the reference does
    (muse_prefill_layer/submission.py:102)."""
    return (1.0 / (theta ** (torch.arange(0, D, 2, device=device).float() / D))).contiguous()


def rope_kv_append(qkv: torch.Tensor, positions: torch.Tensor, page_table: torch.Tensor,
                   k_cache: torch.Tensor, v_cache: torch.Tensor, k_scale: torch.Tensor,
                   v_scale: torch.Tensor, Hq: int, Hkv: int, D: int,
                   inv_freq: torch.Tensor | None, q_out: torch.Tensor | None = None,
                   slots_out: torch.Tensor | None = None, q_scale: float = 1.0,
                   qk_norm: bool = False, norm_eps: float = 1e-5) -> torch.Tensor:
    """RoPE the new token's q and k, store e4m3 k/v at slot = table[b][pos//P]*P + pos%P.
    qk_norm / q_scale add Muse's per-head QK RMSNorm and query scale factor.
    Returns q_out bf16 [B, Hq, D]."""
    dev = _dev_index(qkv)
    _need(qkv, torch.bfloat16, "qkv")
    B = qkv.shape[0]
    qkv2 = qkv.reshape(B, -1)
    if q_out is None:
        q_out = torch.empty((B, Hq, D), dtype=torch.bfloat16, device=qkv.device)
    lib = _lib.load()
    ws = workspace(dev, "attn", 256)
    P = k_cache.shape[1]
    st = lib.okc_rope_kv_append_ex(qkv2.data_ptr(), qkv2.stride(0), positions.data_ptr(), page_table.data_ptr(),
                                   page_table.stride(0), page_table.shape[1], _ptr(inv_freq),
                                   k_scale.data_ptr(), v_scale.data_ptr(), q_out.data_ptr(),
                                   k_cache.data_ptr(), v_cache.data_ptr(), _ptr(slots_out), B, Hq, Hkv, D, P,
                                   k_cache.shape[0], float(q_scale), int(qk_norm), float(norm_eps),
                                   ws.data_ptr(), ws.numel(), _stream(dev))
    check(st, "okc_rope_kv_append_ex")
    return q_out


def gemm_rope_kv_append(x: torch.Tensor, wqkv: torch.Tensor, positions: torch.Tensor, page_table: torch.Tensor,
                        k_cache: torch.Tensor, v_cache: torch.Tensor, k_scale: torch.Tensor,
                        v_scale: torch.Tensor, Hq: int, Hkv: int, D: int, inv_freq: torch.Tensor | None,
                        q_out: torch.Tensor | None = None, slots_out: torch.Tensor | None = None,
                        q_scale: float = 1.0) -> torch.Tensor:
    """qkv = x @ wqkv^T with RoPE + FP8 KV-append fused into the tcgen05 GEMM's epilogue
    (okc_gemm_bf16_rope_kv_append): same results as gemm() followed by rope_kv_append()
    without QK-norm.  Returns q_out bf16 [M, Hq, D]."""
    dev = _dev_index(x)
    _need(x, torch.bfloat16, "x")
    _need(wqkv, torch.bfloat16, "wqkv")
    M, K = x.shape
    N = wqkv.shape[0]
    if q_out is None:
        q_out = torch.empty((M, Hq, D), dtype=torch.bfloat16, device=x.device)
    lib = _lib.load()
    ws = workspace(dev, "gemm", lib.okc_gemm_bf16_workspace_bytes(M, N, K))
    P = k_cache.shape[1]
    st = lib.okc_gemm_bf16_rope_kv_append(x.data_ptr(), x.stride(0), wqkv.data_ptr(), wqkv.stride(0), M, N, K,
                                          positions.data_ptr(), page_table.data_ptr(), page_table.stride(0),
                                          page_table.shape[1], _ptr(inv_freq), k_scale.data_ptr(),
                                          v_scale.data_ptr(), q_out.data_ptr(), k_cache.data_ptr(),
                                          v_cache.data_ptr(), _ptr(slots_out), Hq, Hkv, D, P, k_cache.shape[0],
                                          float(q_scale), ws.data_ptr(), ws.numel(), _stream(dev))
    check(st, "okc_gemm_bf16_rope_kv_append")
    return q_out


def attn_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                page_table: torch.Tensor, seq_lens: torch.Tensor, k_scale: torch.Tensor,
                v_scale: torch.Tensor, sm_scale: float, out: torch.Tensor | None = None,
                num_ctas: int = 0, gate: torch.Tensor | None = None,
                out_eps: float = 1e-5, window: int = 0, q_per_seq: int = 1) -> torch.Tensor:
    """Paged FP8 decode attention.  q bf16 [B, Hq, D]; caches e4m3 [pages, P, Hkv, D];
    page_table int32 [B / q_per_seq, max_pages]; seq_lens int32 [B]; scales fp32 [Hkv].  With
    `gate` (bf16 [B, >= Hq*D], Muse's output gate) the result is rms(o) * sigmoid(gate) per
    head.  `window` > 0 restricts a query at position p to the cached positions (p - window, p];
    `q_per_seq` > 1 treats consecutive groups of that many rows as the query tokens of one
    request (a verify block), each row with its own seq_lens (position + 1) and the request's
    page-table row."""
    dev = _dev_index(q)
    _need(q, torch.bfloat16, "q")
    B, Hq, D = q.shape
    pages, P, Hkv, D2 = k_cache.shape
    if D2 != D or v_cache.shape != k_cache.shape:
        raise _lib.OkcError("cache shape mismatch")
    if page_table.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise _lib.OkcError("page_table and seq_lens must be int32")
    if gate is not None:
        _need(gate, torch.bfloat16, "gate")
    if out is None:
        out = torch.empty((B, Hq, D), dtype=torch.bfloat16, device=q.device)
    lib = _lib.load()
    nbytes = lib.okc_attn_decode_workspace_bytes(B, Hq, Hkv, D, num_ctas)
    ws = workspace(dev, "attn", nbytes)
    st = lib.okc_attn_decode_fp8_ex(q.data_ptr(), q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
                                    page_table.data_ptr(), page_table.stride(0), seq_lens.data_ptr(),
                                    k_scale.data_ptr(), v_scale.data_ptr(), out.data_ptr(), out.stride(0),
                                    B, Hq, Hkv, D, P, pages, float(sm_scale), num_ctas, int(window),
                                    int(q_per_seq), _ptr(gate), 0 if gate is None else gate.stride(0),
                                    float(out_eps), ws.data_ptr(), ws.numel(), _stream(dev))
    check(st, "okc_attn_decode_fp8")
    return out


# ------------------------------------------------------------------------------- MoE
def moe_route(x: torch.Tensor, wr: torch.Tensor, topk: int, renormalize: bool = True,
              return_logits: bool = False):
    dev = _dev_index(x)
    _need(x, torch.bfloat16, "x")
    _need(wr, torch.bfloat16, "router")
    T, H = x.shape
    E = wr.shape[0]
    ids = torch.empty((T, topk), dtype=torch.int32, device=x.device)
    wts = torch.empty((T, topk), dtype=torch.float32, device=x.device)
    logits = torch.empty((T, E), dtype=torch.float32, device=x.device) if return_logits else None
    st = _lib.load().okc_moe_route(x.data_ptr(), wr.data_ptr(), ids.data_ptr(), wts.data_ptr(), _ptr(logits),
                                   T, H, E, topk, int(renormalize), _stream(dev))
    check(st, "okc_moe_route")
    return (ids, wts, logits) if return_logits else (ids, wts)


def route_sigmoid(logits: torch.Tensor, bias: torch.Tensor | None, topk: int,
                  logits_lo: torch.Tensor | None = None, scale: float = 0.1767766952966369,
                  eps: float = 1e-15, route_scale: float = 1.0):
    """Muse's sigmoid + bias routing (okc_moe_route_sigmoid): ids int32 [T, k], weights fp32."""
    dev = _dev_index(logits)
    _need(logits, torch.float32, "logits")
    T, E = logits.shape
    ids = torch.empty((T, topk), dtype=torch.int32, device=logits.device)
    wts = torch.empty((T, topk), dtype=torch.float32, device=logits.device)
    st = _lib.load().okc_moe_route_sigmoid(logits.data_ptr(), logits.stride(0),
                                           logits_lo.data_ptr() if logits_lo is not None else None,
                                           bias.data_ptr() if bias is not None else None, ids.data_ptr(),
                                           wts.data_ptr(), None, T, E, topk, float(scale), float(eps),
                                           float(route_scale), _stream(dev))
    check(st, "okc_moe_route_sigmoid")
    return ids, wts


def router_logits(x: torch.Tensor, w_hilo: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 logits of the bf16 x against the fp32 router held as stacked bf16 [hi; lo] halves."""
    dev = _dev_index(x)
    _need(x, torch.bfloat16, "x")
    _need(w_hilo, torch.bfloat16, "w_hilo")
    T, K = x.shape
    E = w_hilo.shape[0] // 2
    if out is None:
        out = torch.empty((T, E), dtype=torch.float32, device=x.device)
    lib = _lib.load()
    ws = workspace(dev, "router", lib.okc_router_logits_workspace_bytes(T, E, K))
    st = lib.okc_router_logits(x.data_ptr(), x.stride(0), w_hilo.data_ptr(), out.data_ptr(), out.stride(0), T, E, K,
                               ws.data_ptr(), ws.numel(), _stream(dev))
    check(st, "okc_router_logits")
    return out


def moe_max_tiles(T: int, topk: int, E_local: int, bm: int) -> int:
    n = T * topk
    return min(E_local, n) + (n + bm - 1) // bm


def moe_permute(ids: torch.Tensor, expert_lo: int, E_local: int, bm: int = 8) -> dict:
    dev = _dev_index(ids)
    T, topk = ids.shape
    mt = moe_max_tiles(T, topk, E_local, bm)
    counts = torch.empty(E_local, dtype=torch.int32, device=ids.device)
    offsets = torch.empty(E_local + 1, dtype=torch.int32, device=ids.device)
    pairs = torch.empty(T * topk, dtype=torch.int32, device=ids.device)
    tiles = torch.empty(1 + mt, dtype=torch.int32, device=ids.device)
    ids_c = ids.contiguous()
    st = _lib.load().okc_moe_permute(ids_c.data_ptr(), T, topk, expert_lo, E_local, bm, counts.data_ptr(),
                                     offsets.data_ptr(), pairs.data_ptr(), tiles.data_ptr(), mt, _stream(dev))
    check(st, "okc_moe_permute")
    return {"counts": counts, "offsets": offsets, "pairs": pairs, "tiles": tiles}


def moe_experts(x: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor, perm: dict,
                w13: torch.Tensor, w13_sf: torch.Tensor, w13_gs: torch.Tensor,
                w2: torch.Tensor, w2_sf: torch.Tensor, w2_gs: torch.Tensor, expert_lo: int,
                out: torch.Tensor | None = None, out_fp32: bool = False,
                post_gain: torch.Tensor | None = None, post_eps: float = 1e-8) -> torch.Tensor:
    """Routing-weighted sum of the local experts' SwiGLU MLPs ([T, H]; bf16, or with out_fp32
    the unrounded fp32 share of an expert-parallel sum).  With `post_gain` (fp32 [H] =
    1 + post_norm_w) each slot gets Muse's post-expert RMSNorm first."""
    dev = _dev_index(x)
    _need(x, torch.bfloat16, "x")
    T, H = x.shape
    topk = ids.shape[1]
    E_local, two_i, _ = w13.shape
    I = two_i // 2
    if out is None:
        out = torch.empty((T, H), dtype=torch.float32 if out_fp32 else torch.bfloat16, device=x.device)
    lib = _lib.load()
    ws = workspace(dev, "moe", lib.okc_moe_experts_workspace_bytes(T, topk, H, I))
    if post_gain is not None:
        _need(post_gain, torch.float32, "post_gain")
    st = lib.okc_moe_experts_w4a16_post(x.data_ptr(), ids.data_ptr(), wts.data_ptr(), perm["counts"].data_ptr(),
                                        perm["offsets"].data_ptr(), perm["pairs"].data_ptr(), w13.data_ptr(),
                                        w13_sf.data_ptr(), w13_gs.data_ptr(), w2.data_ptr(), w2_sf.data_ptr(),
                                        w2_gs.data_ptr(), out.data_ptr(), T, topk, H, I, expert_lo, E_local,
                                        int(out_fp32), post_gain.data_ptr() if post_gain is not None else None,
                                        float(post_eps), ws.data_ptr(), ws.numel(), _stream(dev))
    check(st, "okc_moe_experts_w4a16")
    return out


def attn_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, page_table: torch.Tensor,
                 positions: torch.Tensor, k_scale: torch.Tensor, v_scale: torch.Tensor, sm_scale: float,
                 B: int, L: int, gate: torch.Tensor | None = None, out_eps: float = 1e-5, window: int = 0,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Prefill-block attention (okc_attn_prefill_fp8): q bf16 [B*L, Hq, D] (rows request-major),
    caches e4m3 [pages, P, Hkv, D], page_table int32 [B, max_pages], positions int64 [B*L];
    returns bf16 [B*L, Hq, D] (with `gate`: Muse's rms(o) * sigmoid(gate) per head)."""
    dev = _dev_index(q)
    _need(q, torch.bfloat16, "q")
    T, Hq, D = q.shape
    if T != B * L:
        raise _lib.OkcError(f"q has {T} rows, B * L = {B * L}")
    Hkv = k_cache.shape[2]
    if out is None:
        out = torch.empty((T, Hq, D), dtype=torch.bfloat16, device=q.device)
    if gate is not None:
        _need(gate, torch.bfloat16, "gate")
    lib = _lib.load()
    ws = workspace(dev, "attn_prefill", 256)
    st = lib.okc_attn_prefill_fp8(q.data_ptr(), q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
                                  page_table.data_ptr(), page_table.stride(0), page_table.shape[1],
                                  positions.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(), _ptr(gate),
                                  gate.stride(0) if gate is not None else 0, float(out_eps), out.data_ptr(),
                                  out.stride(0), B, L, Hq, Hkv, D, k_cache.shape[1], k_cache.shape[0],
                                  float(sm_scale), int(window), ws.data_ptr(), ws.numel(), _stream(dev))
    check(st, "okc_attn_prefill_fp8")
    return out


def attn_workspace_bytes(B: int, Hq: int, Hkv: int, D: int, num_ctas: int = 0) -> int:
    return int(_lib.load().okc_attn_decode_workspace_bytes(B, Hq, Hkv, D, num_ctas))


def sm_scale_default(D: int) -> float:
    return 1.0 / math.sqrt(D)
