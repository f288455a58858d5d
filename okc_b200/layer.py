"""One decode step of a transformer layer (the decode-layer workload: hidden 8192, 64q/8kv heads, batch 128), B200-native.

    x -> RMSNorm -> QKV projection -> RoPE + FP8 KV-append -> paged attention
      -> O projection (+ residual) -> out
(above 32 tokens the RoPE + KV-append run in the QKV projection's epilogue)

Every stage is an okc_b200 kernel; the step is captured in one CUDA graph by the caller
(bench.py) so launch latency does not count.  Tensor parallel over `world` ranks: rank r
owns query heads [r*Hq/W, (r+1)*Hq/W) and KV heads [r*Hkv/W, ...) — its slice of the
QKV weight (column parallel, no communication) and of its own paged cache; the O
projection is row parallel, and one tcgen05 kernel computes it and sums the ranks' partials
over NVLink peer memory with the residual (okc_b200.comm.TPComm; fallback: an fp32 partial
GEMM followed by the peer-memory exchange kernel).  Mirrors the composition of
muse_decode_layer/decode/runtime.py:47-75 (attention -> O -> boundary) without Muse's
gated residual, QK-norm and output gate, which this plain layer (RMSNorm, x + O) does not have.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


@dataclass
class LayerConfig:
    hidden: int = 8192
    num_q_heads: int = 64
    num_kv_heads: int = 8
    head_dim: int = 128
    rope_theta: float = 5e5
    eps: float = 1e-6
    page_size: int = 16


def shard_weights(wqkv: torch.Tensor, wo: torch.Tensor, cfg: LayerConfig, rank: int, world: int):
    """Column-parallel QKV rows and row-parallel O columns of one TP rank."""
    hq, hkv, d = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
    if hq % world or hkv % world:
        raise ValueError(f"heads ({hq}q/{hkv}kv) must divide by the TP degree {world}")
    lq, lkv = hq // world, hkv // world
    q = wqkv[:hq * d].view(hq, d, -1)[rank * lq:(rank + 1) * lq].reshape(lq * d, -1)
    k = wqkv[hq * d:(hq + hkv) * d].view(hkv, d, -1)[rank * lkv:(rank + 1) * lkv].reshape(lkv * d, -1)
    v = wqkv[(hq + hkv) * d:].view(hkv, d, -1)[rank * lkv:(rank + 1) * lkv].reshape(lkv * d, -1)
    wqkv_l = torch.cat([q, k, v], 0).contiguous()
    wo_l = wo[:, rank * lq * d:(rank + 1) * lq * d].contiguous()
    return wqkv_l, wo_l


class DecodeLayer:
    """prepare once (untimed), then step(x, positions, page_table) per decode step."""

    def __init__(self, cfg: LayerConfig, norm_w, wqkv, wo, k_scale, v_scale, rank=0, world=1,
                 group=None):
        self.cfg, self.rank, self.world, self.group = cfg, rank, world, group
        self.lq = cfg.num_q_heads // world
        self.lkv = cfg.num_kv_heads // world
        self.norm_w = norm_w.contiguous()
        if world > 1:
            self.wqkv, self.wo = shard_weights(wqkv, wo, cfg, rank, world)
            sl = slice(rank * self.lkv, (rank + 1) * self.lkv)
            self.k_scale, self.v_scale = k_scale[sl].contiguous(), v_scale[sl].contiguous()
        else:
            self.wqkv, self.wo = wqkv.contiguous(), wo.contiguous()
            self.k_scale, self.v_scale = k_scale.contiguous(), v_scale.contiguous()
        self.inv_freq = ops.rope_inv_freq(cfg.rope_theta, cfg.head_dim, norm_w.device)
        self.sm_scale = cfg.head_dim ** -0.5
        self._comms = {}

    def kernels_per_step(self, tokens: int) -> int:
        """Our kernel launches in one step (for the bench's gpu_launches)."""
        passes = 1 if tokens <= 256 else (tokens + 255) // 256  # tcgen05 GEMM: 256 tokens a launch
        per_gemm = 2 * passes if tokens > 32 else 1  # tcgen05 stream-K + split-tile reduce
        rope = 0 if tokens > 32 else 1  # fused into the QKV reduce on the tcgen05 path
        oproj = per_gemm
        if self.world > 1:
            c = self._comms.get(tokens)
            oproj = 1 if (c is not None and c.fused) else per_gemm + 1
        return 1 + per_gemm + rope + 2 + oproj

    def step(self, x, positions, page_table, k_cache, v_cache, lens=None, out=None):
        """x bf16 [B, H]; positions int64 [B] (= tokens already cached); caches of this rank's
        KV heads; returns bf16 [B, H] (replicated on every rank)."""
        cfg, d = self.cfg, self.cfg.head_dim
        B = x.shape[0]
        xn = ops.rmsnorm(x, self.norm_w, cfg.eps)
        if B > 32:  # tcgen05 projection with RoPE + KV-append in its epilogue
            q = ops.gemm_rope_kv_append(xn, self.wqkv, positions, page_table, k_cache, v_cache, self.k_scale,
                                        self.v_scale, self.lq, self.lkv, d, self.inv_freq)
        else:
            qkv = ops.gemm(xn, self.wqkv)
            q = ops.rope_kv_append(qkv, positions, page_table, k_cache, v_cache, self.k_scale, self.v_scale,
                                   self.lq, self.lkv, d, self.inv_freq)
        if lens is None:
            lens = (positions + 1).to(torch.int32)
        o = ops.attn_decode(q, k_cache, v_cache, page_table, lens, self.k_scale, self.v_scale, self.sm_scale)
        o2 = o.view(B, self.lq * d)
        if self.world == 1:
            return ops.gemm(o2, self.wo, residual=x, out=out)
        return self.o_proj_allreduce(o2, x, out)

    def comm_for(self, tokens: int):
        """The NVLink exchange group for `tokens` rows (created on first use: a collective
        call, so every rank must reach it together and outside CUDA-graph capture)."""
        from .comm import TPComm
        c = self._comms.get(tokens)
        if c is None:
            c = TPComm(tokens, self.cfg.hidden, group=self.group, oproj_k=self.lq * self.cfg.head_dim)
            self._comms[tokens] = c
        return c

    def o_proj_allreduce(self, o2, x, out=None):
        """Row-parallel O projection and out = bf16(x + sum over ranks): one fused tcgen05 +
        NVLink kernel (okc_tp_oproj_allreduce_residual) where the shape allows, else the fp32
        partial GEMM followed by the peer-memory exchange kernel (okc_tp_allreduce_residual)."""
        comm = self.comm_for(x.shape[0])
        if comm.fused:
            res = comm.oproj_allreduce_residual(o2, self.wo, x)
        else:
            ops.gemm(o2, self.wo, out_fp32=True, out=comm.partial)
            res = comm.allreduce_residual(x)
        if out is not None:
            out.copy_(res)
            return out
        return res

    def close(self):
        for c in self._comms.values():
            c.close()
        self._comms.clear()
