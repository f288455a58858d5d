"""GPU parity of the prefill-block attention (okc_attn_prefill_fp8 through ops.attn_prefill)
against the CPU oracle: each of a request's L new tokens attends the positions <= its own (and
inside the window) of the request's paged e4m3 cache, its block's keys appended first.

Cases: Muse's shape (16 q / 2 kv heads of 64, page 1, QK-RMSNorm + RoPE + output gate) against
oracle.attention.muse_attention (append + attention); a plain shape (8 q / 2 kv heads of 128,
4 query heads per KV head, page 16, window 256, per-head scales 1/64 .. 2) against
oracle.attention.attend.  Tolerance: rtol 2e-2 / atol 2e-2 and relative L2 < 1e-2 on the bf16
outputs."""

import math

import pytest
import torch

from oracle import attention as oatt

pytestmark = pytest.mark.gpu


def _close(out, exp, what):
    o, e = out.float().cpu(), exp.float().cpu()
    torch.testing.assert_close(o, e, rtol=2e-2, atol=2e-2, msg=what)
    assert (o - e).norm() / e.norm().clamp_min(1e-30) < 1e-2, what


def _layout(B, L, ctx, page, hkv, d, g, scale):
    from okc_b200 import synth
    lens = torch.randint(ctx[0], ctx[1] + 1, (B,), generator=g, device="cuda")
    lens_l = [int(v) for v in lens.tolist()]
    pool = sum(math.ceil((n + L) / page) for n in lens_l) + 3
    table = synth.paged_layout(lens_l, page, pool, g, "cuda", extra_tokens=L)
    kc = torch.empty((pool, page, hkv, d), dtype=torch.float8_e4m3fn, device="cuda")
    vc = torch.empty_like(kc)
    synth.fill_e4m3_normal(kc, g, scale)
    synth.fill_e4m3_normal(vc, g, scale)
    pos = (lens.long()[:, None] + torch.arange(L, device="cuda")).reshape(-1)
    return table, kc, vc, pos


@pytest.mark.parametrize("B,L,ctx,window", [(2, 64, (100, 300), 0), (1, 200, (600, 900), 2048), (3, 24, (0, 50), 0)])
def test_prefill_attention_muse(B, L, ctx, window):
    from okc_b200 import ops
    hq, hkv, d = 16, 2, 64
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + L)
    table, kc, vc, pos = _layout(B, L, ctx, 1, hkv, d, g, torch.ones(hkv, device="cuda"))
    qkv = torch.randn((B * L, (2 * hq + 2 * hkv) * d), generator=g, device="cuda").to(torch.bfloat16)
    cfg = {"batch": B, "q_len": L, "num_q_heads": hq, "num_kv_heads": hkv, "head_dim": d, "page_size": 1,
           "window": window, "rope_theta": 5e5, "qk_scale_factor": 5.4730064863875, "sm_scale": 0.125}
    ks = torch.ones(hkv, device="cuda")
    kc_ref, vc_ref = kc.cpu().clone(), vc.cpu().clone()
    exp = oatt.muse_attention(qkv.cpu(), pos.cpu(), table.cpu(), kc_ref, vc_ref, ks.cpu(), ks.cpu(), cfg)
    inv = ops.rope_inv_freq(5e5, d, "cuda")
    q = torch.empty((B * L, hq, d), dtype=torch.bfloat16, device="cuda")
    for b in range(B):
        r = slice(b * L, (b + 1) * L)
        ops.rope_kv_append(qkv[r], pos[r], table[b:b + 1].expand(L, -1), kc, vc, ks, ks, hq, hkv, d, inv, q_out=q[r],
                           q_scale=cfg["qk_scale_factor"], qk_norm=True)
    gate = qkv[:, (hq + 2 * hkv) * d:]
    out = ops.attn_prefill(q, kc, vc, table, pos, ks, ks, cfg["sm_scale"], B, L, gate=gate, window=window)
    torch.cuda.synchronize()
    assert ops.read_device_error("attn_prefill") == 0
    _close(out.view(B * L, -1), exp, f"muse B{B} L{L} window{window}")


def test_prefill_attention_plain_d128():
    from okc_b200 import ops
    B, L, hq, hkv, d, page, window = 3, 40, 8, 2, 128, 16, 256
    g = torch.Generator(device="cuda").manual_seed(77)
    scale = torch.tensor([1 / 64, 2.0], device="cuda")
    table, kc, vc, pos = _layout(B, L, (500, 900), page, hkv, d, g, scale)
    q = (torch.randn((B * L, hq, d), generator=g, device="cuda") * 3).to(torch.bfloat16)
    out = ops.attn_prefill(q, kc, vc, table, pos, scale, scale, 1 / math.sqrt(d), B, L, window=window)
    torch.cuda.synchronize()
    exp = oatt.attend(q.cpu(), kc.cpu(), vc.cpu(), table.cpu(), (pos + 1).to(torch.int32).cpu(), scale.cpu(),
                      scale.cpu(), 1 / math.sqrt(d), window=window, q_per_seq=L)
    _close(out, exp.to(torch.bfloat16), "plain d128 window 256")
