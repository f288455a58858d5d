"""The QKV projection with RoPE + FP8 KV-append fused into its epilogue
(okc_gemm_bf16_rope_kv_append) against the unfused pair (okc_gemm_bf16 then
okc_rope_kv_append) on the same inputs: q, every cache byte and the slots bit-exact (the fused
path rounds the projection to bf16 and then applies the same arithmetic)."""

import pytest
import torch

from okc_b200 import ops, synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,H,Hq,Hkv,D,P", [(128, 8192, 64, 8, 128, 16), (48, 1024, 8, 2, 64, 16),
                                            (200, 2048, 16, 4, 128, 32), (64, 1024, 8, 1, 128, 16)])
def test_fused_matches_unfused(M, H, Hq, Hkv, D, P):
    g = torch.Generator(device="cuda").manual_seed(M + H)
    x = torch.randn((M, H), generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(((Hq + 2 * Hkv) * D, H), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    pages = 4 * M + 8
    kc0 = torch.randint(0, 255, (pages, P, Hkv, D), generator=g, device="cuda", dtype=torch.uint8)
    vc0 = torch.randint(0, 255, (pages, P, Hkv, D), generator=g, device="cuda", dtype=torch.uint8)
    ks = (torch.rand(Hkv, generator=g, device="cuda") * 1.5 + 0.5).float()
    vs = (torch.rand(Hkv, generator=g, device="cuda") * 1.5 + 0.5).float()
    table = torch.randperm(pages, generator=g, device="cuda").to(torch.int32)[: M * 4].view(M, 4).contiguous()
    pos = torch.randint(0, 4 * P, (M,), generator=g, device="cuda").long()
    inv = ops.rope_inv_freq(5e5, D, "cuda")
    kc_a, vc_a, kc_b, vc_b = kc0.clone(), vc0.clone(), kc0.clone(), vc0.clone()
    sl_a = torch.empty(M, dtype=torch.int64, device="cuda")
    sl_b = torch.empty(M, dtype=torch.int64, device="cuda")
    qkv = ops.gemm(x, w, family=2)
    q_a = ops.rope_kv_append(qkv, pos, table, kc_a, vc_a, ks, vs, Hq, Hkv, D, inv, slots_out=sl_a)
    q_b = ops.gemm_rope_kv_append(x, w, pos, table, kc_b, vc_b, ks, vs, Hq, Hkv, D, inv, slots_out=sl_b)
    torch.cuda.synchronize()
    assert torch.equal(sl_a, sl_b)
    assert torch.equal(q_a.view(torch.int16), q_b.view(torch.int16)), "q differs"
    assert torch.equal(kc_a, kc_b), "k cache differs"
    assert torch.equal(vc_a, vc_b), "v cache differs"
    assert ops.read_device_error("gemm") == 0
