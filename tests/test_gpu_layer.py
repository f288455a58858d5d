"""GPU parity of one decode step of the layer (okc_b200.layer.DecodeLayer) against the CPU
oracle (oracle.layer.decode_layer): the small decode-layer config exactly, a mid-size case, and a
CUDA-graph replay of the step.  Tolerance: rtol 2e-2 / atol 2e-2 on the bf16 output, cache
append slots bit-exact."""

import math

import pytest
import torch

from oracle import layer as olayer

pytestmark = pytest.mark.gpu


def _run(B, H, Hq, Hkv, D, lens, page, pool, theta, seed):
    from okc_b200 import synth
    from okc_b200.layer import DecodeLayer, LayerConfig
    g = torch.Generator(device="cuda").manual_seed(seed)
    table = synth.paged_layout(lens, page, pool, g, "cuda", extra_tokens=1)
    kc = torch.empty((pool, page, Hkv, D), dtype=torch.float8_e4m3fn, device="cuda")
    vc = torch.empty_like(kc)
    ks = (torch.rand(Hkv, generator=g, device="cuda") * 1.5 + 0.5).float()
    vs = (torch.rand(Hkv, generator=g, device="cuda") * 1.5 + 0.5).float()
    synth.fill_e4m3_normal(kc, g, ks)   # e4m3(N(0,1) / scale_h), as the small config
    synth.fill_e4m3_normal(vc, g, vs)
    x = torch.randn((B, H), generator=g, device="cuda").to(torch.bfloat16)
    nw = (1 + 0.02 * torch.randn(H, generator=g, device="cuda")).to(torch.bfloat16)
    wqkv = (torch.randn(((Hq + 2 * Hkv) * D, H), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    wo = (torch.randn((H, Hq * D), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    pos = torch.tensor(lens, dtype=torch.int64, device="cuda")
    cfg = LayerConfig(hidden=H, num_q_heads=Hq, num_kv_heads=Hkv, head_dim=D, rope_theta=theta, eps=1e-6,
                      page_size=page)
    kc_ref, vc_ref = kc.cpu().clone(), vc.cpu().clone()
    layer = DecodeLayer(cfg, nw, wqkv, wo, ks, vs)
    out = layer.step(x, pos, table, kc, vc)
    exp, slots = olayer.decode_layer(x.cpu(), nw.cpu(), wqkv.cpu(), wo.cpu(), pos.cpu(), table.cpu(), kc_ref,
                                     vc_ref, ks.cpu(), vs.cpu(), Hq, Hkv, D, theta, 1e-6, D ** -0.5)
    torch.cuda.synchronize()
    return layer, (x, pos, table, kc, vc), out, exp, slots, (kc_ref, vc_ref)


def _check(out, exp, what):
    o, e = out.float().cpu(), exp.float()
    torch.testing.assert_close(o, e, rtol=2e-2, atol=2e-2, msg=what)
    assert (o - e).norm() / e.norm() < 1e-2, what


def test_baseline_config0_smoke():
    """Small decode-layer config: batch 2, hidden 1024, 8q/2kv, D128, theta 1e4, eps 1e-6, P16, 64 pages,
    ctx {37, 200}, weights ~N(0, 0.02), x ~N(0, 1)."""
    layer, ins, out, exp, slots, caches = _run(2, 1024, 8, 2, 128, [37, 200], 16, 64, 1e4, 0)
    _check(out, exp, "configs[0]")
    # the appended K/V rows land at the oracle's slots; every other row is untouched
    kc, vc = ins[3].cpu(), ins[4].cpu()
    flat_k, ref_k = kc.view(torch.uint8).view(-1, 2 * 128), caches[0].view(torch.uint8).view(-1, 2 * 128)
    mask = torch.ones(flat_k.shape[0], dtype=torch.bool)
    mask[slots] = False
    assert torch.equal(flat_k[mask], ref_k[mask])
    assert torch.equal(vc.view(torch.uint8).view(-1, 256)[~mask], caches[1].view(torch.uint8).view(-1, 256)[~mask])


def test_mid_size_layer_and_graph_replay():
    lens = [1024, 3000, 17, 4096, 555, 8192, 2049, 100]
    layer, ins, out, exp, _, _ = _run(8, 4096, 32, 4, 128, lens, 16, sum(math.ceil((n + 1) / 16) for n in lens) + 8,
                                      5e5, 1)
    _check(out, exp, "mid-size")
    x, pos, table, kc, vc = ins
    res = torch.empty_like(out)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer.step(x, pos, table, kc, vc, out=res)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        layer.step(x, pos, table, kc, vc, out=res)
    g.replay()  # same inputs: the append rewrites the same slots, so the step is idempotent
    torch.cuda.synchronize()
    _check(res, exp, "graph replay")
