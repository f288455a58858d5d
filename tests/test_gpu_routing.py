"""GPU parity of Muse's routing path (FP32 router through bf16 hi/lo halves, sigmoid + bias
top-k): okc_router_logits against the fp64 product with the fp32 router (the hi/lo split
keeps 16 mantissa bits of each router weight: relative error ~1e-5), okc_moe_route_sigmoid
against oracle.moe.route_sigmoid on the same logits (ids bit-exact where the biased scores are
not within fp32 rounding of each other; weights within 1e-6), and the muse_bf16_proj problem's
router layer."""

import pytest
import torch

from oracle import moe as omoe

pytestmark = pytest.mark.gpu


def _router(E=256, K=8192, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((E, K), generator=g) * 0.02


@pytest.mark.parametrize("T", [1, 8, 16, 32, 128, 256])
def test_router_logits_hilo(T):
    from okc_b200 import ops
    g = torch.Generator().manual_seed(T)
    x = torch.randn((T, 8192), generator=g).to(torch.bfloat16)
    r = _router()
    hilo = omoe.router_hilo(r)
    got = ops.router_logits(x.cuda(), hilo.cuda()).cpu()
    exact = (x.double() @ r.double().T).float()
    err = (got - exact).norm() / exact.norm()
    assert err < 3e-5, f"relative L2 {err}"
    # the hi/lo sum itself: within fp32 summation of the two halves' products
    two = (x.double() @ hilo[:256].double().T + x.double() @ hilo[256:].double().T).float()
    torch.testing.assert_close(got, two, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("T,topk,with_bias", [(1, 8, True), (7, 8, True), (128, 8, True), (256, 8, False),
                                             (64, 4, True)])
def test_route_sigmoid_vs_oracle(T, topk, with_bias):
    from okc_b200 import ops
    g = torch.Generator().manual_seed(100 + T)
    logits = torch.randn((T, 256), generator=g) * 4.0
    bias = torch.randn(256, generator=g) * 0.05 if with_bias else None
    ids, wts = ops.route_sigmoid(logits.cuda(), bias.cuda() if bias is not None else None, topk)
    rid, rw = omoe.route_sigmoid(logits, bias, topk)
    key = torch.sigmoid(logits * 0.1767766952966369) + (bias if bias is not None else 0)
    srt = key.sort(-1, descending=True).values
    gap = (srt[:, : topk] - srt[:, 1: topk + 1]).min(-1).values
    clear = gap > 1e-6
    assert int(clear.sum()) >= max(1, T // 2)
    assert torch.equal(ids.cpu()[clear], rid[clear])
    torch.testing.assert_close(wts.cpu()[clear], rw[clear], rtol=1e-6, atol=1e-6)
    assert torch.allclose(wts.sum(-1).cpu(), torch.ones(T), atol=1e-5)


def test_route_sigmoid_ties_pick_lower_id():
    from okc_b200 import ops
    logits = torch.zeros((2, 64))
    logits[:, 5] = 3.0
    logits[:, 9] = 3.0
    ids, _ = ops.route_sigmoid(logits.cuda(), None, 3)
    assert ids[0].tolist() == [5, 9, 0]


def test_route_sigmoid_with_lo_half():
    """logits + lo summed before the sigmoid: the same as routing the summed logits."""
    from okc_b200 import ops
    g = torch.Generator().manual_seed(3)
    a = torch.randn((32, 256), generator=g)
    b = torch.randn((32, 256), generator=g) * 1e-3
    ids1, w1 = ops.route_sigmoid(a.cuda(), None, 8, logits_lo=b.cuda())
    ids2, w2 = ops.route_sigmoid((a + b).cuda(), None, 8)
    assert torch.equal(ids1, ids2) and torch.equal(w1, w2)


@pytest.mark.parametrize("m", [1, 32, 128])
def test_bf16_proj_router_layer(m):
    from okc_b200.problems import muse_bf16_proj as prob
    r = _router(seed=1).cuda()
    state = prob.prepare({"router": r})
    g = torch.Generator(device="cuda").manual_seed(m)
    x = torch.randn((m, 8192), generator=g, device="cuda").to(torch.bfloat16)
    y = prob.kernel_fn({"x": x, "config": {"layer": "router", "m": m, "n": 256, "k": 8192}}, state)
    assert y.dtype == torch.float32 and y.shape == (m, 256)
    exact = (x.double() @ r.double().T).float()
    assert ((y - exact).norm() / exact.norm()).item() < 3e-5
