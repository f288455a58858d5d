"""GPU parity of Muse's gated residual boundary (okc_residual_boundary) against
oracle.layer.residual_boundary (muse_decode_layer/decode/boundaries.py:17-50) on the same
seeded inputs: the fp32 stream and router rows within rtol/atol 1e-5 (the kernel and the
oracle sum the squares in different orders), the bf16 hidden within one bf16 step."""

import pytest
import torch

from oracle import layer as olayer

pytestmark = pytest.mark.gpu


def _inputs(T, H, seed, ld=None):
    g = torch.Generator().manual_seed(seed)
    stream = torch.randn((T, H), generator=g) * 3.0
    ld = ld or H
    branch = (torch.randn((T, ld), generator=g) * 0.5).to(torch.bfloat16)
    gate = torch.randn(H, generator=g)
    beta = torch.rand(H, generator=g) * 0.3
    # the reference's constants (muse_decode_layer/submission.py:625-626)
    alpha = torch.sqrt(torch.clamp(torch.sigmoid(-gate) * (1.0 + beta), min=1e-3))
    post_w = (torch.randn(H, generator=g) * 0.1).to(torch.bfloat16)
    pre_w = (torch.randn(H, generator=g) * 0.1).to(torch.bfloat16)
    return stream, branch, alpha, beta, post_w, pre_w


def _step_close(got, exp):
    got, exp = got.float(), exp.float()
    step = torch.exp2(torch.floor(torch.log2(torch.maximum(got.abs(), exp.abs()).clamp_min(2 ** -100))) - 7)
    assert bool(((got - exp).abs() <= step).all()), f"max diff {(got - exp).abs().max()}"


@pytest.mark.parametrize("T,H,scaled,ld", [(1, 8192, False, None), (8, 8192, True, None), (128, 8192, False, None),
                                           (5, 4096, True, 4160), (3, 16384, True, None), (2, 8200, False, None)])
def test_boundary_vs_oracle(T, H, scaled, ld):
    from okc_b200 import ops
    stream, branch, alpha, beta, post_w, pre_w = _inputs(T, H, T + H, ld)
    d = lambda t: t.cuda()
    h, st, r = ops.residual_boundary(d(stream), d(branch)[:, :H], d(alpha), d(beta), d(post_w) if scaled else None,
                                     d(pre_w), router=True)
    eh, est, er = olayer.residual_boundary(stream, branch[:, :H], alpha, beta, post_w if scaled else None, pre_w)
    torch.testing.assert_close(st.cpu(), est, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(r.cpu(), er, rtol=1e-5, atol=1e-5)
    _step_close(h.cpu(), eh)


def test_boundary_in_place_and_without_router():
    from okc_b200 import ops
    stream, branch, alpha, beta, post_w, pre_w = _inputs(16, 8192, 3)
    s = stream.cuda()
    h1, st1, r1 = ops.residual_boundary(s, branch.cuda(), alpha.cuda(), beta.cuda(), None, pre_w.cuda())
    assert r1 is None
    s2 = stream.cuda()
    h2, st2, _ = ops.residual_boundary(s2, branch.cuda(), alpha.cuda(), beta.cuda(), None, pre_w.cuda(),
                                       stream_out=s2)
    assert st2.data_ptr() == s2.data_ptr()
    assert torch.equal(st2, st1) and torch.equal(h2, h1)
