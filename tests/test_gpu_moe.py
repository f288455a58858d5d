"""GPU parity of the W4A16 MoE path: routing ids and permutation bit-exact, expert outputs
within rtol 2e-2 / atol 2e-2 (the path's stated tolerance) and relative-L2 below 1e-2.

The oracle dequantises weights as bf16(e2m1 * f32(sf * gs)) (the reference's nibble decoder);
the kernel multiplies the exact e2m1 * sf product by gs on the fp32 accumulator — the two
differ by one bf16 rounding per weight, far inside the tolerance."""

import pytest
import torch

from oracle import moe as ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from okc_b200 import ops
    return ops


@pytest.fixture(scope="module")
def bank():
    from okc_b200 import synth
    return synth.moe_case(T=256, device="cuda", seed=0)


@pytest.mark.parametrize("T", [1, 8, 64, 256])
def test_route_ids_bit_exact(ops, bank, T):
    x = bank["x"][:T]
    ids, wts, lg = ops.moe_route(x, bank["router"], 8, renormalize=True, return_logits=True)
    rid, rw, rlg = ref.route(x.cpu(), bank["router"].cpu(), 8, True)
    assert torch.equal(lg.cpu(), rlg), "router logits must be bit-exact (fixed summation order)"
    assert torch.equal(ids.cpu(), rid), "expert ids must be bit-exact"
    torch.testing.assert_close(wts.cpu(), rw, rtol=1e-5, atol=1e-6)
    ids2, wts2 = ops.moe_route(x, bank["router"], 8, renormalize=False)
    rid2, rw2, _ = ref.route(x.cpu(), bank["router"].cpu(), 8, False)
    assert torch.equal(ids2.cpu(), rid2)
    torch.testing.assert_close(wts2.cpu(), rw2, rtol=1e-5, atol=1e-6)


def test_route_ids_match_plain_fp32_topk(ops, bank):
    """The ids against the reference's plain routing, softmax top-k of x.float() @ Wr.float().T
    (muse_prefill_layer/submission.py:179-184 computes the logits so), not against a copy of the
    kernel's summation order.  The kernel rounds its logits to bf16, so ids can only be pinned
    where the ranking is not decided inside one bf16 step: on tokens whose top-9 plain-fp32
    logits are pairwise more than two bf16 steps apart, ids (and their order) must be equal;
    weights within 2e-2 of the plain softmax over the chosen logits."""
    x = bank["x"]
    ids, wts = ops.moe_route(x, bank["router"], 8, renormalize=True)
    lg = x.float().cpu() @ bank["router"].float().cpu().T
    top = lg.topk(9, dim=-1)
    vals = top.values
    gap = vals[:, :-1] - vals[:, 1:]
    ulp = torch.exp2(torch.floor(torch.log2(vals.abs().clamp_min(1e-30))) - 7)  # bf16 step at each logit
    clear = (gap > 2 * torch.maximum(ulp[:, :-1], ulp[:, 1:])).all(-1)
    assert int(clear.sum()) >= 32, f"too few clearly ranked tokens ({int(clear.sum())}) for a meaningful check"
    got, exp = ids.cpu()[clear], top.indices[clear, :8].to(torch.int32)
    assert torch.equal(got, exp), "ids differ from the plain fp32 top-k on clearly ranked tokens"
    ref_w = torch.softmax(vals[clear, :8], -1)
    torch.testing.assert_close(wts.cpu()[clear], ref_w, rtol=2e-2, atol=2e-2)


def test_route_ties_pick_lower_id(ops):
    # identical router rows give identical logits: ties must resolve to the lower expert id
    wr = torch.zeros((64, 256), dtype=torch.bfloat16, device="cuda")
    wr[10] = 0.5
    wr[3] = 0.5
    wr[40] = 0.5
    x = torch.ones((2, 256), dtype=torch.bfloat16, device="cuda")
    ids, _ = ops.moe_route(x, wr, 4)
    rid, _, _ = ref.route(x.cpu(), wr.cpu(), 4)
    assert torch.equal(ids.cpu(), rid)
    assert ids[0].tolist() == [3, 10, 40, 0]


@pytest.mark.parametrize("T,lo,E", [(1, 0, 64), (8, 0, 64), (33, 0, 64), (256, 0, 64), (256, 16, 8), (5, 60, 4)])
def test_permute_bit_exact(ops, T, lo, E):
    g = torch.Generator().manual_seed(T + lo)
    ids = torch.stack([torch.randperm(64, generator=g)[:8] for _ in range(T)]).to(torch.int32)
    perm = ops.moe_permute(ids.cuda(), lo, E, bm=8)
    counts, offsets, pairs, tiles = ref.permute(ids, lo, E, 8)
    assert torch.equal(perm["counts"].cpu(), counts)
    assert torch.equal(perm["offsets"].cpu(), offsets)
    assert torch.equal(perm["pairs"].cpu()[: int(offsets[-1])], pairs)
    n = int(tiles[0])
    assert torch.equal(perm["tiles"].cpu()[: n + 1], tiles)


@pytest.mark.parametrize("T", [1, 8, 16, 32, 64, 100, 256])
def test_experts(ops, bank, T):
    """T <= 64: the row-owning kernel (token tiles of 8/16/32/64); T = 100 and the MoE workload's
    largest batch T = 256: the per-expert kernel."""
    x = bank["x"][:T]
    ids, wts = ops.moe_route(x, bank["router"], 8)
    perm = ops.moe_permute(ids, 0, 64)
    out = ops.moe_experts(x, ids, wts, perm, bank["w13"], bank["w13_sf"], bank["w13_gs"],
                          bank["w2"], bank["w2_sf"], bank["w2_gs"], 0)
    torch.cuda.synchronize()
    cpu = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in bank.items()}
    exp = ref.experts(x.cpu(), ids.cpu(), wts.cpu(), cpu["w13"], cpu["w13_sf"], cpu["w13_gs"],
                      cpu["w2"], cpu["w2_sf"], cpu["w2_gs"])
    o, e = out.float().cpu(), exp.float()
    torch.testing.assert_close(o, e, rtol=2e-2, atol=2e-2)
    assert (o - e).norm() / e.norm() < 1e-2


def test_experts_expert_parallel_slice(ops, bank):
    """Experts 16..23 only (one EP rank of 8): non-local slots contribute nothing."""
    T = 8
    x = bank["x"][:T]
    ids, wts = ops.moe_route(x, bank["router"], 8)
    lo, E = 16, 8
    perm = ops.moe_permute(ids, lo, E)
    sl = slice(lo, lo + E)
    out = ops.moe_experts(x, ids, wts, perm, bank["w13"][sl], bank["w13_sf"][sl], bank["w13_gs"][sl],
                          bank["w2"][sl], bank["w2_sf"][sl], bank["w2_gs"][sl], lo)
    cpu = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in bank.items()}
    exp = ref.experts(x.cpu(), ids.cpu(), wts.cpu(), cpu["w13"][sl], cpu["w13_sf"][sl], cpu["w13_gs"][sl],
                      cpu["w2"][sl], cpu["w2_sf"][sl], cpu["w2_gs"][sl], expert_lo=lo)
    torch.testing.assert_close(out.float().cpu(), exp.float(), rtol=2e-2, atol=2e-2)


def _r256(n):
    return (n + 255) // 256 * 256


@pytest.mark.parametrize("T,lo,E", [(1, 0, 64), (8, 0, 64), (64, 0, 64), (256, 0, 64), (8, 16, 8)])
def test_experts_post_expert_norm(ops, bank, T, lo, E):
    """Muse's post-expert RMSNorm (`_finalize`, muse_moe_w4a16/submission.py:295-308): the whole
    path against the oracle (the experts' tolerance), and the combine alone, bf16-step exact,
    against oracle.moe.finalize applied to the expert rows the kernel left in its workspace."""
    H = bank["x"].shape[1]
    I = bank["w2"].shape[2] * 2
    x = bank["x"][:T]
    ids, wts = ops.moe_route(x, bank["router"], 8)
    g = torch.Generator().manual_seed(7)
    post_norm_w = (torch.randn(H, generator=g) * 0.1).to(torch.bfloat16)
    gain = (post_norm_w.float() + 1.0).cuda()
    perm = ops.moe_permute(ids, lo, E)
    sl = slice(lo, lo + E)
    out = ops.moe_experts(x, ids, wts, perm, bank["w13"][sl], bank["w13_sf"][sl], bank["w13_gs"][sl],
                          bank["w2"][sl], bank["w2_sf"][sl], bank["w2_gs"][sl], lo, post_gain=gain)
    torch.cuda.synchronize()
    ws = ops.workspace(torch.cuda.current_device(), "moe", 0)
    off = 256 + _r256(T * 8 * H * 2) + _r256(T * 8 * I * 2)
    y = ws[off: off + T * 8 * H * 2].view(torch.bfloat16).view(T * 8, H).cpu()
    local = ((ids.cpu().long() - lo >= 0) & (ids.cpu().long() - lo < E)).reshape(-1)
    y = torch.where(local[:, None], y, torch.zeros_like(y))  # rows of other ranks' slots are stale
    fin = ref.finalize(y, ids.cpu(), wts.cpu(), gain.cpu(), lo, E)
    o, f = out.float().cpu(), fin.float()
    # one bf16 step of the result, plus an absolute 1e-5 for sums that cancel to near zero (eight
    # fp32 terms of magnitude <= ~4 summed in another order differ by up to ~2e-6)
    step = torch.exp2(torch.floor(torch.log2(torch.maximum(o.abs(), f.abs()).clamp_min(2 ** -100))) - 7)
    bad = (o - f).abs() > step + 1e-5
    assert not bool(bad.any()), (f"{int(bad.sum())} elements off, e.g. {o[bad][:4].tolist()} vs {f[bad][:4].tolist()}")
    cpu = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in bank.items()}
    exp = ref.experts(x.cpu(), ids.cpu(), wts.cpu(), cpu["w13"][sl], cpu["w13_sf"][sl], cpu["w13_gs"][sl],
                      cpu["w2"][sl], cpu["w2_sf"][sl], cpu["w2_gs"][sl], expert_lo=lo, post_gain=gain.cpu())
    torch.testing.assert_close(o, exp.float(), rtol=2e-2, atol=2e-2)
    assert (o - exp.float()).norm() / exp.float().norm() < 1e-2


def test_experts_post_norm_fp32_share(ops, bank):
    """out_fp32 with the post-norm: the unrounded share equals the bf16 output before rounding."""
    T = 8
    x = bank["x"][:T]
    ids, wts = ops.moe_route(x, bank["router"], 8)
    gain = torch.full((x.shape[1],), 1.25, device="cuda")
    perm = ops.moe_permute(ids, 0, 64)
    args = (x, ids, wts, perm, bank["w13"], bank["w13_sf"], bank["w13_gs"], bank["w2"], bank["w2_sf"],
            bank["w2_gs"], 0)
    b = ops.moe_experts(*args, post_gain=gain)
    f = ops.moe_experts(*args, post_gain=gain, out_fp32=True)
    assert torch.equal(f.to(torch.bfloat16), b)


@pytest.mark.parametrize("T,tc", [(8, "1"), (8, "0"), (16, "1"), (16, "0"), (32, "1"), (64, "0"), (256, "1")])
def test_experts_kernel_families(ops, bank, T, tc, monkeypatch):
    """The tcgen05 expert kernels (OKC_MOE_TC=1: gather + dequantise-to-shared-memory +
    tcgen05.mma) and the mma.sync kernels (0) against the same oracle, on both sides of the
    switch (16 tokens)."""
    monkeypatch.setenv("OKC_MOE_TC", tc)
    x = bank["x"][:T]
    ids, wts = ops.moe_route(x, bank["router"], 8)
    perm = ops.moe_permute(ids, 0, 64)
    out = ops.moe_experts(x, ids, wts, perm, bank["w13"], bank["w13_sf"], bank["w13_gs"],
                          bank["w2"], bank["w2_sf"], bank["w2_gs"], 0)
    assert ops.read_device_error("moe") == 0
    cpu = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in bank.items()}
    exp = ref.experts(x.cpu(), ids.cpu(), wts.cpu(), cpu["w13"], cpu["w13_sf"], cpu["w13_gs"],
                      cpu["w2"], cpu["w2_sf"], cpu["w2_gs"])
    o, e = out.float().cpu(), exp.float()
    torch.testing.assert_close(o, e, rtol=2e-2, atol=2e-2)
    assert (o - e).norm() / e.norm() < 1e-2


def test_experts_tc_activation_range(ops, bank, monkeypatch):
    """Activations far outside the f16 range go through the tcgen05 path as the same inputs
    scaled back: the per-row power-of-two scaling before each GEMM is exact, so x * 2^k gives
    the reference's outputs for x * 2^k (checked against the oracle at 2^-20 and 2^12, where a
    plain f16 conversion would flush or overflow)."""
    monkeypatch.setenv("OKC_MOE_TC", "1")
    T = 32
    cpu = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in bank.items()}
    for k in (-20, 12):
        x = (bank["x"][:T].float() * 2.0 ** k).to(torch.bfloat16)
        ids, wts = ops.moe_route(bank["x"][:T], bank["router"], 8)
        perm = ops.moe_permute(ids, 0, 64)
        out = ops.moe_experts(x, ids, wts, perm, bank["w13"], bank["w13_sf"], bank["w13_gs"], bank["w2"],
                              bank["w2_sf"], bank["w2_gs"], 0)
        assert ops.read_device_error("moe") == 0
        exp = ref.experts(x.cpu(), ids.cpu(), wts.cpu(), cpu["w13"], cpu["w13_sf"], cpu["w13_gs"],
                          cpu["w2"], cpu["w2_sf"], cpu["w2_gs"]).float()
        o = out.float().cpu()
        assert torch.isfinite(o).all()
        assert (o - exp).norm() / exp.norm() < 1e-2, f"scale 2^{k}"
