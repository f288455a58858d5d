"""GPU parity of the Muse decode-layer drop-in (okc_b200/problems/muse_decode_layer.py) against
the CPU oracle's composition of the same layer (oracle/layer.py muse_decode_layer), on the
reference problem's shapes and data formats: 16 q / 2 kv heads of 64, page 1 and 64, full and
sliding-window (2048) layers, decode steps and verify blocks of 8, kv_scale 1 and 1/64, 1 to 40
tokens (both router paths: the fp32 router input up to 8 tokens, bf16 hi/lo beyond; both
expert kernel families), and prefill blocks of 144-2100 tokens per request (the same layer as
muse_prefill_layer: projections in 256-row blocks, the append per request, experts in 2048-token
passes).

Routing: every expert the device chose must score within 1e-3 of the oracle's 8th biased score,
and every oracle choice more than 1e-3 above its 9th score must be among the device's.  The
oracle routes from its own hidden state, which differs from the device's by bf16
steps in scattered elements (the attention/O/boundary chain above it); that moves a score by up to
~1e-4, so over thousands of tokens closer choices may legitimately differ.  The oracle then
evaluates the experts the device chose (weights from its own scores).  Tolerance on hidden (bf16) and stream (fp32): relative L2 < 1e-2 (measured ~4.4e-3, about one
bf16 step, at every case) and elementwise rtol 2e-2 / atol 8e-2.  The elementwise bound is wider
than a single operator's because the steps chain: each stage agrees with the oracle to a bf16
step given the same input, but the expert outputs (three bf16 roundings deep, summation order
differing between the device and the CPU) differ by ~5e-3 relative, and the FFN boundary
normalises a branch of 1024 nonzero columns over 8192 (up to 8 tokens), which scales that
difference ~2.8x into the stream and the next hidden.  The written cache rows within one e4m3
step (2^-3 of the value, 2^-9 / kv_scale near zero); k rows also within 1.6e-2 / kv_scale
absolute (a rotated small value is the difference of two O(1) products of the projected qkv,
whose bf16 rounding may differ by a step)."""

from pathlib import Path

import pytest
import torch

from oracle import layer as olayer

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"

CASES = [  # B, L, ctx, page, window, kv_scale
    (1, 1, (1000, 3000), 1, 2048, 1.0),
    (1, 1, (2000, 3000), 1, 0, 1.0),
    (1, 8, (3000, 6000), 64, 0, 1.0),
    (4, 1, (500, 7000), 1, 2048, 1 / 64),
    (2, 8, (2000, 5000), 1, 2048, 1.0),
    (33, 1, (1000, 4000), 1, 0, 1.0),
    (5, 8, (1000, 5000), 1, 2048, 1.0),
    # prefill blocks (muse_prefill_layer): a long block under one projection block; 256 + 32 token
    # projection blocks (the tail on the skinny kernel); 9 projection blocks and 2 expert passes
    (1, 200, (300, 600), 1, 0, 1.0),
    (2, 144, (50, 400), 64, 2048, 1.0),
    (1, 2100, (100, 200), 1, 2048, 1.0),
]


@pytest.fixture(scope="module")
def bank():
    from okc_b200 import synth
    from okc_b200.problems import muse_decode_layer as prob
    w, _ = synth.muse_layer_case(B=1, ctx=(4, 8), seed=11, device="cuda")
    return w, {k: v.cpu() for k, v in w.items()}, prob.prepare(w)


def _close(out, exp, what):
    o, e = out.float().cpu(), exp.float().cpu()
    d = (o - e).abs()
    rel = float((o - e).norm() / e.norm().clamp_min(1e-30))
    i = int(d.argmax())
    info = f"{what}: relL2 {rel:.2e} max|d| {float(d.max()):.3e} at {i} (got {float(o.view(-1)[i]):.4f}, " \
           f"exp {float(e.view(-1)[i]):.4f})"
    print(info)
    torch.testing.assert_close(o, e, rtol=2e-2, atol=8e-2, msg=info)
    assert rel < 1e-2, info


@pytest.mark.parametrize("B,L,ctx,page,window,kv_scale", CASES)
def test_muse_decode_layer(bank, B, L, ctx, page, window, kv_scale):
    from okc_b200 import synth
    from okc_b200.problems import muse_decode_layer as prob
    w_gpu, w_cpu, state = bank
    _, data = synth.muse_layer_case(B=B, L=L, ctx=ctx, page=page, window=window, kv_scale=kv_scale,
                                    seed=100 + B * 10 + L, device="cuda", weights=w_gpu)
    cpu = {k: (v.cpu().clone() if torch.is_tensor(v) else v) for k, v in data.items()}
    hidden, stream, ids = prob.kernel_fn(data, state)
    torch.cuda.synchronize()
    T = B * L
    assert hidden.shape == (T, 8192) and hidden.dtype == torch.bfloat16
    assert stream.shape == (T, 8192) and stream.dtype == torch.float32
    assert ids.shape == (T, 8) and ids.dtype == torch.int32
    exp_h, exp_s, _, scores = olayer.muse_decode_layer(cpu, w_cpu, ids_in=ids.cpu())
    # routing against the oracle's own scores: every device choice is within TIE of the oracle's
    # 8th score, and every oracle choice clearly above its 9th score is a device choice
    TIE = 1e-3
    top = torch.sort(scores, dim=-1, descending=True, stable=True)
    s8, s9 = top.values[:, 7:8], top.values[:, 8:9]
    got = ids.cpu().long()
    assert (scores.gather(1, got) >= s8 - TIE).all(), "a device choice scores well below the oracle's top 8"
    clear = top.values[:, :8] > s9 + TIE
    chosen = (top.indices[:, :8, None] == got[:, None, :]).any(-1)
    assert chosen[clear].all(), "an oracle choice clear of the 9th score was not chosen"
    assert clear.float().mean() > 0.5, "too many near-ties to check the routing"
    what = f"B{B} L{L} P{page} window{window} s{kv_scale}"
    _close(hidden, exp_h, what + " hidden")
    _close(stream, exp_s, what + " stream")
    rows = data["cache_loc"].cpu()
    for name in ("k_cache", "v_cache"):
        g = data[name].cpu().view(-1, 2, 64)[rows].float()
        e = cpu[name].view(-1, 2, 64)[rows].float()
        d = (g - e).abs()
        # one e4m3 step; for k also the absolute error a rotation passes on when the two products
        # it subtracts are O(1) and the projected qkv differs by a bf16 step (2^-7 per input)
        atol = (1.6e-2 if name == "k_cache" else 2e-3) / kv_scale
        bad = d > 0.13 * e.abs() + atol
        idx = torch.nonzero(bad)[:4].tolist()
        assert not bad.any(), f"{what} {name}: {int(bad.sum())} of {bad.numel()} values beyond one e4m3 step, " \
            f"e.g. {[(i, float(g[tuple(i)]), float(e[tuple(i)])) for i in idx]}"



@pytest.mark.parametrize("i", range(4))
def test_muse_layer_matches_reference_kernel_fn(i):
    """The device layer against the reference's own PyTorch layer (`kernel_fn` of
    muse_prefill_layer/submission.py, tests/golden/muse_layer_ref.pt: 2 x 1 tokens page 1,
    1 x 8 window 2048, 3 x 1 page 64, a 200-token prefill block (its stored rows)) on inputs
    regenerated from the fixture's seeds.  Routing
    against the reference's own scores (the tie-tolerant rule above); hidden and stream within the
    layer tolerance (relative L2 < 1e-2: the decode task's extra bf16 rounding points, which
    that `kernel_fn` skips, plus the device/CPU summation order)."""
    from okc_b200 import synth
    from okc_b200.problems import muse_decode_layer as prob
    fx = torch.load(GOLD / "muse_layer_ref.pt", weights_only=False)
    c = fx["cases"][i]
    w, _ = synth.muse_layer_case(B=1, ctx=(4, 8), seed=fx["weights_seed"], device="cpu")
    _, d = synth.muse_layer_case(B=c["B"], L=c["L"], ctx=tuple(c["ctx"]), page=c["page"], window=c["window"],
                                 seed=c["seed"], device="cpu", weights=w)
    state = prob.prepare({k: v.cuda() for k, v in w.items()})
    data = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in d.items()}
    hidden, stream, ids = prob.kernel_fn(data, state)
    torch.cuda.synchronize()
    rows = c["rows"]
    hidden, stream, ids = hidden.cpu()[rows], stream.cpu()[rows], ids.cpu()[rows]
    TIE = 1e-3
    scores = c["scores"]
    top = torch.sort(scores, dim=-1, descending=True, stable=True)
    s8, s9 = top.values[:, 7:8], top.values[:, 8:9]
    got = ids.cpu().long()
    assert (scores.gather(1, got) >= s8 - TIE).all(), "a device choice scores well below the reference's top 8"
    clear = top.values[:, :8] > s9 + TIE
    chosen = (top.indices[:, :8, None] == got[:, None, :]).any(-1)
    assert chosen[clear].all(), "a reference choice clear of the 9th score was not chosen"
    # rows whose expert set equals the reference's (a near-tie may legitimately pick another one)
    same = (torch.sort(got, -1).values == torch.sort(c["ids"].long(), -1).values).all(-1)
    assert same.float().mean() >= 0.5, "too few tokens with the reference's expert set"
    _close(hidden[same], c["hidden"][same], f"reference case {i} hidden")
    _close(stream[same], c["stream"][same], f"reference case {i} stream")
