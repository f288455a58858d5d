"""Pins the CPU oracle to fixtures produced by running the reference's own code
(tests/golden/make_golden.py): the NVFP4 nibble decoder, the `_route` permutation kernel and
the prefill layer's rms / rope / route / gated decode attention."""

import json
from pathlib import Path

import pytest
import torch

from oracle import attention as oatt
from oracle import moe as omoe

GOLD = Path(__file__).resolve().parent / "golden"


def test_nvfp4_decode_matches_reference_decoder_bit_exactly():
    table = json.loads((GOLD / "nvfp4_decode.json").read_text())
    assert len(table["rows"]) == 16 * 7 * 3
    for code, sf, gs, expected in table["rows"]:
        packed = torch.tensor([[code | (code << 4)] * 8], dtype=torch.uint8)  # 16 values, one block
        sfe = torch.tensor([[sf]], dtype=torch.float32).to(torch.float8_e4m3fn)
        got = omoe.dequantize(packed, sfe, gs)[0, 0].float().item()
        assert got == expected, (code, sf, gs, got, expected)


@pytest.mark.parametrize("idx", range(6))
def test_permutation_matches_reference_route_kernel(idx):
    case = json.loads((GOLD / "route_perm.json").read_text())["cases"][idx]
    ids = torch.tensor(case["ids"], dtype=torch.int32)
    counts, offsets, pairs, tiles = omoe.permute(ids, case["local_start"], case["local_count"], case["bm"])
    assert counts.tolist() == case["count"]
    for e in range(case["local_count"]):
        assert pairs[offsets[e]:offsets[e + 1]].tolist() == case["pairs"][e]
    assert tiles.tolist() == case["tiles"]


@pytest.fixture(scope="module")
def pre():
    return torch.load(GOLD / "prefill_ops.pt", weights_only=False)


def test_rms_and_rope_bit_exact(pre):
    assert torch.equal(oatt.rms(pre["rms_in"]), pre["rms_out"])
    assert torch.equal(oatt.rope(pre["rope_in"], pre["rope_pos"], 500000.0), pre["rope_out_5e5"])
    assert torch.equal(oatt.rope(pre["rope_in"], pre["rope_pos"], 10000.0), pre["rope_out_1e4"])


def test_muse_route(pre):
    ids, w = omoe.muse_route(pre["route_h"], pre["route_w"], pre["route_bias"], 8)
    assert torch.equal(ids, pre["route_ids"])
    assert torch.equal(w, pre["route_weights"])


@pytest.mark.parametrize("i", range(6))
def test_gated_attention_and_cache_append(pre, i):
    """Cases 0-2: decode (q_len 1, full attention); 3: a sliding-window layer; 4-5: verify blocks
    of 8 tokens (full and sliding window), all against the reference's own attention()."""
    c = pre["attention_cases"][i]
    cfg = c["cfg"]
    qkv = c["x"] @ c["wqkv"].T
    kc, vc = c["k_cache_in"].clone(), c["v_cache_in"].clone()
    s = torch.tensor(c["kv_scale"])
    out = oatt.muse_attention(qkv, c["positions"], c["table"], kc, vc, s, s, cfg)
    # the append writes the same e4m3 bytes at the same rows
    assert torch.equal(kc.view(torch.uint8), c["k_cache_out"].view(torch.uint8))
    assert torch.equal(vc.view(torch.uint8), c["v_cache_out"].view(torch.uint8))
    rows = c["table"].repeat_interleave(cfg["q_len"], dim=0)
    assert torch.equal(oatt.cache_slots(rows, c["positions"], cfg["page_size"]), c["cache_loc"])
    torch.testing.assert_close(out.float(), c["out"].float(), rtol=1e-2, atol=1e-2)


@pytest.fixture(scope="module")
def mb():
    return torch.load(GOLD / "moe_boundary.pt", weights_only=False)


def _within_one_bf16_step(got, exp, frac=0.999):
    got, exp = got.float(), exp.float()
    step = torch.exp2(torch.floor(torch.log2(torch.maximum(got.abs(), exp.abs()).clamp_min(2 ** -126))) - 7)
    ok = (got - exp).abs() <= step
    assert ok.float().mean() >= frac, f"{(~ok).sum()} elements more than one bf16 step apart"
    assert bool(((got - exp).abs() <= 2 * step).all())


def test_post_expert_norm_finalize(mb):
    """oracle.moe.finalize against the reference's `_finalize`, run under Triton's CPU
    interpreter, which rounds to bf16 toward zero: with that rounding the oracle's formula gives
    the same values up to the fp32 summation order."""
    from oracle import moe as omoe
    gain = mb["fin_post_norm_w"].float() + 1.0
    out = omoe.finalize(mb["fin_y"], mb["fin_ids"], mb["fin_w"], gain, mb["fin_local_start"], mb["fin_local_count"],
                        rounding="trunc")
    _within_one_bf16_step(out, mb["fin_out"])


@pytest.mark.parametrize("name,scaled", [("attn", False), ("ffn", True)])
def test_residual_boundary(mb, name, scaled):
    """oracle.layer.residual_boundary against the reference's `_boundary` (Triton interpreter)."""
    from oracle import layer as olayer
    h, st, r = olayer.residual_boundary(mb["bnd_stream"], mb["bnd_branch"], mb["bnd_alpha"], mb["bnd_beta"],
                                        mb["bnd_post_w"] if scaled else None, mb["bnd_pre_w"], rounding="trunc")
    torch.testing.assert_close(st, mb[name + "_stream_out"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(r, mb[name + "_router"], rtol=1e-5, atol=1e-5)
    _within_one_bf16_step(h, mb[name + "_hidden"])


def test_interpreter_rounds_bf16_toward_zero():
    """The rounding the interpreter fixtures carry (checked on the fixture itself): every hidden
    value the interpreter stored is the truncation, not the nearest-even rounding, of the fp32
    value it computed (`_boundary` stores both)."""
    from oracle.numerics import bf16_round
    mb = torch.load(GOLD / "moe_boundary.pt", weights_only=False)
    r, h = mb["attn_router"], mb["attn_hidden"].float()
    assert torch.equal(bf16_round(r, "trunc"), h)
    assert not torch.equal(bf16_round(r, "rne"), h)


def test_muse_layer_oracle_matches_reference_kernel_fn():
    """The oracle's whole Muse layer (oracle/layer.py muse_decode_layer) against the reference's
    own PyTorch layer (`kernel_fn` of muse_prefill_layer/submission.py, tests/golden/
    muse_layer_ref.pt) on its first case (2 requests x 1 token, page 1), the experts the reference
    chose.  The oracle follows the decode task's rounding points (bf16 attention output before
    its per-head norm, the unrounded fp32 hidden as router input up to 8 tokens, the scaled FFN
    branch rounded to bf16: muse_decode_layer/decode/attention.py:114-117, runtime.py:56-58,
    boundaries.py:24-26), which that `kernel_fn` does not round: relative L2 ~4e-3, one bf16 step."""
    from okc_b200 import synth
    from oracle import layer as olayer
    fx = torch.load(GOLD / "muse_layer_ref.pt", weights_only=False)
    c = fx["cases"][0]
    w, _ = synth.muse_layer_case(B=1, ctx=(4, 8), seed=fx["weights_seed"], device="cpu")
    _, d = synth.muse_layer_case(B=c["B"], L=c["L"], ctx=tuple(c["ctx"]), page=c["page"], window=c["window"],
                                 seed=c["seed"], device="cpu", weights=w)
    assert torch.equal(c["rows"], torch.arange(c["B"] * c["L"]))
    h, st, _, _ = olayer.muse_decode_layer(d, w, ids_in=c["ids"])
    for got, exp, what in ((h, c["hidden"], "hidden"), (st, c["stream"], "stream")):
        torch.testing.assert_close(got.float(), exp.float(), rtol=2e-2, atol=8e-2, msg=what)
        assert float((got.float() - exp.float()).norm() / exp.float().norm()) < 1e-2, what
