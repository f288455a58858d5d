"""Generates the golden fixtures of tests/golden/ by running the reference's OWN code here.

Needs a checkout of the reference, named by $OKC_REFERENCE, and runs on CPU:

  nvfp4_decode.json  the NVFP4 nibble decoder `_decode_nvfp4` of
                     muse_decode_layer/decode/nvfp4_gemv.py:9-18, executed with scalar fp32/bf16
                     semantics over all 16 E2M1 codes x 7 block scales x 3 global scales (the
                     grid of muse_decode_layer/tests/test_nvfp4_gemv.py:56-69).
  route_perm.json    the Triton `_route` kernel of muse_moe_w4a16/submission.py:274-291 run under
                     Triton's CPU interpreter: per-expert pair lists, counts and tile tables.
  prefill_ops.pt     `rms`, `rope`, `route` and the gated decode `attention` (q_len 1 and 8,
                     full and sliding-window layers) of
                     muse_prefill_layer/submission.py (its `nvfp4` import is stubbed: the
                     attention path never calls it), on small seeded inputs.
  moe_boundary.pt    the Triton `_finalize` (post-expert RMSNorm + routing-weighted sum) of
                     muse_moe_w4a16/submission.py:295-308 and `_boundary` (gated residual
                     stream + next RMSNorm) of muse_decode_layer/decode/boundaries.py:17-37, both
                     under Triton's CPU interpreter.  That interpreter rounds fp32 -> bf16 toward
                     zero (the GPU rounds to nearest even), so the tests pin the oracle's formula
                     against these with its rounding set to "trunc".
  muse_layer_ref.pt  the whole layer, `kernel_fn` of muse_prefill_layer/submission.py:201-218, on
                     four seeded cases (q_len 1, 8 and a 200-token prefill block, page 1 and
                     64, full and window 2048; the prefill block's every 25th token stored)
                     whose inputs synth.muse_layer_case regenerates from the stored seeds; its
                     `nvfp4` import is stubbed with oracle.moe.dequantize (pinned to the
                     reference's `_decode_nvfp4` by nvfp4_decode.json).

    python tests/golden/make_golden.py              # every fixture
    python tests/golden/make_golden.py muse_layer   # muse_layer_ref.pt only
"""

from __future__ import annotations

import ast
import importlib.util
import json
import os
import struct
import subprocess
import sys
import types
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("OKC_REFERENCE", "reference-checkout-not-set"))


# ------------------------------------------------------------------------ NVFP4 decode
def _f32(x):
    return struct.unpack("f", struct.pack("f", x))[0]


def _bf16(x):
    bits = struct.unpack("I", struct.pack("f", x))[0]
    bits = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
    return struct.unpack("f", struct.pack("I", bits))[0]


class _Scalar:
    """Scalar stand-in for a Triton tensor with fp32 / bf16 / uint32 semantics, enough to
    execute the reference decoder line by line."""

    def __init__(self, v, kind="fp32"):
        self.kind = kind
        self.v = _f32(v) if kind == "fp32" else v

    def to(self, kind, bitcast=False):
        if bitcast:
            return _Scalar(struct.unpack("f", struct.pack("I", int(self.v) & 0xFFFFFFFF))[0])
        if kind == "bf16":
            return _Scalar(_bf16(self.v), "bf16")
        if kind == "fp32":
            return _Scalar(float(self.v))
        return _Scalar(self.v, kind)

    def _bin(self, o, f):
        ov = o.v if isinstance(o, _Scalar) else o
        kind = self.kind
        r = f(self.v, ov)
        return _Scalar(r, kind) if kind != "fp32" else _Scalar(_f32(r))

    def __and__(self, o): return self._bin(o, lambda a, b: int(a) & int(b))
    def __or__(self, o): return self._bin(o, lambda a, b: int(a) | int(b))
    def __rshift__(self, o): return self._bin(o, lambda a, b: int(a) >> int(b))
    def __lshift__(self, o): return self._bin(o, lambda a, b: (int(a) << int(b)) & 0xFFFFFFFF)
    def __add__(self, o): return self._bin(o, lambda a, b: a + b)
    def __mul__(self, o): return self._bin(o, lambda a, b: a * b)
    def __rmul__(self, o): return self.__mul__(o)
    def __neg__(self): return _Scalar(-self.v, self.kind)
    def __lt__(self, o): return self.v < (o.v if isinstance(o, _Scalar) else o)
    def __ne__(self, o): return self.v != (o.v if isinstance(o, _Scalar) else o)


def nvfp4_decode_table():
    src = (REF / "muse_decode_layer/decode/nvfp4_gemv.py").read_text()
    fn = next(n for n in ast.parse(src).body if isinstance(n, ast.FunctionDef) and n.name == "_decode_nvfp4")
    fn.decorator_list = []
    ns = {"tl": types.SimpleNamespace(uint32="uint32", float32="fp32", bfloat16="bf16",
                                      where=lambda c, a, b: a if (c.v if isinstance(c, _Scalar) else c) else b)}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), "<reference _decode_nvfp4>", "exec"), ns)
    dec = ns["_decode_nvfp4"]
    scales = (0.015625, 0.125, 0.5, 1.0, 8.0, 128.0, 448.0)
    globals_ = (1e-5, 0.00314159, 0.1)
    rows = []
    for code in range(16):
        for sf in scales:
            for gs in globals_:
                v = dec(_Scalar(code, "uint32"), _Scalar(sf), _Scalar(gs)).v
                rows.append([code, sf, gs, v])
    return {"source": "muse_decode_layer/decode/nvfp4_gemv.py:9-18", "rows": rows}


# ------------------------------------------------------------------------- _route
ROUTE_SNIPPET = r'''
import importlib.util, json, sys, torch, triton
spec = importlib.util.spec_from_file_location("moe_ref", sys.argv[1])
m = importlib.util.module_from_spec(spec); spec.loader.exec_module(m)
cases = []
for M, seed, bm in [(1, 0, 8), (5, 1, 8), (8, 2, 8), (16, 3, 16), (33, 4, 16), (64, 5, 8)]:
    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(64, generator=g)[:8] for _ in range(M)]).to(torch.int32)
    max_tiles = min(32, M * 8) + triton.cdiv(M * 8, bm)
    count = torch.zeros(32, dtype=torch.int32)
    pairs = torch.full((32, M), -1, dtype=torch.int32)
    tiles = torch.full((1 + max_tiles,), -1, dtype=torch.int32)
    m._route[(1,)](ids, count, pairs, tiles, M, 0, P=triton.next_power_of_2(M * 8), BM=bm,
                   MT=triton.next_power_of_2(triton.cdiv(M, bm)), num_warps=4)
    n = int(tiles[0])
    cases.append({"M": M, "bm": bm, "local_start": 0, "local_count": 32, "ids": ids.tolist(),
                  "count": count.tolist(),
                  "pairs": [pairs[e, :int(count[e])].tolist() for e in range(32)],
                  "tiles": tiles[:n + 1].tolist()})
print(json.dumps(cases))
'''


# ------------------------------------------------------------- _finalize, _boundary
FINALIZE_BOUNDARY_SNIPPET = r'''
import importlib.util, sys, torch
spec = importlib.util.spec_from_file_location("moe_ref", sys.argv[1])
m = importlib.util.module_from_spec(spec); spec.loader.exec_module(m)
spec = importlib.util.spec_from_file_location("bnd_ref", sys.argv[2])
bnd = importlib.util.module_from_spec(spec); spec.loader.exec_module(bnd)
out = {"source": "muse_moe_w4a16/submission.py:295-308 (_finalize), "
                 "muse_decode_layer/decode/boundaries.py:17-37 (_boundary), Triton interpreter"}
g = torch.Generator().manual_seed(7)
# post-expert RMSNorm + routing-weighted sum: 3 tokens, top-8, hidden 4096, local experts [8, 40)
M = 3
y = (torch.randn((M * 8, 4096), generator=g) * 3).to(torch.bfloat16)
ids = torch.randint(0, 64, (M, 8), generator=g).to(torch.int32)
w = torch.rand((M, 8), generator=g)
post_norm_w = (torch.randn(4096, generator=g) * 0.1).to(torch.bfloat16)
norm_w = post_norm_w.float() + 1.0
fin = torch.empty((M, 4096), dtype=torch.bfloat16)
m._finalize[(M,)](y, w, ids, norm_w, fin, 8, 32, num_warps=8)
out.update(fin_y=y, fin_ids=ids, fin_w=w, fin_post_norm_w=post_norm_w, fin_local_start=8, fin_local_count=32,
           fin_out=fin)
# gated residual boundaries: attention (unscaled branch) and FFN (branch * (1 + post_ffn_norm))
T = 3
stream = torch.randn((T, 8192), generator=g) * 2
branch = (torch.randn((T, 8192), generator=g) * 0.5).to(torch.bfloat16)
gate = torch.randn(8192, generator=g)
beta = torch.sigmoid(gate / 0.3)
alpha = torch.sqrt(torch.clamp(torch.sigmoid(-gate / 0.3) * (1. + beta), min=1e-3))
post_w = (torch.randn(8192, generator=g) * 0.1).to(torch.bfloat16)
pre_w = (torch.randn(8192, generator=g) * 0.1).to(torch.bfloat16)
for name, scaled in (("attn", False), ("ffn", True)):
    hidden = torch.empty((T, 8192), dtype=torch.bfloat16)
    s_out = torch.empty((T, 8192), dtype=torch.float32)
    router = torch.empty((T, 8192), dtype=torch.float32)
    bnd._boundary[(T,)](stream, branch, alpha, beta, post_w, pre_w, hidden, s_out, router, 8192, scaled, True,
                        num_warps=8)
    out[name + "_hidden"], out[name + "_stream_out"], out[name + "_router"] = hidden, s_out, router
out.update(bnd_stream=stream, bnd_branch=branch, bnd_alpha=alpha, bnd_beta=beta, bnd_gate=gate,
           bnd_post_w=post_w, bnd_pre_w=pre_w)
torch.save(out, sys.argv[3])
'''


def finalize_boundary(path):
    env = dict(os.environ, TRITON_INTERPRET="1")
    subprocess.run([sys.executable, "-c", FINALIZE_BOUNDARY_SNIPPET, str(REF / "muse_moe_w4a16/submission.py"),
                    str(REF / "muse_decode_layer/decode/boundaries.py"), str(path)], env=env, check=True)


def route_cases():
    env = dict(os.environ, TRITON_INTERPRET="1")
    out = subprocess.run([sys.executable, "-c", ROUTE_SNIPPET, str(REF / "muse_moe_w4a16/submission.py")],
                         env=env, capture_output=True, text=True, check=True)
    return {"source": "muse_moe_w4a16/submission.py:274-291 (_route, Triton interpreter)",
            "cases": json.loads(out.stdout.strip().splitlines()[-1])}


# ------------------------------------------------------------------ prefill functions
def prefill_ops():
    import torch
    sys.modules.setdefault("nvfp4", types.SimpleNamespace(dequantize=None))
    spec = importlib.util.spec_from_file_location("prefill_ref", REF / "muse_prefill_layer/submission.py")
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    g = torch.Generator().manual_seed(1234)
    out = {"source": "muse_prefill_layer/submission.py"}
    x = torch.randn((6, 4, 64), generator=g) * 3
    pos = torch.tensor([0, 1, 7, 100, 4095, 70000])
    out["rms_in"], out["rms_out"] = x, ref.rms(x)
    out["rope_in"], out["rope_pos"] = x, pos
    out["rope_out_5e5"] = ref.rope(x, pos, 500000.0)
    out["rope_out_1e4"] = ref.rope(x, pos, 10000.0)
    # Muse routing: sigmoid scores, bias to choose, renormalised weights
    h = torch.randn((5, 128), generator=g).to(torch.bfloat16)
    router = torch.randn((32, 128), generator=g) * 0.05
    bias = torch.randn((32,), generator=g) * 0.1
    ids, w = ref.route(h, {"router": router, "router_bias": bias}, 8)
    out.update(route_h=h, route_w=router, route_bias=bias, route_ids=ids, route_weights=w)
    # gated decode attention (q_len 1) over a paged FP8 cache, two page sizes / two scales
    cases = []
    for page, kv_scale, theta, seed in [(16, 1.0, 500000.0, 1), (1, 1 / 64, 0.0, 2), (4, 0.5, 10000.0, 3)]:
        gg = torch.Generator().manual_seed(seed)
        B, hq, hkv, d, hidden = 3, 16, 2, 64, 64
        lens = torch.tensor([5, 37, 60])
        max_pages = (int(lens.max()) + 1 + page - 1) // page
        pages = B * max_pages
        perm = torch.randperm(pages, generator=gg).to(torch.int32)
        table = perm.view(B, max_pages).clone()
        kc = (torch.randn((pages, page, hkv, d), generator=gg) / kv_scale).to(torch.float8_e4m3fn)
        vc = (torch.randn((pages, page, hkv, d), generator=gg) / kv_scale).to(torch.float8_e4m3fn)
        x_in = torch.randn((B, hidden), generator=gg).to(torch.bfloat16)
        wqkv = (torch.randn(((2 * hq + 2 * hkv) * d, hidden), generator=gg) * 0.05).to(torch.bfloat16)
        positions = lens.long()
        cache_loc = table.long()[torch.arange(B), positions // page] * page + positions % page
        cfg = {"batch": B, "q_len": 1, "num_q_heads": hq, "num_kv_heads": hkv, "head_dim": d,
               "page_size": page, "window": 0, "rope_theta": theta, "qk_scale_factor": 5.4730064863875,
               "sm_scale": 0.125}
        kc0, vc0 = kc.clone(), vc.clone()
        data = {"config": cfg, "positions": positions, "page_table": table, "cache_loc": cache_loc,
                "k_cache": kc, "v_cache": vc, "k_scale": torch.tensor(kv_scale), "v_scale": torch.tensor(kv_scale)}
        o = ref.attention(data, x_in, {"qkv_gate": wqkv})
        cases.append({"cfg": cfg, "x": x_in, "wqkv": wqkv, "table": table, "positions": positions,
                      "cache_loc": cache_loc, "k_cache_in": kc0, "v_cache_in": vc0, "k_cache_out": kc,
                      "v_cache_out": vc, "kv_scale": kv_scale, "out": o})
    # sliding-window layers and speculative-verify blocks (q_len 8: every block token attends the
    # cache and the block up to its own position), with the reference's own attention()
    for page, kv_scale, theta, window, L, seed in [(16, 1.0, 500000.0, 16, 1, 4), (4, 0.5, 10000.0, 0, 8, 5),
                                                    (1, 1 / 64, 500000.0, 20, 8, 6)]:
        gg = torch.Generator().manual_seed(seed)
        B, hq, hkv, d, hidden = 3, 16, 2, 64, 64
        seq = torch.tensor([5, 37, 60])
        max_pages = (int(seq.max()) + L + page - 1) // page
        pages = B * max_pages
        perm = torch.randperm(pages, generator=gg).to(torch.int32)
        table = perm.view(B, max_pages).clone()
        kc = (torch.randn((pages, page, hkv, d), generator=gg) / kv_scale).to(torch.float8_e4m3fn)
        vc = (torch.randn((pages, page, hkv, d), generator=gg) / kv_scale).to(torch.float8_e4m3fn)
        x_in = torch.randn((B * L, hidden), generator=gg).to(torch.bfloat16)
        wqkv = (torch.randn(((2 * hq + 2 * hkv) * d, hidden), generator=gg) * 0.05).to(torch.bfloat16)
        positions = (seq[:, None] + torch.arange(L)).reshape(-1).long()
        rows = torch.arange(B).repeat_interleave(L)
        cache_loc = table.long()[rows, positions // page] * page + positions % page
        cfg = {"batch": B, "q_len": L, "num_q_heads": hq, "num_kv_heads": hkv, "head_dim": d,
               "page_size": page, "window": window, "rope_theta": theta, "qk_scale_factor": 5.4730064863875,
               "sm_scale": 0.125}
        kc0, vc0 = kc.clone(), vc.clone()
        data = {"config": cfg, "positions": positions, "page_table": table, "cache_loc": cache_loc,
                "k_cache": kc, "v_cache": vc, "k_scale": torch.tensor(kv_scale), "v_scale": torch.tensor(kv_scale)}
        o = ref.attention(data, x_in, {"qkv_gate": wqkv})
        cases.append({"cfg": cfg, "x": x_in, "wqkv": wqkv, "table": table, "positions": positions,
                      "seq_lens": seq.to(torch.int32), "cache_loc": cache_loc, "k_cache_in": kc0,
                      "v_cache_in": vc0, "k_cache_out": kc, "v_cache_out": vc, "kv_scale": kv_scale, "out": o})
    out["attention_cases"] = cases
    return out


# ------------------------------------------------------------- whole Muse layer (kernel_fn)
MUSE_LAYER_CASES = [  # (B, q_len, ctx, page, window, data seed, stored row stride); weights seed 500
    (2, 1, (300, 600), 1, 0, 501, 1),
    (1, 8, (200, 400), 1, 2048, 502, 1),
    (3, 1, (100, 300), 64, 0, 503, 1),
    (1, 200, (100, 200), 1, 0, 504, 25),  # a prefill block: every 25th token's rows stored
]


def muse_layer_reference():
    """The reference's own PyTorch layer, muse_prefill_layer/submission.py:201-218 `kernel_fn`
    (the layer the decode and prefill tasks share), on CPU inputs that synth.muse_layer_case
    regenerates bit for bit from their seeds (1.1 GB of weights are not stored).  Its `nvfp4`
    import (a module of the challenge harness, not in the checkout) is stubbed with
    oracle.moe.dequantize, which tests/test_oracle_golden.py pins bit-exact to the reference's own
    `_decode_nvfp4`.  Stored per case: hidden, stream, ids and the routing scores + bias the
    reference chose from (its `route` wrapped to record its input)."""
    import torch
    sys.path.insert(0, str(HERE.parent.parent))
    from oracle.moe import dequantize
    from okc_b200 import synth
    sys.modules["nvfp4"] = types.SimpleNamespace(dequantize=dequantize)
    spec = importlib.util.spec_from_file_location("prefill_layer_ref", REF / "muse_prefill_layer/submission.py")
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    seen = {}
    route = ref.route

    def recording_route(h, weights, top_k):
        seen["h"] = h
        return route(h, weights, top_k)
    ref.route = recording_route
    w, _ = synth.muse_layer_case(B=1, ctx=(4, 8), seed=500, device="cpu")
    out = {"source": "muse_prefill_layer/submission.py:201-218 (kernel_fn), CPU", "weights_seed": 500, "cases": []}
    for B, L, ctx, page, window, seed, stride in MUSE_LAYER_CASES:
        _, d = synth.muse_layer_case(B=B, L=L, ctx=ctx, page=page, window=window, seed=seed, device="cpu",
                                     weights=w)
        hidden, stream, ids = ref.kernel_fn(d, w)
        scores = torch.sigmoid((seen["h"].float() @ w["router"].T) * 0.1767766952966369) + w["router_bias"]
        rows = torch.arange(0, B * L, stride)
        out["cases"].append({"B": B, "L": L, "ctx": ctx, "page": page, "window": window, "seed": seed,
                             "rows": rows, "hidden": hidden[rows].clone(), "stream": stream[rows].clone(),
                             "ids": ids[rows].clone(), "scores": scores[rows].clone()})
    return out


def main():
    if not REF.exists():
        raise SystemExit(f"reference checkout not found at {REF}")
    (HERE / "nvfp4_decode.json").write_text(json.dumps(nvfp4_decode_table()))
    (HERE / "route_perm.json").write_text(json.dumps(route_cases()))
    import torch
    torch.save(prefill_ops(), HERE / "prefill_ops.pt")
    finalize_boundary(HERE / "moe_boundary.pt")
    torch.save(muse_layer_reference(), HERE / "muse_layer_ref.pt")
    print("wrote", *(p.name for p in sorted(HERE.glob("*")) if p.suffix in (".json", ".pt")))


if __name__ == "__main__":
    if sys.argv[1:] == ["muse_layer"]:  # only the whole-layer fixture (the others unchanged)
        import torch
        torch.save(muse_layer_reference(), HERE / "muse_layer_ref.pt")
    else:
        main()
