"""The no-alloc attention entry point, for callers that are not allowed to allocate device
memory (a plugin that may only enqueue work on a stream it is given, or a process whose device
footprint must not grow after start-up).  It keeps its split-KV partials in a fixed array
inside the library instead of a caller-provided workspace.

Checks, through the C ABI, that two calls in a row give the same output as the workspace
entry point okc_attn_decode_fp8 on the same inputs (same tolerance as the attention parity
tests: rtol 2e-2 / atol 2e-2), and that an oversized request is refused.  The file is named
to be collected last, so a run that stops at the first failure has run every other test."""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(seed, lens, B, Hq, Hkv, D, page):
    from okc_b200 import synth
    g = torch.Generator(device="cuda").manual_seed(seed)
    pool = sum(math.ceil(n / page) for n in lens) + 5
    table = synth.paged_layout(lens, page, pool, g, "cuda")
    kc = torch.empty((pool, page, Hkv, D), dtype=torch.float8_e4m3fn, device="cuda")
    vc = torch.empty_like(kc)
    synth.fill_e4m3_normal(kc, g)
    synth.fill_e4m3_normal(vc, g)
    q = torch.randn((B, Hq, D), generator=g, device="cuda").to(torch.bfloat16)
    ks = (torch.rand(Hkv, generator=g, device="cuda") + 0.5).float()
    vs = (torch.rand(Hkv, generator=g, device="cuda") + 0.5).float()
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return q, kc, vc, table, sl, ks, vs


def _args(q, kc, vc, table, sl, ks, vs, out, num_ctas):
    B, Hq, D = q.shape
    pool, page, Hkv, _ = kc.shape
    return [q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), table.data_ptr(), table.stride(0),
            sl.data_ptr(), ks.data_ptr(), vs.data_ptr(), out.data_ptr(), out.stride(0), B, Hq, Hkv, D, page,
            pool, ctypes.c_float(1 / math.sqrt(D)), num_ctas]


def test_noalloc_matches_workspace_entry_point_twice():
    from okc_b200 import _lib
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    cases = [(1, [37, 200, 1, 1000, 64], 64, 8, 128, 16), (2, [3000, 17, 512], 16, 2, 64, 1)]
    for seed, lens, Hq, Hkv, D, page in cases:  # two calls in a row, different shapes
        q, kc, vc, table, sl, ks, vs = _inputs(seed, lens, len(lens), Hq, Hkv, D, page)
        ref = torch.empty_like(q)
        ws_bytes = lib.okc_attn_decode_workspace_bytes(len(lens), Hq, Hkv, D, 0)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
        st = lib.okc_attn_decode_fp8(*_args(q, kc, vc, table, sl, ks, vs, ref, 0), ws.data_ptr(), ws_bytes, stream)
        assert st == _lib.OKC_OK
        out = torch.full_like(q, float("nan"))
        st = lib.okc_attn_decode_fp8_noalloc(*_args(q, kc, vc, table, sl, ks, vs, out, 0), stream)
        assert st == _lib.OKC_OK
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_noalloc_rejects_requests_beyond_its_scratch():
    from okc_b200 import _lib
    lib = _lib.load()
    q, kc, vc, table, sl, ks, vs = _inputs(3, [16] * 8, 8, 8, 1, 128, 16)
    out = torch.empty_like(q)
    # 4096 CTAs x 8 sub-tiles x 8 heads of (128 + 2) floats is far beyond 16 MiB
    st = lib.okc_attn_decode_fp8_noalloc(*_args(q, kc, vc, table, sl, ks, vs, out, 4096),
                                         torch.cuda.current_stream().cuda_stream)
    assert st == _lib.OKC_ERR_TOO_LARGE
