"""The no-alloc attention entry point, for callers that are not allowed to allocate device
memory (a plugin that may only enqueue work on a stream it is given, or a process whose device
footprint must not grow after start-up).  It keeps its split-KV partials in a fixed array
inside the library instead of a caller-provided workspace.

Checks, through the C ABI:
  * two calls in a row (different shapes) give the same bits as the workspace entry point
    okc_attn_decode_fp8 on the same inputs (same kernel, same CTA count: bit-identical), and
    both match the CPU oracle within the attention tolerance (rtol 2e-2 / atol 2e-2);
  * a page id outside the pool is skipped, not read: the call succeeds, the error word reports
    OKC_DEVERR_PAGE through okc_attn_decode_fp8_noalloc_error (which also clears it), the
    other sequences are unchanged and the context stays usable;
  * an oversized request is refused.
The file is named to be collected last, so a run that stops at the first failure has run every
other test."""

import ctypes
import math

import pytest
import torch

from oracle import attention as oatt

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


def _workspace_call(lib, ins, out, stream):
    q = ins[0]
    B, Hq, D = q.shape
    Hkv = ins[1].shape[2]
    ws_bytes = lib.okc_attn_decode_workspace_bytes(B, Hq, Hkv, D, 0)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    return lib.okc_attn_decode_fp8(*_args(*ins, out, 0), ws.data_ptr(), ws_bytes, stream)


def test_noalloc_matches_workspace_entry_point_twice():
    from okc_b200 import _lib
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    cases = [(1, [37, 200, 1, 1000, 64], 64, 8, 128, 16), (2, [3000, 17, 512], 16, 2, 64, 1)]
    for seed, lens, Hq, Hkv, D, page in cases:  # two calls in a row, different shapes
        ins = _inputs(seed, lens, len(lens), Hq, Hkv, D, page)
        q = ins[0]
        ref = torch.empty_like(q)
        assert _workspace_call(lib, ins, ref, stream) == _lib.OKC_OK
        out = torch.full_like(q, float("nan"))
        st = lib.okc_attn_decode_fp8_noalloc(*_args(*ins, out, 0), stream)
        assert st == _lib.OKC_OK
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), "same kernel, same CTAs: same bits"
        assert lib.okc_attn_decode_fp8_noalloc_error(stream) == 0
        cpu = [t.cpu() for t in ins]
        exp = oatt.decode(*cpu, 1 / math.sqrt(D))
        torch.testing.assert_close(out.float().cpu(), exp.float(), rtol=2e-2, atol=2e-2)


def test_noalloc_bad_page_id_is_reported_not_read():
    from okc_b200 import _lib
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    lens = [300, 129, 700]
    ins = _inputs(5, lens, 3, 16, 2, 128, 16)
    q, kc, vc, table, sl, ks, vs = ins
    ref = torch.empty_like(q)
    assert _workspace_call(lib, ins, ref, stream) == _lib.OKC_OK
    bad = table.clone()
    bad[1, 3] = kc.shape[0] + 1000  # sequence 1, page 3: outside the pool
    out = torch.empty_like(q)
    st = lib.okc_attn_decode_fp8_noalloc(*_args(q, kc, vc, bad, sl, ks, vs, out, 0), stream)
    assert st == _lib.OKC_OK
    err = lib.okc_attn_decode_fp8_noalloc_error(stream)
    assert err & _lib.DEVERR_PAGE, f"error word {err}"
    assert lib.okc_attn_decode_fp8_noalloc_error(stream) == 0, "the accessor clears the word"
    for b in (0, 2):  # the sequences with valid tables are unaffected
        assert torch.equal(out[b].view(torch.int16), ref[b].view(torch.int16))
    # the context is still usable: a clean call afterwards matches again and reports nothing
    st = lib.okc_attn_decode_fp8_noalloc(*_args(*ins, out, 0), stream)
    assert st == _lib.OKC_OK
    assert lib.okc_attn_decode_fp8_noalloc_error(stream) == 0
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_noalloc_rejects_requests_beyond_its_scratch():
    from okc_b200 import _lib
    lib = _lib.load()
    q, kc, vc, table, sl, ks, vs = _inputs(3, [16] * 8, 8, 8, 1, 128, 16)
    out = torch.empty_like(q)
    # 4096 CTAs x 8 sub-tiles x 8 heads of (128 + 2) floats is far beyond 16 MiB
    st = lib.okc_attn_decode_fp8_noalloc(*_args(q, kc, vc, table, sl, ks, vs, out, 4096),
                                         torch.cuda.current_stream().cuda_stream)
    assert st == _lib.OKC_ERR_TOO_LARGE
