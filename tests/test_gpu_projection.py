"""GPU parity of the projection kernels (C ABI okc_gemm_bf16) against the CPU oracle.

Tolerance (the path's stated tolerance): bf16 outputs within rtol 2e-2 / atol 2e-2 of the fp32-
accumulated reference, plus a relative-L2 bound of 5e-3 (one bf16 rounding of the output
is ~2e-3 relative).
"""

import pytest
import torch

from oracle import projection as ref

pytestmark = pytest.mark.gpu

KN = [(4096, 6144), (4096, 4096), (8192, 10240), (8192, 8192), (28672, 8192)]


def _close(out, exp, what):
    out, exp = out.float().cpu(), exp.float().cpu()
    torch.testing.assert_close(out, exp, rtol=2e-2, atol=2e-2, msg=what)
    rel = (out - exp).norm() / exp.norm().clamp_min(1e-30)
    assert rel < 5e-3, f"{what}: rel L2 {rel:.2e}"


@pytest.fixture(scope="module")
def ops():
    from okc_b200 import ops
    return ops


@pytest.mark.parametrize("M", [1, 4, 16, 64])
@pytest.mark.parametrize("K,N", KN)
def test_baseline_shapes(ops, M, K, N):
    from okc_b200 import synth
    x, w = synth.projection_case(M, K, N, seed=M * 7 + K + N, device="cuda")
    y = ops.gemm(x, w)
    torch.cuda.synchronize()
    _close(y, ref.gemm(x.cpu(), w.cpu()), f"M{M} K{K} N{N}")


@pytest.mark.parametrize("M,K,N", [(1, 64, 8), (3, 136, 200), (7, 1000, 129), (9, 2048, 300),
                                   (17, 512, 1000), (33, 4096, 513), (65, 1024, 256), (130, 512, 384)])
def test_ragged_shapes(ops, M, K, N):
    from okc_b200 import synth
    x, w = synth.projection_case(M, K, N, seed=11, device="cuda")
    _close(ops.gemm(x, w), ref.gemm(x.cpu(), w.cpu()), f"M{M} K{K} N{N}")


@pytest.mark.parametrize("splits", [1, 2, 3, 5, 8])
def test_forced_splits_and_residual(ops, splits):
    from okc_b200 import synth
    M, K, N = 5, 4096, 1024
    x, w = synth.projection_case(M, K, N, seed=3, device="cuda")
    r = torch.randn((M, N), device="cuda").to(torch.bfloat16)
    y = ops.gemm(x, w, residual=r, family=1, splits=splits)
    _close(y, ref.gemm(x.cpu(), w.cpu(), residual=r.cpu()), f"splits {splits}")
    y32 = ops.gemm(x, w, out_fp32=True, family=1, splits=splits)
    torch.testing.assert_close(y32.cpu(), ref.gemm(x.cpu(), w.cpu(), out_fp32=True), rtol=1e-3, atol=1e-3)


def test_strided_input_and_determinism(ops):
    from okc_b200 import synth
    x, w = synth.projection_case(16, 8192, 2048, seed=5, device="cuda")
    xs = torch.zeros((16, 8192 + 64), device="cuda", dtype=torch.bfloat16)
    xs[:, :8192] = x
    y1 = ops.gemm(xs[:, :8192], w)
    y2 = ops.gemm(xs[:, :8192], w)
    assert torch.equal(y1, y2), "split-K reduction must be deterministic"
    _close(y1, ref.gemm(x.cpu(), w.cpu()), "strided x")


def test_rmsnorm(ops):
    x = torch.randn((5, 8192), device="cuda").to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(8192, device="cuda")).to(torch.bfloat16)
    for unit in (False, True):
        y = ops.rmsnorm(x, w, 1e-6, unit_offset=unit)
        torch.testing.assert_close(y.float().cpu(), ref.rmsnorm(x.cpu(), w.cpu(), 1e-6, unit).float(),
                                   rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("M", [33, 48, 64, 65, 100, 128, 200, 256])
@pytest.mark.parametrize("K,N", [(8192, 10240), (8192, 8192), (4096, 6144), (1000, 300)])
def test_tcgen05_family(ops, M, K, N):
    """The tcgen05 kernel (family 2) against the oracle and against the split-K CUDA-core path."""
    from okc_b200 import synth
    x, w = synth.projection_case(M, K, N, seed=M + N, device="cuda")
    y = ops.gemm(x, w, family=2)
    _close(y, ref.gemm(x.cpu(), w.cpu()), f"tc M{M} K{K} N{N}")
    r = torch.randn((M, N), device="cuda").to(torch.bfloat16)
    y2 = ops.gemm(x, w, residual=r, family=2)
    _close(y2, ref.gemm(x.cpu(), w.cpu(), residual=r.cpu()), f"tc+res M{M}")
    y3 = ops.gemm(x, w, out_fp32=True, family=2)
    torch.testing.assert_close(y3.cpu(), ref.gemm(x.cpu(), w.cpu(), out_fp32=True), rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("M,family", [(300, 0), (544, 0), (600, 2)])
def test_prefill_token_counts(ops, M, family):
    """M > 256 (prefill blocks): 256-row blocks of the tcgen05 kernel, a tail of <= 32 rows on the
    skinny kernel (M = 544 = 2 x 256 + 32), with and without a residual."""
    from okc_b200 import synth
    x, w = synth.projection_case(M, 4096, 2304, seed=M, device="cuda")
    _close(ops.gemm(x, w, family=family), ref.gemm(x.cpu(), w.cpu()), f"prefill M{M}")
    r = torch.randn((M, 2304), device="cuda").to(torch.bfloat16)
    _close(ops.gemm(x, w, residual=r, family=family), ref.gemm(x.cpu(), w.cpu(), residual=r.cpu()), f"prefill+res M{M}")


def test_contract_short_names(ops):
    """okc_gemv_bf16 / okc_rmsnorm (the contract's short names) give the same bytes as the
    full entry points."""
    import ctypes as C
    from okc_b200 import _lib, synth
    lib = _lib.load()
    x, w = synth.projection_case(4, 4096, 6144, device="cuda")
    y_ref = ops.gemm(x, w)
    y = torch.empty_like(y_ref)
    scratch = torch.zeros(lib.okc_gemm_bf16_workspace_bytes(4, 6144, 4096) + 256, dtype=torch.uint8, device="cuda")
    st = lib.okc_gemv_bf16(x.data_ptr(), w.data_ptr(), y.data_ptr(), 4, 6144, 4096, 4096, scratch.data_ptr(),
                           torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))
    g = torch.Generator(device="cuda").manual_seed(5)
    xn = torch.randn((3, 1024), generator=g, device="cuda").to(torch.bfloat16)
    nw = torch.randn((1024,), generator=g, device="cuda").to(torch.bfloat16)
    r_ref = ops.rmsnorm(xn, nw, 1e-6)
    r = torch.empty_like(r_ref)
    assert lib.okc_rmsnorm(xn.data_ptr(), nw.data_ptr(), r.data_ptr(), 3, 1024, C.c_float(1e-6),
                           torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(r.view(torch.int16), r_ref.view(torch.int16))
