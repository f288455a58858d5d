"""Failure detection of the tensor-parallel kernels without a GPU fault: a peer that never
arrives.  One process, one GPU; the "peer" rank 1 is a set of local stand-in buffers that no
kernel ever writes, so every flag wait of rank 0 runs out after its 2 s bound.  The kernel must
then return on its own with OKC_DEVERR_TIMEOUT in the error word (not hang, not fault), and the
CUDA context must stay usable.  Each case spends ~4 s of GPU time in bounded waits."""

import ctypes as C
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

OKC_DEVERR_TIMEOUT = 1


def _context_still_usable():
    from oracle import projection as oproj
    from okc_b200 import ops, synth
    x, w = synth.projection_case(4, 256, 128, seed=3, device="cuda:0")
    y = ops.gemm(x, w)
    torch.testing.assert_close(y.float().cpu(), oproj.gemm(x.cpu(), w.cpu()).float(), rtol=2e-2, atol=2e-2)


def test_exchange_times_out_when_a_peer_never_arrives():
    from okc_b200 import _lib, ops
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    n = 64 * 1024
    part0 = torch.randn(n, device=dev)
    part1 = torch.zeros(n, device=dev)                 # the absent peer's partial
    out0 = torch.empty(n, dtype=torch.bfloat16, device=dev)
    out1 = torch.empty_like(out0)
    flags0 = torch.zeros(8192, dtype=torch.int32, device=dev)
    flags1 = torch.zeros_like(flags0)
    state = torch.zeros(1024, dtype=torch.int32, device=dev)
    ws = ops.workspace(0, "tp_timeout", 4096)
    arr = C.c_void_p * 2
    t0 = time.time()
    st = lib.okc_tp_allreduce_residual(arr(part0.data_ptr(), part1.data_ptr()), arr(out0.data_ptr(), out1.data_ptr()),
                                       arr(flags0.data_ptr(), flags1.data_ptr()), None, state.data_ptr(), 0, 2, n,
                                       ws.data_ptr(), torch.cuda.current_stream(0).cuda_stream)
    assert st == 0
    err = ops.read_device_error("tp_timeout", 0)       # synchronises
    elapsed = time.time() - t0
    assert err == OKC_DEVERR_TIMEOUT, err
    assert elapsed > 1.5, elapsed                       # it did wait (entry, then exit: ~4 s)
    # rank 0 still published its entry and exit flags (epoch 1) to the stand-in peer
    assert int(flags1[0]) == 1 and int(flags1[4096]) == 1
    assert int(state[0]) == 1                           # the CTA's call epoch advanced
    _context_still_usable()


def test_fused_oproj_times_out_when_a_peer_never_arrives():
    from okc_b200 import _lib, ops
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    T, H, K = 64, 1024, 256
    rb, fw = C.c_size_t(), C.c_int()
    assert lib.okc_tp_oproj_plan(T, H, K, 2, C.byref(rb), C.byref(fw)) == 0
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn((T, K), generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn((H, K), generator=g, device=dev) * 0.05).to(torch.bfloat16)
    recv0 = torch.zeros(rb.value // 4, device=dev)
    recv1 = torch.zeros_like(recv0)                    # the absent peer's receive slots
    out0 = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    out1 = torch.empty_like(out0)
    flags0 = torch.zeros(fw.value, dtype=torch.int32, device=dev)
    flags1 = torch.zeros_like(flags0)
    state = torch.zeros(1024, dtype=torch.int32, device=dev)
    ws = ops.workspace(0, "tp_timeout", 4096)
    arr = C.c_void_p * 2
    t0 = time.time()
    st = lib.okc_tp_oproj_allreduce_residual(x.data_ptr(), K, w.data_ptr(), K, T, H, K,
                                             arr(recv0.data_ptr(), recv1.data_ptr()),
                                             arr(out0.data_ptr(), out1.data_ptr()),
                                             arr(flags0.data_ptr(), flags1.data_ptr()), None, H, state.data_ptr(),
                                             0, 2, ws.data_ptr(), torch.cuda.current_stream(0).cuda_stream)
    assert st == 0
    err = ops.read_device_error("tp_timeout", 0)
    elapsed = time.time() - t0
    assert err == OKC_DEVERR_TIMEOUT, err
    assert elapsed > 1.5, elapsed
    # rank 0's pushes of the slices rank 1 owns (tokens 16..31 of each tile's first half) landed
    # in the stand-in peer's receive slots, and its push flag for CTA 0 carries epoch 1
    assert float(recv1.abs().sum()) > 0
    assert int(flags1[0]) == 1
    _context_still_usable()
