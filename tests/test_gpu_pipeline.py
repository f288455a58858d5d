"""GPU checks of okc_b200.pipeline.HostPipeline, the double-buffered host I/O around a step:
every submitted step's output reaches its own host buffer, bit-identical to the step run in
series, and steps run in submission order (a stateful step sees the state in series)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_pipeline_outputs_match_series():
    from okc_b200 import ops
    from okc_b200.pipeline import HostPipeline
    T, K, N, steps = 16, 1024, 2048, 7
    g = torch.Generator(device="cuda").manual_seed(5)
    w = (torch.randn((N, K), generator=g, device="cuda") * 0.05).to(torch.bfloat16)

    def step(inp):
        return ops.gemm(inp.view(torch.bfloat16).view(T, K), w)

    pipe = HostPipeline(step, T * K * 2, "cuda")
    xs = [(torch.randn((T, K), generator=g, device="cuda")).to(torch.bfloat16) for _ in range(steps)]
    host_in = [x.view(torch.uint8).reshape(-1).cpu().pin_memory() for x in xs]
    host_out = [torch.empty((T, N), dtype=torch.bfloat16).pin_memory() for _ in range(steps)]
    for k in range(steps):
        pipe.submit(host_in[k], host_out[k])
    pipe.synchronize()
    for k in range(steps):
        assert torch.equal(host_out[k], ops.gemm(xs[k], w).cpu()), f"step {k}"
    pipe.close()


def test_pipeline_keeps_submission_order():
    from okc_b200.pipeline import HostPipeline
    n, steps = 1 << 16, 9
    state = torch.zeros(n, dtype=torch.float32, device="cuda")

    def step(inp):  # out_k = sum of the inputs of steps 0..k
        state.add_(inp.view(torch.float32))
        return state.clone()

    pipe = HostPipeline(step, n * 4, "cuda")  # its two runs on zeros leave the state at zero
    vals = [torch.full((n,), float(k + 1)) for k in range(steps)]
    host_in = [v.view(torch.uint8).pin_memory() for v in vals]
    host_out = [torch.empty(n, dtype=torch.float32).pin_memory() for _ in range(steps)]
    for k in range(steps):
        pipe.submit(host_in[k], host_out[k])
    pipe.synchronize()
    for k in range(steps):
        want = float((k + 1) * (k + 2) // 2)
        assert torch.all(host_out[k] == want), f"step {k}: {host_out[k][0].item()} != {want}"
    pipe.close()


def test_pipeline_rejects_unpinned_or_mis_sized_buffers():
    from okc_b200.pipeline import HostPipeline
    pipe = HostPipeline(lambda inp: inp.view(torch.float32) * 2, 64, "cuda")
    ok_in = torch.arange(64, dtype=torch.uint8).pin_memory()
    ok_out = torch.empty(16, dtype=torch.float32).pin_memory()
    with pytest.raises(RuntimeError, match="pinned"):
        pipe.submit(torch.zeros(64, dtype=torch.uint8), ok_out)
    with pytest.raises(RuntimeError, match="input bytes"):
        pipe.submit(torch.zeros(32, dtype=torch.uint8).pin_memory(), ok_out)
    with pytest.raises(RuntimeError, match="host_out"):
        pipe.submit(ok_in, torch.empty(8, dtype=torch.float32).pin_memory())
    pipe.submit(ok_in, ok_out)
    pipe.synchronize()
    assert torch.equal(ok_out, ok_in.view(torch.float32) * 2)
    pipe.close()
