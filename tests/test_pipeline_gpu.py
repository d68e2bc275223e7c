"""HostDevicePipeline: every step's pinned H2D input and D2H result, with the
copies of neighbouring steps overlapping the compute; results must match a
plain per-step computation."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_pipeline_results_match_per_step(depth):
    from kiwi_b200.utils.pipeline import HostDevicePipeline

    steps, n = 7, 1 << 20
    ins = [torch.randn(n).pin_memory() for _ in range(steps)]
    outs = [torch.empty(n).pin_memory() for _ in range(steps)]

    def fn(x, out):
        torch.mul(x, 3.0, out=out)
        out.add_(1.0)

    pipe = HostDevicePipeline(fn, [((n,), torch.float32)], ((n,), torch.float32), depth=depth)
    ms = pipe.run(steps, lambda i: (ins[i],), lambda i: outs[i])
    torch.cuda.synchronize()
    assert ms > 0
    for i in range(steps):
        assert torch.equal(outs[i], ins[i] * 3.0 + 1.0), i
