"""Tiny end-to-end pass used by the driver's smoke check (cuda:0): one
forward of a small expert-parallel MoE layer (FP8 dispatch, both tcgen05
grouped GEMMs, fused NVLink-path combine on a world of one) checked against the
fp32 reference, then a device->host queue round of pushes.  The queue ring
holds every message of the round, so the kernel finishes even when its host
side only starts popping after the launch call returns (as under a profiler
that replays the kernel inside the launch)."""


def run():
    """Runs the smoke pass on the current CUDA device; raises on any mismatch."""
    import torch

    import kiwi_b200
    from kiwi_b200.models import moe
    from kiwi_b200.parallel.ep import ExpertParallelMoE
    from kiwi_b200.utils import dist

    C = kiwi_b200.native()
    dist.init()
    cfg = moe.MoEConfig(hidden=1024, ffn=256, num_experts=16, topk=4, tokens_per_rank=64, quant="fp8",
                        name="smoke")
    layer = ExpertParallelMoE(cfg)
    x, logits = moe.synthetic_inputs(cfg, 0, "cuda")
    out = layer(x, logits)
    torch.cuda.synchronize()
    layer.check()
    idx, w = moe.route_reference(logits, cfg.topk)
    ref = moe.moe_reference(cfg, x, idx, w, device=x.device)
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-3, (err, ref.abs().max().item())

    r = C.bench.d2h_push_test("global", False, 256, 1, 50, [8, 100], 1, 1)
    assert r["mismatches"] == 0 and r["popped"] == 50, r
