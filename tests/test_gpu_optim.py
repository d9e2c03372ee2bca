"""Fused per-cell Adam against torch.optim.Adam with the reference's groups."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_cell_adam_matches_torch_adam():
    from vorotracing_b200.optim import CellAdam
    from vorotracing_b200.shard import GradBucket

    torch.manual_seed(0)
    n, cols = 1000, 48
    pb = GradBucket(n, cols, "cuda")
    for t in pb.views():
        t.normal_()
    pb.density.add_(29.5)  # some entries cross the clamp
    ref = [t.clone().requires_grad_() for t in (pb.points, pb.density, pb.diffuse, pb.specular)]
    lrs = (1e-3, 5e-2, 2e-2, 1e-2)
    opt = torch.optim.Adam([{"params": [r], "lr": lr} for r, lr in zip(ref, lrs)], eps=1e-15)
    ours = CellAdam(pb, lrs=lrs)
    for step in range(5):
        grads = [torch.randn_like(r) for r in ref]
        for r, g in zip(ref, grads):
            r.grad = g.clone()
        for dst, g in zip((ours.grads.points, ours.grads.density, ours.grads.diffuse,
                           ours.grads.specular), grads):
            dst.copy_(g)
        opt.step()
        with torch.no_grad():
            ref[1].clamp_(max=30.0)
        ours.step()
        for a, b in zip((pb.points, pb.density, pb.diffuse, pb.specular), ref):
            torch.testing.assert_close(a, b.detach(), rtol=1e-5, atol=1e-6)
    assert pb.density.max().item() <= 30.0
