"""The native mean cross-entropy against F.cross_entropy (fp32 math on the same
stored logits), forward and backward, with ignored and counted targets."""

from __future__ import annotations

import pytest
import torch
from torch.nn import functional as F

from mednext_accel_b200 import _native as nat
from mednext_accel_b200.loss import cross_entropy

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(1, 3, 128, 128, 128), (2, 3, 9, 10, 11), (2, 5, 33), (1, 2, 8, 8, 8)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_cross_entropy_matches_torch(shape, dtype):
    gen = torch.Generator().manual_seed(sum(shape))
    logits = (torch.randn(shape, generator=gen) * 3).to(dtype).cuda()
    target = torch.randint(0, shape[1], (shape[0], *shape[2:]), generator=gen).cuda()
    target.view(-1)[::7] = -100  # ignored voxels
    x1 = logits.clone().requires_grad_()
    x2 = logits.clone().requires_grad_()
    loss = cross_entropy(x1, target)
    want = F.cross_entropy(x2.float(), target)
    assert loss.dtype == torch.float32
    assert torch.allclose(loss, want, rtol=1e-5, atol=1e-6), (loss.item(), want.item())
    (g1,) = torch.autograd.grad(loss * 1.7, x1)
    (g2,) = torch.autograd.grad(want * 1.7, x2)
    assert g1.dtype == dtype
    tol = 1e-6 if dtype == torch.float32 else 0.0
    err = (g1.float() - g2.float()).abs()
    # the same fp32 value rounded to the logits' dtype, up to one rounding step
    ulp = g2.float().abs() * (2.0**-7 if dtype == torch.bfloat16 else 2.0**-20) + tol + 1e-12
    assert bool((err <= ulp).all()), err.max().item()


def test_cross_entropy_under_autocast_and_graph_capture():
    # every use of the leaf runs on the side stream: autograd records a leaf's
    # stream at its first use, and a leaf first used on the legacy stream cannot
    # take a gradient inside a capture
    target = torch.randint(0, 3, (1, 16, 16, 16), device="cuda")
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        logits = torch.randn((1, 3, 16, 16, 16), device="cuda", dtype=torch.bfloat16, requires_grad=True)
        want = F.cross_entropy(logits.detach().float(), target)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = cross_entropy(logits, target)
        assert torch.allclose(loss, want, rtol=1e-5)
        loss.backward()
        want_grad = logits.grad.clone()
        logits.grad = None
        del loss  # free the eager graph: no AccumulateGrad node of it outlives the capture
        with torch.cuda.graph(g):
            out = cross_entropy(logits, target)
            out.backward()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.allclose(out, want, rtol=1e-5)
    assert torch.equal(logits.grad, want_grad)


def test_all_ignored_gives_nan_like_torch():
    logits = torch.randn((1, 3, 4, 4, 4), device="cuda")
    target = torch.full((1, 4, 4, 4), -100, device="cuda", dtype=torch.long)
    assert torch.isnan(cross_entropy(logits, target)) and torch.isnan(F.cross_entropy(logits, target))


def test_no_device_error_recorded():
    assert nat.device_error() == 0
