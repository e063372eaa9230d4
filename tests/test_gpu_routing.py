"""Standalone convolutions wrapped by ``install_adaptive_operators`` and the custom
op registrations, on the GPU.

The reference pins these with ``torch.library.opcheck`` on its custom ops
(tests/ops/test_depthwise.py:8-28), dX/dW routing under autocast
(tests/ops/test_phase_routing.py:114-139) and the gradient-mask matrix
(tests/ops/test_phase_routing.py:318-370).  Here:

* every sm_100a custom op passes opcheck's schema, autograd-registration and
  fake-tensor checks;
* wrapped depthwise Conv3d (stride 1, k 3/5/7; stride 2) and ConvTranspose3d
  (stride 2) run the sm_100a ops in forward and backward, and match the fp64
  oracle in float32 (max relative error <= 1e-5 of each tensor's largest value)
  and PyTorch's own convolution under bf16 autocast (relative L2 <= 2e-2);
* wrapped 1x1x1 Conv3d / ConvTranspose3d run the tensor-core pointwise op under
  autocast (relative L2 <= 2e-2);
* requesting a subset of the gradients (x, weight, bias) computes exactly that
  subset.
"""

from __future__ import annotations

import copy
import itertools

import numpy as np
import pytest
import torch
from torch import nn
from torch.utils._python_dispatch import TorchDispatchMode

import mednext_accel_b200 as mx
from mednext_accel_b200 import depthwise as dwk
from mednext_accel_b200.adaptive import ModelOptimizationContext
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
OPCHECK = ("test_schema", "test_autograd_registration", "test_faketensor")


class Spy(TorchDispatchMode):
    def __init__(self):
        super().__init__()
        self.ops = []

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        self.ops.append(func._schema.name)
        return func(*args, **(kwargs or {}))


def _install(module: nn.Module) -> nn.Module:
    model = nn.Sequential(module)
    n = mx.install_adaptive_operators(model, resolver=mx.PolicyResolver(),
                                      model_context=ModelOptimizationContext("mednext_v1", "base", "none"))
    assert n == 1
    return model.cuda().train()


def _opcheck(op, args):
    res = torch.library.opcheck(op, args, test_utils=OPCHECK, raise_exception=False)
    assert res == {k: "SUCCESS" for k in OPCHECK}, res


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_opcheck_depthwise_ops(dtype):
    dev = "cuda"
    x = torch.randn(1, 2, 6, 6, 6, device=dev, dtype=dtype, requires_grad=True)
    w = torch.randn(2, 1, 3, 3, 3, device=dev, dtype=dtype, requires_grad=True)
    b = torch.randn(2, device=dev, dtype=dtype, requires_grad=True)
    _opcheck(dwk.depthwise_conv3d_regular, (x, w, b, 3, 2, 6, 2, 128, 128))
    _opcheck(dwk.depthwise_conv3d_stride2_regular, (x, w, b, 3, 2, 6, 128))
    xs = torch.randn(1, 2, 4, 4, 4, device=dev, dtype=dtype, requires_grad=True)
    _opcheck(dwk.depthwise_conv_transpose3d_regular, (xs, w, b, 3, 2, 4, 2, 128))
    dy = torch.randn(1, 2, 6, 6, 6, device=dev, dtype=dtype)
    _opcheck(dwk.depthwise_input_grad_regular, (dy, w.detach(), 3, 2, 6, 128))
    _opcheck(dwk.depthwise_weight_grad_regular, (x.detach(), dy, 3, 2, 6, 2, 128))


def test_opcheck_pointwise_grn_and_loss_ops():
    from mednext_accel_b200.grn import grn_forward
    from mednext_accel_b200.loss import cross_entropy_mean
    from mednext_accel_b200.pointwise import pointwise_conv3d

    bf = torch.bfloat16
    x = torch.randn(2, 32, 4, 4, 8, device="cuda", dtype=bf, requires_grad=True)
    w = (torch.randn(48, 32, 1, 1, 1, device="cuda") * 0.2).to(bf).requires_grad_()
    b = torch.randn(48, device="cuda", dtype=bf, requires_grad=True)
    _opcheck(pointwise_conv3d, (x, w, b))
    g = torch.randn(1, 32, 1, 1, 1, device="cuda", requires_grad=True)
    beta = torch.randn(1, 32, 1, 1, 1, device="cuda", requires_grad=True)
    _opcheck(grn_forward, (x, g, beta, 1e-6))
    logits = torch.randn(2, 3, 4, 4, 8, device="cuda", dtype=bf, requires_grad=True)
    target = torch.randint(0, 3, (2, 4, 4, 8), device="cuda")
    _opcheck(cross_entropy_mean, (logits, target, -100))


CONVS = [
    ("regular", 3), ("regular", 5), ("regular", 7), ("downsample", 3), ("downsample", 5), ("transpose", 3),
]


def _conv(direction: str, k: int, c: int) -> nn.Module:
    if direction == "transpose":
        return nn.ConvTranspose3d(c, c, k, stride=2, padding=k // 2, groups=c)
    return nn.Conv3d(c, c, k, stride=1 if direction == "regular" else 2, padding=k // 2, groups=c)


def _oracle(direction, k, x, w, b, dy):
    """(y, dx, dw, db) in fp64 from the C oracle."""
    if direction == "regular":
        y = orc.dw_fwd(x, w, b, k)
        dx = orc.dw_dgrad(dy, w, k)
        dw, db = orc.dw_wgrad(x, dy, k)
    elif direction == "downsample":
        y = orc.s2_fwd(x, w, b, k)
        dx = orc.s2_dgrad(dy, w, x.shape[2:], k)
        dw, db = orc.s2_wgrad(x, dy, k)
    else:
        y = orc.t_fwd(x, w, b, k)
        dx = orc.t_dgrad(dy, w, k)
        dw, db = orc.t_wgrad(x, dy, k)
    return y, dx, dw, db


def _max_rel(got: torch.Tensor, want: np.ndarray) -> float:
    g = got.detach().double().cpu().numpy().reshape(want.shape)
    return float(np.abs(g - want).max() / max(np.abs(want).max(), 1e-30))


@pytest.mark.parametrize("direction,k", CONVS)
def test_wrapped_depthwise_float32_matches_oracle(direction, k):
    torch.manual_seed(k)
    conv = _conv(direction, k, 6)
    model = _install(copy.deepcopy(conv))
    size = 7 if direction == "transpose" else 12
    x = torch.randn(2, 6, size, size, size, device="cuda", requires_grad=True)
    with Spy() as fwd:
        y = model(x)
    assert any(op.startswith("mednext_accel_b200::depthwise") for op in fwd.ops), fwd.ops
    dy = torch.randn_like(y)
    with Spy() as bwd:
        y.backward(dy)
    assert not any(op == "aten::convolution_backward" for op in bwd.ops)
    m = model[0]
    w64 = m.weight.detach().double().cpu().numpy()
    b64 = m.bias.detach().double().cpu().numpy()
    oy, odx, odw, odb = _oracle(direction, k, x.detach().double().cpu().numpy(), w64, b64,
                                dy.double().cpu().numpy())
    assert _max_rel(y, oy) <= 1e-5
    assert _max_rel(x.grad, odx) <= 1e-5
    assert _max_rel(m.weight.grad, odw.reshape(m.weight.shape)) <= 1e-5
    assert _max_rel(m.bias.grad, odb) <= 1e-5
    for p in (m.weight, m.bias):
        assert p.grad.dtype == torch.float32


@pytest.mark.parametrize("direction,k", CONVS)
def test_wrapped_depthwise_bf16_autocast_matches_torch(direction, k):
    torch.manual_seed(100 + k)
    ref = _conv(direction, k, 8).cuda()
    model = _install(copy.deepcopy(ref))
    size = 9 if direction == "transpose" else 16
    x = torch.randn(2, 8, size, size, size, device="cuda")
    xa, xb = x.clone().requires_grad_(), x.clone().requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        want = ref(xa)
        with Spy() as fwd:
            got = model(xb)
    assert any(op.startswith("mednext_accel_b200::depthwise") for op in fwd.ops)
    assert got.dtype == want.dtype == torch.bfloat16
    dy = torch.randn_like(want)
    gw = torch.autograd.grad(want, (xa, *ref.parameters()), dy)
    gg = torch.autograd.grad(got, (xb, *model[0].parameters()), dy)

    def rel(a, b):
        return ((a.float() - b.float()).norm() / b.float().norm()).item()

    assert rel(got, want) <= 2e-2
    for a, b in zip(gg, gw, strict=True):
        assert a.dtype == b.dtype
        assert rel(a, b) <= 2e-2


@pytest.mark.parametrize("transposed", [False, True])
def test_wrapped_pointwise_bf16_autocast_matches_torch(transposed):
    torch.manual_seed(7)
    ref = (nn.ConvTranspose3d(32, 3, 1) if transposed else nn.Conv3d(32, 48, 1)).cuda()
    model = _install(copy.deepcopy(ref))
    x = torch.randn(2, 32, 8, 8, 16, device="cuda")
    xa, xb = x.clone().requires_grad_(), x.clone().requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        want = ref(xa)
        with Spy() as fwd:
            got = model(xb)
    assert "mednext_accel_b200::pointwise_conv3d" in fwd.ops
    dy = torch.randn_like(want)
    gw = torch.autograd.grad(want, (xa, *ref.parameters()), dy)
    gg = torch.autograd.grad(got, (xb, *model[0].parameters()), dy)
    for a, b in zip((got, *gg), (want, *gw), strict=True):
        assert ((a.float() - b.float()).norm() / b.float().norm()).item() <= 2e-2


@pytest.mark.parametrize("direction", ["regular", "downsample", "transpose"])
@pytest.mark.parametrize("mask", [m for m in itertools.product([False, True], repeat=3) if any(m)])
def test_requested_gradient_subsets(direction, mask):
    torch.manual_seed(47)
    ref = _conv(direction, 3, 2).cuda()
    model = _install(copy.deepcopy(ref))
    for module in (ref, model[0]):
        module.weight.requires_grad_(mask[1])
        module.bias.requires_grad_(mask[2])
    size = 5
    x = torch.randn(1, 2, size, size, size, device="cuda", dtype=torch.bfloat16)
    xa = x.clone().requires_grad_(mask[0])
    xb = x.clone().requires_grad_(mask[0])
    with torch.autocast("cuda", dtype=torch.bfloat16):
        want, got = ref(xa), model(xb)
    dy = torch.randn_like(want)
    want.backward(dy)
    got.backward(dy)
    for a, b, needed in zip((xb, *model[0].parameters()), (xa, *ref.parameters()), mask, strict=True):
        if needed:
            assert a.grad is not None
            assert ((a.grad.float() - b.grad.float()).norm() / b.grad.float().norm()).item() <= 2e-2
        else:
            assert a.grad is None
