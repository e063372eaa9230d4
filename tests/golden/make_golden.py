"""Generate the golden fixtures in this folder by running the reference package.

Run here (where the reference checkout is readable), not on the GPU box:

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py

It imports the reference ``mednext_accel`` and executes its own modules on CPU
(the pure-PyTorch path its tests use as ground truth), in float64, on seeded
inputs with the shapes of the reference's tests:

* ``depthwise.npz``  — ``AdaptiveDepthwise3d`` on CPU (its native branch,
  ops/adaptive.py:235-255): stride-1 k in {1,3,5} on [2,3,5,6,7]
  (tests/ops/test_depthwise.py:31-62), stride 2 on [2,3,5,6,7]
  (test_depthwise.py:65-79), transpose on [2,3,4,5,6] (test_depthwise.py:82-96):
  outputs, input grads, weight and bias grads.
* ``blocks.npz``     — reference ``MedNeXtBlock`` / ``MedNeXtDownBlock`` /
  ``MedNeXtUpBlock`` (models/blocks.py:47-182) forward + backward in float64 with
  seeded default init: parameters, input, upstream grad, output and all grads.
* ``model_init.json`` — seed-0 ``mednext_base(1, 3, deep_supervision=True)``
  parameter count, ordered state-dict keys and per-tensor checksums.
* ``small_model.npz`` — seed-0 ``mednext_small(base_channels=4)`` float64
  forward/backward on a 32^3 input: the five deep-supervision heads, the
  mean cross-entropy loss and the stem/head grads.
* ``grn.npz``        — the v2 Global Response Norm, ``GlobalResponseNorm3d``
  (ops/grn.py:16-46) with seeded gamma/beta, forward and autograd backward in
  float64 on [2,6,5,6,7] (one all-zero channel: the zero-norm case) and on
  [1,3,4,4,4].

``python tests/golden/make_golden.py grn`` writes only the named fixtures.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch
from torch import nn
from torch.nn import functional as F

OUT = Path(__file__).resolve().parent


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().double().numpy()


def depthwise() -> dict[str, np.ndarray]:
    from mednext_accel.ops.adaptive import AdaptiveDepthwise3d, ModelOptimizationContext
    from mednext_accel.optimization.policies import PolicyRegistry

    resolver = PolicyRegistry().resolver()
    ctx = ModelOptimizationContext("mednext_v1", "base", "none")
    out: dict[str, np.ndarray] = {}

    def run(tag, conv, shape, seed):
        torch.manual_seed(seed)
        conv = conv.double()
        with torch.no_grad():
            conv.weight.copy_(torch.randn_like(conv.weight))
            conv.bias.copy_(torch.randn_like(conv.bias))
        module = AdaptiveDepthwise3d(conv, resolver, ctx)
        x = torch.randn(*shape, dtype=torch.float64, requires_grad=True)
        y = module(x)
        dy = torch.randn_like(y)
        dx, dw, db = torch.autograd.grad(y, (x, module.weight, module.bias), dy)
        for name, value in (("x", x), ("w", module.weight), ("b", module.bias), ("y", y), ("dy", dy),
                            ("dx", dx), ("dw", dw), ("db", db)):
            out[f"{tag}/{name}"] = _np(value)

    for k in (1, 3, 5):
        run(f"s1_k{k}", nn.Conv3d(3, 3, k, padding=k // 2, groups=3), (2, 3, 5, 6, 7), 17 + k)
    run("s2_k3", nn.Conv3d(3, 3, 3, stride=2, padding=1, groups=3), (2, 3, 5, 6, 7), 47)
    run("s2_k5", nn.Conv3d(3, 3, 5, stride=2, padding=2, groups=3), (2, 3, 6, 5, 7), 48)
    run("t_k3", nn.ConvTranspose3d(3, 3, 3, stride=2, padding=1, groups=3), (2, 3, 4, 5, 6), 41)
    run("t_k5", nn.ConvTranspose3d(3, 3, 5, stride=2, padding=2, groups=3), (2, 3, 3, 4, 5), 42)
    return out


def blocks() -> dict[str, np.ndarray]:
    from mednext_accel.models.blocks import MedNeXtBlock, MedNeXtDownBlock, MedNeXtUpBlock

    out: dict[str, np.ndarray] = {}
    cases = (
        ("regular_k3", MedNeXtBlock, dict(in_channels=4, out_channels=4, expansion_ratio=2, kernel_size=3), (2, 4, 6, 6, 6)),
        ("regular_k5", MedNeXtBlock, dict(in_channels=4, out_channels=4, expansion_ratio=3, kernel_size=5), (1, 4, 7, 6, 5)),
        ("down_k3", MedNeXtDownBlock, dict(in_channels=4, out_channels=8, expansion_ratio=2, kernel_size=3), (2, 4, 6, 6, 6)),
        ("up_k3", MedNeXtUpBlock, dict(in_channels=8, out_channels=4, expansion_ratio=2, kernel_size=3), (2, 8, 4, 4, 4)),
    )
    for seed, (tag, cls, kw, shape) in enumerate(cases):
        torch.manual_seed(seed)
        block = cls(spatial_dims=3, **kw).double().train()
        # non-trivial GroupNorm affine so its gradients are exercised
        with torch.no_grad():
            block.norm.weight.copy_(1.0 + 0.1 * torch.randn_like(block.norm.weight))
            block.norm.bias.copy_(0.1 * torch.randn_like(block.norm.bias))
        x = torch.randn(*shape, dtype=torch.float64, requires_grad=True)
        y = block(x)
        dy = torch.randn_like(y)
        params = dict(block.named_parameters())
        grads = torch.autograd.grad(y, (x, *params.values()), dy)
        out[f"{tag}/x"] = _np(x)
        out[f"{tag}/y"] = _np(y)
        out[f"{tag}/dy"] = _np(dy)
        out[f"{tag}/dx"] = _np(grads[0])
        for (name, p), g in zip(params.items(), grads[1:], strict=True):
            out[f"{tag}/param/{name}"] = _np(p)
            out[f"{tag}/grad/{name}"] = _np(g)
    return out


def model_init() -> dict:
    from mednext_accel import mednext_base

    torch.manual_seed(0)
    model = mednext_base(in_channels=1, out_channels=3, deep_supervision=True, optimization="reference")
    state = model.state_dict()
    return {
        "parameters": sum(p.numel() for p in model.parameters()),
        "keys": list(state),
        "checksums": {
            k: [float(v.double().sum()), float((v.double() ** 2).sum()), [float(a) for a in v.flatten()[:4]]]
            for k, v in state.items()
        },
    }


def small_model() -> dict[str, np.ndarray]:
    from mednext_accel import mednext_small

    torch.manual_seed(0)
    model = mednext_small(in_channels=1, out_channels=3, base_channels=4, deep_supervision=True,
                          optimization="reference").double().train()
    x = torch.randn(1, 1, 32, 32, 32, dtype=torch.float64)
    target = torch.randint(3, (1, 32, 32, 32))
    heads = model(x)
    loss = sum(
        F.cross_entropy(h, target if h.shape[2:] == target.shape[1:] else
                        F.interpolate(target[:, None].double(), size=h.shape[2:], mode="nearest")[:, 0].long())
        for h in heads
    ) / len(heads)
    loss.backward()
    out = {"x": _np(x), "target": target.numpy().astype(np.int64), "loss": np.array([loss.item()])}
    for i, h in enumerate(heads):
        out[f"head{i}"] = _np(h)
    for name, p in model.named_parameters():
        out[f"param/{name}"] = _np(p)
        out[f"grad/{name}"] = _np(p.grad)
    return out


def grn() -> dict[str, np.ndarray]:
    from mednext_accel.ops.grn import GlobalResponseNorm3d

    out: dict[str, np.ndarray] = {}
    for case, shape in enumerate(((2, 6, 5, 6, 7), (1, 3, 4, 4, 4))):
        gen = torch.Generator().manual_seed(100 + case)
        layer = GlobalResponseNorm3d(shape[1]).double()
        with torch.no_grad():
            layer.gamma.copy_(torch.randn(layer.gamma.shape, generator=gen, dtype=torch.float64))
            layer.beta.copy_(torch.randn(layer.beta.shape, generator=gen, dtype=torch.float64))
        x = torch.randn(shape, generator=gen, dtype=torch.float64)
        if case == 0:
            x[1, 2].zero_()  # a channel with zero norm
        x.requires_grad_()
        dy = torch.randn(shape, generator=gen, dtype=torch.float64)
        y = layer(x)
        y.backward(dy)
        for name, value in (("x", x), ("gamma", layer.gamma), ("beta", layer.beta), ("dy", dy), ("y", y),
                            ("dx", x.grad), ("dgamma", layer.gamma.grad), ("dbeta", layer.beta.grad)):
            out[f"{case}/{name}"] = _np(value)
    return out


def main() -> int:
    try:
        import mednext_accel  # noqa: F401
    except ImportError:
        print("put the reference src/ directory on PYTHONPATH", file=sys.stderr)
        return 2
    wanted = set(sys.argv[1:])

    def want(name: str) -> bool:
        return not wanted or name in wanted

    if want("depthwise"):
        np.savez_compressed(OUT / "depthwise.npz", **depthwise())
    if want("blocks"):
        np.savez_compressed(OUT / "blocks.npz", **blocks())
    if want("model_init"):
        (OUT / "model_init.json").write_text(json.dumps(model_init()))
    if want("small_model"):
        np.savez_compressed(OUT / "small_model.npz", **small_model())
    if want("grn"):
        np.savez_compressed(OUT / "grn.npz", **grn())
    print("wrote", sorted(p.name for p in OUT.iterdir()))
    return 0


if __name__ == "__main__":
    sys.exit(main())
