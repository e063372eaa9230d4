"""The CPU restatement that bench.py times as the reference's CPU step
(oracle/reference_model.py) against the reference package's own forward and
backward (tests/golden/small_model.npz, written by tests/golden/make_golden.py
from ``mednext_small(base_channels=4, optimization="reference")`` in float64).

Two checks: the functional forward, the five-head loss and autograd in float64
at round-off tolerance, and one ``ReferenceTrainer.step`` (the exact code the
CPU baseline times, float32) against the same gradients at float32 tolerance.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import reference_model as rm


def _params(fx, dtype):
    names = [k[len("param/"):] for k in fx.files if k.startswith("param/")]
    return {n: torch.from_numpy(fx[f"param/{n}"]).to(dtype) for n in names}


def _rel(a: np.ndarray, b: np.ndarray) -> float:
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den > 0 else float(np.linalg.norm(a - b))


def test_functional_forward_and_backward_match_reference_float64(golden):
    fx = golden("small_model.npz")
    params = {n: t.clone().requires_grad_() for n, t in _params(fx, torch.float64).items()}
    x = torch.from_numpy(fx["x"])
    target = torch.from_numpy(fx["target"])
    heads = rm.forward(params, x, "small", 3)
    assert len(heads) == 5
    for i, h in enumerate(heads):
        np.testing.assert_allclose(h.detach().numpy(), fx[f"head{i}"], rtol=1e-10, atol=1e-12)
    loss = rm.loss_fn(heads, rm.targets_for(target, heads))
    np.testing.assert_allclose(loss.item(), fx["loss"][0], rtol=1e-12)
    loss.backward()
    for n, p in params.items():
        want = fx[f"grad/{n}"]
        if n.endswith("depthwise.bias"):
            # zero in exact arithmetic (GroupNorm(C, C) follows): compare absolutely
            assert np.abs(p.grad.numpy() - want).max() <= 1e-12, n
            continue
        assert _rel(p.grad.numpy(), want) <= 1e-9, n


def test_reference_trainer_step_gradients_match_reference(golden):
    fx = golden("small_model.npz")
    state = _params(fx, torch.float64)
    trainer = rm.ReferenceTrainer(state, "small", 3)
    x = torch.from_numpy(fx["x"]).float()
    target = torch.from_numpy(fx["target"])
    with torch.no_grad():
        targets = rm.targets_for(target, rm.forward(trainer.params, x, "small", 3))
    before = {n: p.detach().clone() for n, p in trainer.params.items()}
    loss = trainer.step(x, targets)
    np.testing.assert_allclose(loss, fx["loss"][0], rtol=1e-5)
    for n, p in trainer.params.items():
        want = fx[f"grad/{n}"]
        got = p.grad.double().numpy()
        if n.endswith("depthwise.bias"):
            assert np.abs(got - want).max() <= 1e-5, n
            continue
        assert _rel(got, want) <= 1e-4, n
        # AdamW moved every parameter that has a gradient
        assert not torch.equal(p.detach(), before[n]), n
