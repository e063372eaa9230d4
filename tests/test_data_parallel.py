"""Batch-sharded data parallelism on CPU: two ``gloo`` ranks run the bucketed
gradient reducer and must end with the gradient of the mean loss over both
ranks' samples, identical on every rank, with the same bucket order."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model(seed: int) -> nn.Module:
    torch.manual_seed(seed)
    return nn.Sequential(
        nn.Conv3d(2, 8, 3, padding=1), nn.GroupNorm(8, 8), nn.GELU(),
        nn.Conv3d(8, 16, 1), nn.GELU(), nn.Conv3d(16, 3, 1),
    )


def _sample(rank: int) -> tuple[torch.Tensor, torch.Tensor]:
    gen = torch.Generator().manual_seed(100 + rank)
    return torch.randn((1, 2, 6, 6, 6), generator=gen), torch.randint(0, 3, (1, 6, 6, 6), generator=gen)


def _loss(model: nn.Module, x: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
    return nn.functional.cross_entropy(model(x), t)


def _worker(rank: int, port: int, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(WORLD))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        _run(rank, queue)
    except Exception:  # report instead of leaving the parent waiting
        import traceback

        queue.put((rank, "error", traceback.format_exc(), None))
    finally:
        dist.destroy_process_group()


def _run(rank: int, queue) -> None:
    from mednext_accel_b200.data_parallel import GradientBucketReducer, broadcast_parameters

    model = _model(seed=rank)  # different init per rank: broadcast must fix it
    broadcast_parameters(model)
    reducer = GradientBucketReducer(model, bucket_cap_mb=1e-4)  # 26 floats: several buckets
    assert len(reducer.buckets) > 1
    for _ in range(2):  # two steps: zero_grad must reset the buckets
        reducer.zero_grad()
        x, t = _sample(rank)
        _loss(model, x, t).backward()
        reducer.finish()
    # numpy copies: tensors would travel as shared-memory handles that die with the process
    grads = [p.grad.detach().numpy().copy() for p in model.parameters()]
    params = [p.detach().numpy().copy() for p in model.parameters()]
    queue.put((rank, grads, params, list(reducer.order)))


def test_bucketed_all_reduce_averages_gradients_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, queue)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(WORLD):
        rank, grads, params, order = queue.get(timeout=180)
        assert grads != "error", params
        results[rank] = (grads, params, order)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0

    # reference: rank 0's initial weights, mean of the per-sample losses, one process
    ref = _model(seed=0)
    total = sum(_loss(ref, *_sample(r)) for r in range(WORLD)) / WORLD
    want = torch.autograd.grad(total, list(ref.parameters()))
    for rank in range(WORLD):
        grads, params, order = results[rank]
        for p_ref, p_got in zip(ref.parameters(), params, strict=True):
            torch.testing.assert_close(torch.from_numpy(p_got), p_ref.detach(), rtol=0, atol=0)
        for g_want, g_got in zip(want, grads, strict=True):
            torch.testing.assert_close(torch.from_numpy(g_got), g_want, rtol=1e-5, atol=1e-6)
    assert results[0][2] == results[1][2]  # same bucket order on every rank
    for g0, g1 in zip(results[0][0], results[1][0], strict=True):
        torch.testing.assert_close(torch.from_numpy(g0), torch.from_numpy(g1), rtol=0, atol=0)


def test_single_process_reducer_keeps_local_gradients():
    from mednext_accel_b200.data_parallel import GradientBucketReducer

    model = _model(seed=3)
    reducer = GradientBucketReducer(model, bucket_cap_mb=1e-4)
    reducer.zero_grad()
    x, t = _sample(0)
    _loss(model, x, t).backward()
    reducer.finish()
    ref = _model(seed=3)
    want = torch.autograd.grad(_loss(ref, x, t), list(ref.parameters()))
    for p, g in zip(model.parameters(), want, strict=True):
        torch.testing.assert_close(p.grad, g, rtol=1e-6, atol=1e-7)
    assert sorted(reducer.order) == list(range(len(reducer.buckets)))


if __name__ == "__main__":  # pragma: no cover
    pytest.main([__file__, "-q"])
