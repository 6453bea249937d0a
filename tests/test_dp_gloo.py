"""Host logic of the multi-GPU step (tinygs_b200/dp.py) on two CPU ranks over
gloo: view assignment, the gradient all-reduce, the Adam gradient scale and
the max-over-ranks timing reduction.  The reference semantics it must
reproduce: accumulate_grad_steps = N adds the gradients of N consecutive
views into one arena and steps once with scale 1/(grad_scaler * N)
(tinygs/src/orchestrator.cu:343-403)."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2
N_VIEWS = 60
ARENA = 4 * 59 * 8  # a small gradient arena, 59 floats per Gaussian


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _view_grads(view: int) -> np.ndarray:
    return np.random.default_rng(1000 + view).normal(size=ARENA).astype(np.float32)


def _worker(rank: int, port: int, out_dir: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        from tinygs_b200.dp import DataParallel

        dp = DataParallel.from_env()
        steps = 5
        views = [dp.view_index(k, N_VIEWS) for k in range(steps)]
        grads = [torch.from_numpy(_view_grads(v)) for v in views]
        reduced = [dp.reduce_gradients(g.clone()) for g in grads]
        scale = dp.gradient_scale(10.0)
        t = dp.max_over_ranks(float(rank + 1) * 3.5, "cpu")
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), views=np.array(views),
                 reduced=np.stack([r.numpy() for r in reduced]), scale=scale, tmax=t, world=dp.world)
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_rank_step_semantics(tmp_path):
    mp.start_processes(_worker, args=(_free_port(), str(tmp_path)), nprocs=WORLD, start_method="spawn")
    r = [np.load(tmp_path / f"rank{k}.npz") for k in range(WORLD)]
    assert all(int(x["world"]) == WORLD for x in r)
    steps = len(r[0]["views"])
    for k in range(steps):
        # the ranks of step k render the consecutive views k*N .. k*N+N-1
        vk = sorted(int(x["views"][k]) for x in r)
        assert vk == [(k * WORLD + j) % N_VIEWS for j in range(WORLD)]
        # every rank holds the sum of the step's per-view gradients
        expect = sum(_view_grads(v) for v in vk)
        for x in r:
            np.testing.assert_allclose(x["reduced"][k], expect, rtol=1e-6, atol=1e-6)
    # scale 1/(grad_scaler * N): the same as the reference's accumulation
    for x in r:
        assert float(x["scale"]) == pytest.approx(1.0 / (10.0 * WORLD))
        assert float(x["tmax"]) == pytest.approx(3.5 * WORLD)


def test_single_process_is_identity():
    from tinygs_b200.dp import DataParallel

    dp = DataParallel.from_env()
    assert (dp.world, dp.rank) == (1, 0)
    g = torch.arange(6, dtype=torch.float32)
    assert torch.equal(dp.reduce_gradients(g.clone()), g)
    assert [dp.view_index(k, 4) for k in range(6)] == [0, 1, 2, 3, 0, 1]
    assert dp.gradient_scale(10.0) == pytest.approx(0.1)
    assert dp.max_over_ranks(2.5, "cpu") == 2.5
