"""The data-parallel optimizer step over peer memory on two GPUs
(tgs_dp_reduce_adam through tinygs_b200.dp.PeerAdam): after one step every
rank holds exactly the parameters that one GPU gets from Adam over the sum
of both ranks' gradients (the reference's accumulation of two views).
Needs two GPUs; skipped otherwise."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

N = 50_001  # not a multiple of 4: the last slice has a scalar tail


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _arrays(seed: int, n: int, scale: float):
    rng = np.random.default_rng(seed)
    w = {"means": 3, "opacities": 1, "rotations": 4, "scales": 3, "sh0": 3, "sh_rest": 45}
    return {k: (rng.normal(0, scale, (n, c))).astype(np.float32) for k, c in w.items()}


def _worker(rank: int, port: int, out_dir: str, mode: str = "peer") -> None:
    import torch.distributed as dist

    from tinygs_b200 import dp as dpm
    from tinygs_b200 import runtime as rt

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        dp = dpm.DataParallel.from_env()
        if mode == "multicast":
            params = dpm.symmetric_gaussian_set(dp, N, 3)
            grads = dpm.symmetric_gaussian_set(dp, N, 3)
        else:
            params = dpm.shared_gaussian_set(N, 3)
            grads = dpm.shared_gaussian_set(N, 3)
        params.copy_from_numpy(_arrays(1, N, 1.0))
        grads.copy_from_numpy(_arrays(100 + rank, N, 1e-2))
        cls = dpm.MulticastAdam if mode == "multicast" else dpm.PeerAdam
        opt = cls(dp, params, grads, rt.AdamParams(max_grad_1=0.3))
        for _ in range(2):
            opt.step(dp.gradient_scale(10.0))
        torch.cuda.synchronize()
        out = params.to_numpy()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **out)
        opt.barrier()
        opt.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["peer", "multicast"])
def test_peer_adam_two_gpus(tmp_path, mode):
    """With two ranks the switch's sum a + b equals the rank-order sum, so
    both exchange paths must match one GPU bit for bit."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    from tinygs_b200 import runtime as rt

    mp.start_processes(_worker, args=(_free_port(), str(tmp_path), mode), nprocs=2, start_method="spawn")
    r0, r1 = (np.load(tmp_path / f"rank{k}.npz") for k in range(2))
    # one GPU: Adam twice over g0 + g1 (summed in rank order)
    g0, g1 = _arrays(100, N, 1e-2), _arrays(101, N, 1e-2)
    p = rt.GaussianSet.from_numpy(_arrays(1, N, 1.0), 3)
    g = rt.GaussianSet.from_numpy({k: g0[k] + g1[k] for k in g0}, 3)
    opt = rt.SimpleAdam(p, g, rt.AdamParams(max_grad_1=0.3))
    for _ in range(2):
        opt.step(1.0 / (10.0 * 2))
    ref = p.to_numpy()
    for k in ref:
        np.testing.assert_array_equal(r0[k], ref[k])
        np.testing.assert_array_equal(r1[k], ref[k])
