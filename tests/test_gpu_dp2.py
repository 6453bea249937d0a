"""The data-parallel optimizer steps on two GPUs: over peer memory
(tgs_dp_reduce_adam, tinygs_b200.dp.PeerAdam) and through NVLink SHARP
(tgs_dp_reduce_adam_multicast, MulticastAdam) every rank ends with exactly
the parameters that one GPU gets from Adam over the sum of both ranks'
gradients (the reference's accumulation of two views); a whole routed
training step (tgs_raster_backward_routed + tgs_dp_inbox_adam, InboxAdam)
against one GPU accumulating the same two views.  Needs two GPUs; skipped
otherwise."""
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


def _train_worker(rank: int, port: int, out_dir: str) -> None:
    """One routed training step per rank (rank r renders view r)."""
    import torch.distributed as dist

    from tinygs_b200 import dp as dpm
    from tinygs_b200 import runtime as rt
    from tinygs_b200 import scenes

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        dp = dpm.DataParallel.from_env()
        cfg = scenes.CONFIGS["cfg1"]
        n = 20_001
        params = scenes.gaussian_params(n, cfg.sh_degree, cfg.means, 9)
        cam = scenes.cameras(cfg)[dp.view_index(0, len(scenes.cameras(cfg)))]
        W, H = cam["width"], cam["height"]
        g = dpm.shared_gaussian_set(n, cfg.sh_degree)
        g.copy_from_numpy(params)
        opt = dpm.InboxAdam(dp, g, rt.AdamParams(max_grad_1=0.3))
        rast = rt.FastGSB200Rasterizer(n, W, H)
        rast.set_gaussians(g)
        img = torch.zeros(rt.image_numel(W, H), device="cuda")
        gimg, lmap = torch.zeros_like(img), torch.zeros_like(img)
        tgt = torch.from_numpy(scenes.target_image(W, H, 3).reshape(-1)).cuda()
        loss = rt.FusedLoss(W, H)
        ctx = rt.RasterizeContext(fwd_input=cam, fwd_output_image=img, grad_output_image=gimg, grad_scaler=10.0)
        rast.forward(ctx)
        loss.evaluate(img, tgt, lmap, gimg, W, H, grad_scaler=10.0)
        rast.backward_routed(ctx, *opt.route())
        opt.step(dp.gradient_scale(10.0))
        torch.cuda.synchronize()
        np.savez(os.path.join(out_dir, f"train{rank}.npz"), **g.to_numpy())
        opt.barrier()
        opt.close()
        rast.close()
        loss.close()
    finally:
        dist.destroy_process_group()


def test_routed_training_step_two_gpus(tmp_path):
    """Both ranks end with identical parameters (every slice broadcast by its
    owner), equal to one GPU accumulating the two views' gradients and
    stepping once, up to float-atomic order noise of the blend backward."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    from tinygs_b200 import runtime as rt
    from tinygs_b200 import scenes

    mp.start_processes(_train_worker, args=(_free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    r0, r1 = (np.load(tmp_path / f"train{k}.npz") for k in range(2))
    for k in r0.files:
        np.testing.assert_array_equal(r0[k], r1[k])
    # one GPU: views 0 and 1 accumulated, one Adam step at scale 1/(10*2)
    cfg = scenes.CONFIGS["cfg1"]
    n = 20_001
    params = scenes.gaussian_params(n, cfg.sh_degree, cfg.means, 9)
    cams = scenes.cameras(cfg)
    g = rt.GaussianSet.from_numpy(params, cfg.sh_degree)
    grads = g.zeros_like()
    opt = rt.SimpleAdam(g, grads, rt.AdamParams(max_grad_1=0.3))
    for v in range(2):
        cam = cams[v]
        W, H = cam["width"], cam["height"]
        rast = rt.FastGSB200Rasterizer(n, W, H)
        rast.set_gaussians(g)
        img = torch.zeros(rt.image_numel(W, H), device="cuda")
        gimg, lmap = torch.zeros_like(img), torch.zeros_like(img)
        tgt = torch.from_numpy(scenes.target_image(W, H, 3).reshape(-1)).cuda()
        loss = rt.FusedLoss(W, H)
        ctx = rt.RasterizeContext(fwd_input=cam, fwd_output_image=img, grad_output_image=gimg,
                                  gaussians_grad=grads, grad_scaler=10.0, accumulate=True)
        rast.forward(ctx)
        loss.evaluate(img, tgt, lmap, gimg, W, H, grad_scaler=10.0)
        rast.backward(ctx)
        rast.close()
        loss.close()
    opt.step(1.0 / (10.0 * 2))
    ref = g.to_numpy()
    for k in ref:
        close = np.abs(r0[k] - ref[k]) <= 1e-6 + 1e-5 * np.abs(ref[k])
        assert close.mean() > 0.999, (k, close.mean())


def _owner_worker(rank: int, port: int, out_dir: str, dtype_name: str) -> None:
    """Two owner-split training steps per rank (rank r renders view 2s + r)."""
    import torch.distributed as dist

    from tinygs_b200 import dp as dpm
    from tinygs_b200 import runtime as rt
    from tinygs_b200 import scenes

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        dp = dpm.DataParallel.from_env()
        cfg = scenes.CONFIGS["cfg1"]
        n = 20_001
        params = scenes.gaussian_params(n, cfg.sh_degree, cfg.means, 9)
        cams = scenes.cameras(cfg)
        W, H = cams[0]["width"], cams[0]["height"]
        fp16 = dtype_name == "fp16"
        dt = torch.float16 if fp16 else torch.float32
        g = rt.GaussianSet.from_numpy(params, cfg.sh_degree)
        rast = rt.FastGSB200Rasterizer(n, W, H)
        rast.set_gaussians(g)
        opt = dpm.OwnerSplit(dp, rast, g, rt.AdamParams(max_grad_1=0.3),
                             rt._abi.TGS_FLOAT16 if fp16 else rt._abi.TGS_FLOAT32)
        img = torch.zeros(rt.image_numel(W, H), dtype=dt, device="cuda")
        gimg, lmap = torch.zeros_like(img), torch.zeros_like(img)
        loss = rt.FusedLoss(W, H)
        loss.set_accumulate(False)  # each evaluation overwrites the loss map and gradient image
        images = []
        for s in range(2):
            views = [cams[2 * s + r] for r in range(2)]
            tgt = torch.from_numpy(scenes.target_image(W, H, 3 + 2 * s + rank).reshape(-1)).to(dt).cuda()
            opt.forward(views, img)
            loss.evaluate(img, tgt, lmap, gimg, W, H, grad_scaler=10.0)
            opt.backward_adam(views, img, gimg, dp.gradient_scale(10.0))
            images.append(img.float().cpu().numpy())
        torch.cuda.synchronize()
        out = {k: v[opt.first:opt.last] for k, v in g.to_numpy().items()}
        np.savez(os.path.join(out_dir, f"owner{rank}.npz"), first=opt.first, last=opt.last, img0=images[0],
                 img1=images[1], **out)
        opt.barrier()
        opt.close()
        dist.barrier()
        rast.close()
        loss.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dtype_name", ["fp32", "fp16"])
def test_owner_split_two_gpus(tmp_path, dtype_name):
    """Each rank's slice after two owner-split steps equals one GPU
    accumulating the same two views per step and stepping Adam, up to the
    float-atomic order noise of the blend backward; the first step's images
    are those of one GPU rendering the view."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    from tinygs_b200 import runtime as rt
    from tinygs_b200 import scenes

    mp.start_processes(_owner_worker, args=(_free_port(), str(tmp_path), dtype_name), nprocs=2,
                       start_method="spawn")
    rk = [np.load(tmp_path / f"owner{k}.npz") for k in range(2)]
    assert int(rk[0]["first"]) == 0 and int(rk[0]["last"]) == int(rk[1]["first"])
    cfg = scenes.CONFIGS["cfg1"]
    n = 20_001
    assert int(rk[1]["last"]) == n
    params = scenes.gaussian_params(n, cfg.sh_degree, cfg.means, 9)
    cams = scenes.cameras(cfg)
    W, H = cams[0]["width"], cams[0]["height"]
    fp16 = dtype_name == "fp16"
    dt = torch.float16 if fp16 else torch.float32
    g = rt.GaussianSet.from_numpy(params, cfg.sh_degree)
    grads = g.zeros_like()
    opt = rt.SimpleAdam(g, grads, rt.AdamParams(max_grad_1=0.3))
    rast = rt.FastGSB200Rasterizer(n, W, H)
    rast.set_gaussians(g)
    loss = rt.FusedLoss(W, H)
    loss.set_accumulate(False)
    img = torch.zeros(rt.image_numel(W, H), dtype=dt, device="cuda")
    gimg, lmap = torch.zeros_like(img), torch.zeros_like(img)
    for s in range(2):
        for r in range(2):
            ctx = rt.RasterizeContext(fwd_input=cams[2 * s + r], fwd_output_image=img, grad_output_image=gimg,
                                      gaussians_grad=grads, grad_scaler=10.0, accumulate=r > 0)
            rast.forward(ctx)
            if s == 0:
                np.testing.assert_array_equal(rk[r]["img0"], img.float().cpu().numpy())
            tgt = torch.from_numpy(scenes.target_image(W, H, 3 + 2 * s + r).reshape(-1)).to(dt).cuda()
            loss.evaluate(img, tgt, lmap, gimg, W, H, grad_scaler=10.0)
            rast.backward(ctx)
        opt.step(1.0 / (10.0 * 2))
    ref = g.to_numpy()
    rast.close()
    loss.close()
    for k in ref:
        got = np.concatenate([rk[0][k], rk[1][k]])
        close = np.abs(got - ref[k]) <= 1e-6 + 1e-5 * np.abs(ref[k])
        assert close.mean() > 0.999, (k, close.mean())
