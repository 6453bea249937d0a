"""The owner-split data-parallel step emulated on ONE GPU: N rasterizer
handles stand for N ranks (their arenas all local), one shared parameter /
moment arena of which each emulated owner touches only its slice.  Two steps
must equal the reference's accumulate_grad_steps = N on one GPU
(orchestrator.cu:343-403: N views rendered in turn, their gradients added in
view order, one Adam step with gradient scale 1/(grad_scaler * N)):
  * every view's image bit-identical to a plain forward of that view (the
    forward is deterministic and the gathered records are the same bytes);
  * the densification records' radii (maximum over the views) and counters
    identical;
  * the parameters after Adam equal up to the float-atomic order of the blend
    backward (which Adam's per-coordinate normalisation can amplify only for
    gradients at that noise level)."""
import numpy as np
import pytest
import torch

from tinygs_b200 import dp as dpm
from tinygs_b200 import runtime as rt
from tinygs_b200 import scenes

from gpu_helpers import scene

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("fp16", [False, True], ids=["fp32", "fp16"])
def test_owner_split_step_equals_accumulated_views(cuda_lib, world, fp16):
    cfg, params, sh, _ = scene("cfg1", n=60_001)
    all_cams = scenes.cameras(cfg)
    W, H = cfg.width, cfg.height
    n = params["means"].shape[0]
    dt = torch.float16 if fp16 else torch.float32
    dtype = rt._abi.TGS_FLOAT16 if fp16 else rt._abi.TGS_FLOAT32
    acfg = rt.AdamParams(max_grad_1=0.3)
    scale = 1.0 / (10.0 * world)
    steps = 2
    targets = [torch.from_numpy(scenes.target_image(W, H, 500 + v).reshape(-1)).to(dt).cuda()
               for v in range(world * steps)]
    numel = rt.image_numel(W, H)
    loss = rt.FusedLoss(W, H)
    loss.set_accumulate(False)  # every evaluation overwrites the loss map and gradient image

    def views(s):
        return all_cams[s * world:(s + 1) * world]

    # reference: one GPU, per step the N views accumulated, one Adam step
    g_ref = rt.GaussianSet.from_numpy(params, sh)
    grads_ref = g_ref.zeros_like()
    opt_ref = rt.SimpleAdam(g_ref, grads_ref, acfg)
    dens_ref = torch.zeros(n, 4, device="cuda")
    rast_ref = rt.FastGSB200Rasterizer(n, W, H)
    rast_ref.set_gaussians(g_ref)
    ref_images = []
    for s in range(steps):
        for v, cam in enumerate(views(s)):
            img, gimg, lmap = (torch.zeros(numel, dtype=dt, device="cuda") for _ in range(3))
            ctx = rt.RasterizeContext(fwd_input=cam, fwd_output_image=img, grad_output_image=gimg,
                                      gaussians_grad=grads_ref, densification_info=dens_ref, accumulate=v > 0)
            rast_ref.forward(ctx)
            loss.evaluate(img, targets[s * world + v], lmap, gimg, W, H, grad_scaler=10.0)
            rast_ref.backward(ctx)
            if s == 0:
                ref_images.append(img)
        opt_ref.step(scale)

    # N emulated owners on this GPU
    g = rt.GaussianSet.from_numpy(params, sh)
    rasts = [rt.FastGSB200Rasterizer(n, W, H) for _ in range(world)]
    arenas = [r.arena() for r in rasts]
    for r, ra in enumerate(rasts):
        ra.attach_views(arenas, r)
    m, v_ = g.zeros_like(), g.zeros_like()
    dens = torch.zeros(n, 4, device="cuda")
    slices = [dpm.owner_slice(n, world, r) for r in range(world)]
    assert slices[0][0] == 0 and slices[-1][1] == n and all(a % 256 == 0 for a, _ in slices)
    images = []
    img, gimg, lmap = (torch.zeros(numel, dtype=dt, device="cuda") for _ in range(3))
    for s in range(steps):
        cams = views(s)
        for r, ra in enumerate(rasts):
            ra.preprocess_views(g, cams, dtype, *slices[r], dens)
        for r, ra in enumerate(rasts):
            out = torch.zeros(numel, dtype=dt, device="cuda")
            ra.forward_gathered(n, cams[r], out)
            loss.evaluate(out, targets[s * world + r], lmap, gimg, W, H, grad_scaler=10.0)
            ra.backward_screen(cams[r], out, gimg)
            if s == 0:
                images.append(out)
        for r, ra in enumerate(rasts):
            ra.backward_views_adam(g, cams, *slices[r], None, m, v_, acfg, s + 1, scale, dens)
    torch.cuda.synchronize()

    for v in range(world):
        assert torch.equal(images[v], ref_images[v]), v
    # densification records over both steps; the second step's forward sees
    # parameters that already differ at the noise level, so a decision on a
    # tile boundary may flip for a handful of Gaussians
    d, dr = dens.cpu().numpy(), dens_ref.cpu().numpy()
    got, want = g.to_numpy(), g_ref.to_numpy()
    fr = {"count": (d[:, 0] == dr[:, 0]).mean(),
          "radius": (np.abs(d[:, 3] - dr[:, 3]) <= 1e-5 * np.abs(dr[:, 3])).mean(),
          "grad": (np.abs(d[:, 1] - dr[:, 1]) <= 1e-9 + 1e-4 * np.abs(dr[:, 1])).mean(),
          "grad3": (np.abs(d[:, 1] - dr[:, 1]) <= 1e-9 + 1e-3 * np.abs(dr[:, 1])).mean()}
    for k in want:
        a, b = got[k].ravel(), want[k].ravel()
        fr[k] = (np.abs(a - b) <= 1e-6 + 1e-5 * np.abs(b)).mean()
        fr[k + "_max"] = float(np.abs(a - b).max())
    # the fp16 rasterizer's half-precision intermediates turn the step-1
    # noise in the parameters into rounding flips for a few Gaussians more
    # (measured: 99.82 % of the gradient statistics within 1e-4, 99.98 %
    # within 1e-3; opacities 99.90 % within the parameter bound)
    assert fr["count"] > 0.9999  # views in which a Gaussian touched a tile
    assert fr["radius"] > 0.999  # max screen radius
    assert fr["grad3" if fp16 else "grad"] > 0.999
    for k in want:
        assert fr[k] > (0.998 if fp16 else 0.999), (k, fr[k])
        assert fr[k + "_max"] <= 2.5e-2, k
    for ra in rasts:
        ra.close()
    rast_ref.close()
    loss.close()
