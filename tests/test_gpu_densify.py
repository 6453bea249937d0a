"""Densification on the GPU (tgs_densify_step) against the oracle: the same
decisions, order and random split offsets, in place within the arrays'
capacity."""
import ctypes

import numpy as np
import pytest
import torch

from densify_cases import WIDTHS, make_case
from tinygs_b200 import _abi
from tinygs_b200 import runtime as rt

pytestmark = pytest.mark.gpu


def _gpu_sets(params, m, v, grads, cap):
    P = rt.GaussianSet.from_numpy(params, 3, capacity=cap)
    M = rt.GaussianSet.from_numpy(m, 3, capacity=cap)
    V = rt.GaussianSet.from_numpy(v, 3, capacity=cap)
    G = rt.GaussianSet.from_numpy(grads, 3, capacity=cap)
    return P, M, V, G


def _run_gpu(params, m, v, grads, dens, cap, cfg: rt.DensifyParams, step, width=1280, height=720):
    lib = _abi.load_library()
    P, M, V, G = _gpu_sets(params, m, v, grads, cap)
    d = torch.zeros((cap, 4), dtype=torch.float32, device="cuda")
    d[: dens.shape[0]] = torch.from_numpy(dens).cuda()
    h = ctypes.c_void_p()
    _abi.check(lib.tgs_densify_create(cap, ctypes.byref(h)), "create")
    rng = _abi.TgsPcg32()
    lib.tgs_pcg32_seed(ctypes.byref(rng), cfg.seed, 1)
    c = cfg.abi(1.0, 10.0, width, height)
    n = ctypes.c_int64(params["means"].shape[0])
    p, g, mm, vv = P.abi(), G.abi(), M.abi(), V.abi()
    st = lib.tgs_densify_step(h, ctypes.byref(p), ctypes.byref(g), ctypes.byref(mm), ctypes.byref(vv),
                              d.data_ptr(), ctypes.byref(c), step, ctypes.byref(rng), ctypes.byref(n), None)
    torch.cuda.synchronize()
    lib.tgs_densify_destroy(h)
    for s in (P, M, V, G):
        s.resize(max(n.value, 0))
    return st, n.value, P, M, V, G, d.cpu().numpy(), (rng.state, rng.inc)


def _run_oracle(oracle, params, m, v, grads, dens, cap, cfg: rt.DensifyParams, step, width=1280, height=720):
    P, M = oracle.alloc_set(cap, params), oracle.alloc_set(cap, m)
    V, G = oracle.alloc_set(cap, v), oracle.alloc_set(cap, grads)
    d = np.zeros((cap, 4), np.float32)
    d[: dens.shape[0]] = dens
    oc = oracle.densify_config(duplicate_grad_threshold=cfg.duplicate_grad_threshold,
                               duplicate_scale_threshold=cfg.duplicate_scale_threshold,
                               pruning_opacity_threshold=cfg.pruning_opacity_threshold,
                               pruning_scale_threshold=cfg.pruning_scale_threshold,
                               max_screen_size=cfg.max_screen_size, refine_every=cfg.refine_every,
                               start_refine=cfg.start_refine, end_refine=cfg.end_refine, reset_every=cfg.reset_every,
                               image_width=width, image_height=height, max_num_gaussians=cfg.max_num_gaussians)
    rng = oracle.pcg32(cfg.seed, 1)
    n = oracle.densify_step(params["means"].shape[0], P, G, M, V, d, oc, step, rng)
    return n, P, M, V, G, d, (rng.state, rng.inc)


def _np(s: rt.GaussianSet, k):
    return s.views[k].detach().cpu().numpy()


def test_refine_matches_oracle(oracle):
    n, cap = 20000, 40000
    params, (m, v), grads, dens = make_case(n, seed=21)
    cfg = rt.DensifyParams(max_screen_size=100.0 / 1280.0, reset_every=500)
    st, gn, P, M, V, G, gd, grng = _run_gpu(params, m, v, grads, dens, cap, cfg, 600)
    assert st == 0
    on, oP, oM, oV, oG, od, orng = _run_oracle(oracle, params, m, v, grads, dens, cap, cfg, 600)
    assert gn == on and gn != n
    assert grng == orng  # the generator moved by the same number of draws
    # copies, the compaction and zeroed rows are exact; the split rows carry
    # exp / log / sqrt of the fast-math build (the logistic noise amplifies a
    # last-bit difference of log near u = 0 or 1)
    for k in ("rotations", "sh0", "sh_rest"):
        np.testing.assert_array_equal(_np(P, k), oP[k][:on])
    for k in ("means", "scales", "opacities"):
        np.testing.assert_allclose(_np(P, k), oP[k][:on], rtol=1e-4, atol=1e-5)
    for S, O in ((M, oM), (V, oV), (G, oG)):
        for k in WIDTHS:
            np.testing.assert_array_equal(_np(S, k), O[k][:on])
    assert not gd[:gn].any()


def test_opacity_reset_matches_oracle(oracle):
    n = 5000
    params, (m, v), grads, dens = make_case(n, seed=22)
    cfg = rt.DensifyParams(refine_every=300, reset_every=500)
    st, gn, P, M, V, G, gd, _ = _run_gpu(params, m, v, grads, dens, n, cfg, 1000)
    assert st == 0 and gn == n
    on, oP, oM, oV, oG, od, _ = _run_oracle(oracle, params, m, v, grads, dens, n, cfg, 1000)
    np.testing.assert_allclose(_np(P, "opacities"), oP["opacities"][:n], rtol=2e-5, atol=2e-6)
    assert not _np(M, "opacities").any() and not _np(V, "opacities").any()
    np.testing.assert_array_equal(_np(M, "means"), m["means"])
    np.testing.assert_array_equal(gd[:n], dens)  # no refine: statistics kept


def test_growth_past_capacity_is_refused():
    n = 3000
    params, (m, v), grads, dens = make_case(n, seed=23)
    cfg = rt.DensifyParams()
    st, gn, P, M, V, G, gd, _ = _run_gpu(params, m, v, grads, dens, n, cfg, 500)
    assert st == _abi.TGS_ERR_CAPACITY and gn == n
    for k in WIDTHS:
        np.testing.assert_array_equal(_np(P, k), np.asarray(params[k], np.float32).reshape(n, -1))


def test_training_loop_with_densification():
    """Forward / loss / backward / Adam / densify for a few steps on a small
    scene: the rasterizer follows the changing Gaussian count."""
    from tinygs_b200 import scenes

    cfg0 = scenes.CONFIGS["cfg0"]
    n0, cap = 3000, 12000
    params = scenes.gaussian_params(n0, 0, cfg0.means, 5)
    cam = scenes.cameras(cfg0)[0]
    W, H = cam["width"], cam["height"]
    g = rt.GaussianSet.from_numpy(params, 0, capacity=cap)
    grads = g.zeros_like()
    opt = rt.SimpleAdam(g, grads, rt.AdamParams(max_grad_1=0.3))
    dens = rt.Densifier(g, grads, opt, rt.DensifyParams(refine_every=2, start_refine=2, end_refine=20,
                                                        duplicate_grad_threshold=1e-6, reset_every=1000))
    rast = rt.FastGSB200Rasterizer(cap, W, H)
    rast.set_gaussians(g)
    img = torch.zeros(rt.image_numel(W, H), device="cuda")
    gimg, lmap = torch.zeros_like(img), torch.zeros_like(img)
    tgt = torch.from_numpy(scenes.target_image(W, H, 3).reshape(-1)).cuda()
    loss = rt.FusedLoss(W, H)
    counts = []
    for step in range(6):
        ctx = rt.RasterizeContext(fwd_input=cam, fwd_output_image=img, grad_output_image=gimg, gaussians_grad=grads,
                                  grad_scaler=10.0, densification_info=dens.densification_info)
        gimg.zero_()
        lmap.zero_()
        rast.set_gaussians(g)
        rast.forward(ctx)
        loss.evaluate(img, tgt, lmap, gimg, W, H, grad_scaler=10.0)
        ctx.accumulate = False
        rast.backward(ctx)
        opt.step(0.1)
        counts.append(dens.step(ctx))
        torch.cuda.synchronize()
        assert torch.isfinite(img).all()
    assert counts[0] == counts[1] == n0  # strategy steps 0 and 1 do not refine
    assert counts[2] != n0  # the refine at strategy step 2 changed the count
    assert all(0 < c <= cap for c in counts)
