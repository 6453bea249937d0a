"""Row operations on Gaussian sets and the Morton reorder, through the C ABI
(tgs_arena_gather / _compact / _keep_index / _fill_rows, tgs_dens_gather,
tgs_morton_order), against the CPU oracle and numpy.

Reference behaviour: GPUGaussian3d::reorder / remove / append
(tinygs/src/core/gpu_gaussian.cu:117-171, 273-311), SimpleAdam::remove /
duplicate / reset / reset_opacity / reorder (simple_adam.cu:841-1099) and
Orchestrator::reorder_gaussians (orchestrator.cu:26-100, 1038-1060).  The
Morton permutation is bit-exact: the codes are integer functions of IEEE
float operations and the sort is stable."""
import numpy as np
import pytest
import torch

from tinygs_b200 import runtime as rt
from tinygs_b200 import scenes

from gpu_helpers import GpuRun, scene

pytestmark = pytest.mark.gpu


def _set(n, seed, sh=3):
    params = scenes.gaussian_params(n, sh, "normal", seed)
    return params, rt.GaussianSet.from_numpy(params, sh)


# 4096 / 4097 / 12288: whole 2048-item sort tiles, one item past them, six tiles
@pytest.mark.parametrize("n", [1, 1000, 4096, 4097, 12288, 1_000_003])
def test_morton_order_matches_oracle(oracle, cuda_lib, n):
    params, g = _set(n, 11)
    perm = rt.morton_order(g).cpu().numpy().view(np.uint32)
    np.testing.assert_array_equal(perm, oracle.morton_order(params["means"]))


def test_morton_order_degenerate_means(oracle, cuda_lib):
    params, _ = _set(5000, 12)
    params["means"][:, 1] = 0.5          # flat axis: extent clamped to 1e-8
    params["means"][1000:3000] = params["means"][1000]  # many equal codes
    g = rt.GaussianSet.from_numpy(params, 3)
    perm = rt.morton_order(g).cpu().numpy().view(np.uint32)
    np.testing.assert_array_equal(perm, oracle.morton_order(params["means"]))
    g.resize(0)
    assert rt.morton_order(g).numel() == 0


def test_gather_compact_fill_match_numpy(cuda_lib):
    n = 100_003
    params, g = _set(n, 13)
    rng = np.random.default_rng(5)
    idx = rng.permutation(n).astype(np.int32)
    g.reorder(torch.from_numpy(idx).cuda())
    out = g.to_numpy()
    for k, v in params.items():
        np.testing.assert_array_equal(out[k], v.reshape(out[k].shape)[idx], err_msg=k)
    keep = rng.random(n) < 0.37
    kept = g.remove(torch.from_numpy(keep.astype(np.uint8)).cuda())
    assert kept == int(keep.sum()) and g.n == kept
    out2 = g.to_numpy()
    for k in params:
        np.testing.assert_array_equal(out2[k], out[k][keep], err_msg=k)
    rows = np.unique(rng.integers(0, kept, 500)).astype(np.int32)
    g.fill_rows(torch.from_numpy(rows).cuda(), 0.0, -1)
    out3 = g.to_numpy()
    for k in params:
        want = out2[k].copy()
        want[rows] = 0
        np.testing.assert_array_equal(out3[k], want, err_msg=k)
    g.fill_rows(torch.from_numpy(rows).cuda(), 7.0, 1)  # opacities only
    assert np.all(g.to_numpy()["opacities"][rows] == 7.0)
    np.testing.assert_array_equal(g.to_numpy()["means"], out3["means"])
    # nothing kept, everything kept
    assert g.remove(torch.zeros(g.n, dtype=torch.uint8, device="cuda")) == 0
    params, g = _set(999, 14)
    assert g.remove(torch.ones(999, dtype=torch.uint8, device="cuda")) == 999
    for k, v in g.to_numpy().items():
        np.testing.assert_array_equal(v, params[k].reshape(v.shape))


def test_optimizer_row_hooks(cuda_lib):
    n = 4096
    params, g = _set(n, 15)
    grads = g.zeros_like()
    opt = rt.SimpleAdam(g, grads, rt.AdamParams(max_grad_1=0.3))
    grads.storage.normal_()
    opt.step(0.1)
    m0, v0 = opt.exp_avg.to_numpy(), opt.exp_avg_sq.to_numpy()
    rng = np.random.default_rng(6)
    keep = rng.random(n) < 0.5
    kt = torch.from_numpy(keep.astype(np.uint8)).cuda()
    assert opt.remove(kt) == int(keep.sum())
    for k in m0:
        np.testing.assert_array_equal(opt.exp_avg.to_numpy()[k], m0[k][keep])
        np.testing.assert_array_equal(opt.exp_avg_sq.to_numpy()[k], v0[k][keep])
    kept = int(keep.sum())
    opt.duplicate(None, None, 10)  # new rows start at zero
    assert opt.exp_avg.n == kept + 10
    for k, v in opt.exp_avg.to_numpy().items():
        assert np.all(v[kept:] == 0), k
    opt.exp_avg.resize(kept), opt.exp_avg_sq.resize(kept)
    g.resize(kept)
    opt.reset_opacity()
    assert np.all(opt.exp_avg.to_numpy()["opacities"] == 0) and np.all(opt.exp_avg_sq.to_numpy()["opacities"] == 0)
    assert np.any(opt.exp_avg.to_numpy()["means"] != 0)


def test_reorder_gaussians_keeps_the_render(cuda_lib):
    """Orchestrator::reorder_gaussians moves rows only: the image is the same
    after the Morton reorder, and the densification records follow their
    Gaussians."""
    cfg, params, sh, cam = scene("cfg1", n=50_000)
    run = GpuRun(params, sh, cam, False).forward()
    before = run.image.clone()
    dens = torch.rand(run.n, 4, device="cuda")
    dens0 = dens.clone()
    perm = rt.reorder_gaussians(run.g, run.grads, None, dens)
    p = perm.long()
    np.testing.assert_array_equal(dens.cpu().numpy(), dens0[p].cpu().numpy())
    np.testing.assert_array_equal(run.g.to_numpy()["means"], params["means"][p.cpu().numpy()])
    run.forward()
    np.testing.assert_allclose(run.image.cpu().numpy(), before.cpu().numpy(), rtol=0, atol=1e-6)
