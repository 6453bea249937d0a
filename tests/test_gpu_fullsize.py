"""Parity with the CPU oracle at the full sizes of the benchmark's
configurations: cfg1 (500k Gaussians, SH3, fp32, 1280 x 720) and cfg2 (3M
Gaussians, SH3, fp16 rasterizer, 1920 x 1080, the configuration of the
headline number).  The 10k- and 20k-Gaussian tests do not reach what only
the full sizes exercise: per-tile lists of ~23.5M instances, ~0.74M
buckets, the super-tile entry sort at 1080p, capacity sizing, 120 x 68
tiles and the fp16 path's 16-bit contributor counts.

Each stage is fed this build's own output of the previous stage, so the
comparison of a stage is exact where its arithmetic is integer:
  * tile counts: exact against the oracle's tile test on this build's own
    screen-space records, outside tests whose final comparison sits on the
    threshold (within 1e-3 relative in fp16, 2e-5 in fp32); against the oracle's records computed from the
    parameters, exact outside the decisions the oracle marks fragile (its
    IEEE fp32 arithmetic against the GPU's fast-math; for the fp16 path a
    band of 4e-3 relative to the threshold, about eight half ulps), with at
    most 1e-5 of the Gaussians differing outside that band in fp16, where
    half-rounded conics one half ulp apart are amplified by the tile test's
    cancellation;
  * instance lists (order included), tile ranges, bucket offsets: exact;
  * images: fp32 within 1e-5 on every pixel; fp16 within 2e-3 except at
    most 1e-4 of the values (the GPU's ex2.approx.f16x2 against the oracle's
    correctly rounded exp2), none beyond 8e-3;
    contributor counts equal except where the transmittance stop moves (at
    most 1e-5 of the pixels in fp32; in fp16 at most 5e-2, the oracle's
    correctly rounded exp2 against the GPU's ex2.approx.f16x2);
  * screen-space and parameter gradients (sh_rest included): within 1e-3
    relative, +1e-4 of the array's maximum for entries near zero.
"""
import numpy as np
import pytest
import torch

from tinygs_b200 import runtime as rt
from tinygs_b200 import scenes

from gpu_helpers import GpuRun, close_rel, scene

pytestmark = pytest.mark.gpu

FP16_BAND = 4e-3


@pytest.mark.parametrize("name,fp16", [("cfg1", False), ("cfg2", True)], ids=["cfg1-fp32", "cfg2-fp16"])
def test_full_size_view_matches_oracle(oracle, cuda_lib, name, fp16):
    cfg, params, sh, cam = scene(name)
    run = GpuRun(params, sh, cam, fp16, max_instances=64_000_000).forward()
    c = run.counts
    assert c.overflow == 0
    gp = run.prims()
    oracle.set_fragile_f16(FP16_BAND)
    try:
        op = oracle.preprocess(params, sh, cam, fp16)
    finally:
        oracle.set_fragile_f16(0)
    # the tile decisions themselves, recomputed by the oracle from this
    # build's own screen-space records: exact except tests whose final
    # fp32 comparison sits within 1e-3 (fp16; 2e-5 fp32) of the threshold,
    # where the GPU's fused multiply-adds, half divisions and fast log move
    # the last bits
    cnt, fr = oracle.count_tiles(gp, cam, fp16, band=1e-3 if fp16 else 2e-5)
    sure = fr == 0
    print(f"{name}: {int((~sure).sum())} of {cfg.n} Gaussians with a tile test on its threshold")
    assert (~sure).mean() < 1e-2
    np.testing.assert_array_equal(gp["n_touched"][sure], cnt[sure])
    # from the parameters: the oracle's IEEE records and the GPU's fast-math
    # ones differ in the last bits, so decisions near a threshold are fragile
    stable = op["fragile"] == 0
    diff = stable & (gp["n_touched"] != op["n_touched"])
    print(f"{name}: {int((~stable).sum())} fragile of {cfg.n}, {int(diff.sum())} stable mismatches")
    assert (~stable).mean() < (5e-2 if fp16 else 1e-3)
    assert diff.sum() <= (1e-5 * cfg.n if fp16 else 0), int(diff.sum())

    # binning of this build's records (with the oracle's own tile counts),
    # order included; instances of Gaussians with a test on its threshold
    # are left out on both sides
    ob = oracle.binning(dict(gp, n_touched=cnt), cam, fp16)
    gb = run.bins()
    keep_g = sure[gb["inst_prim"]]
    keep_o = sure[ob["inst_prim"]]
    np.testing.assert_array_equal(gb["inst_tile"][keep_g], ob["inst_tile"][keep_o])
    np.testing.assert_array_equal(gb["inst_prim"][keep_g], ob["inst_prim"][keep_o])
    gw = (run.W + 15) // 16
    clean = np.ones(gb["ranges"].shape[0], bool)
    clean[gb["inst_tile"][~keep_g].astype(np.int64)] = False
    np.testing.assert_array_equal(gb["ranges"][clean, 1] - gb["ranges"][clean, 0],
                                  ob["ranges"][clean, 1] - ob["ranges"][clean, 0])
    if sure.all():
        np.testing.assert_array_equal(gb["ranges"], ob["ranges"])
        np.testing.assert_array_equal(gb["bucket_offsets"], ob["bucket_offsets"])

    # blending of this build's records and lists
    fs = run.fwd_state()
    ob = gb
    of = oracle.blend_forward(gp, ob, cam, fp16)
    err = np.abs(fs["image"].astype(np.float64) - of["image"].astype(np.float64))
    if fp16:
        # the GPU's ex2.approx.f16x2 against the oracle's correctly rounded
        # exp2 (one half ulp apart at most) shifts a few pixels by a few
        # half ulps; against the reference's own kernels every pixel is
        # within 2e-3 (test_gpu_reference)
        print(f"{name}: {int((err > 2e-3).sum())} of {err.size} values beyond 2e-3, max {err.max():.2e}")
        assert (err > 2e-3).mean() <= 1e-4 and err.max() <= 8e-3, (int((err > 2e-3).sum()), err.max())
    else:
        assert err.max() <= 1e-5, err.max()
    # contributor counts: the stop at T < 1e-4 depends on the exponential
    # (the GPU's ex2.approx / __expf against the oracle's libm), which moves
    # it for a few pixels whose transmittance lands on the threshold
    moved = fs["n_contrib"].astype(np.int64) != of["n_contrib"].astype(np.int64)
    print(f"{name}: contributor counts differ at {int(moved.sum())} of {moved.size} pixels")
    # (in fp16 the oracle's correctly rounded exp2 differs from the GPU's
    # ex2.approx.f16x2 by one half ulp often enough to move the stop of ~3%
    # of the pixels; against the reference's own kernels at most 1e-4 of
    # the pixels differ, test_gpu_reference)
    assert moved.mean() <= (5e-2 if fp16 else 1e-5), int(moved.sum())

    # backward of the loss gradient
    W, H = run.W, run.H
    tgt = torch.from_numpy(scenes.target_image(W, H, 77).reshape(-1)).to(run.dt).cuda()
    lo, go = torch.zeros_like(run.image), torch.zeros_like(run.image)
    loss = rt.FusedLoss(W, H)
    loss.evaluate(run.image, tgt, lo, go, W, H, grad_scaler=10.0)
    torch.cuda.synchronize()
    loss.close()
    gimg = go.float().cpu().numpy()
    run.backward(gimg)
    # the oracle's backward starts from this build's forward state
    # (checkpoints, contributor counts), so that it restarts every bucket
    # where the GPU's backward does
    screen = oracle.blend_backward(gp, ob, fs, go.cpu().numpy(), cam, fp16)
    hp = run.helpers()
    for k in ("grad_mean2d", "grad_conic", "grad_color", "grad_opacity"):
        ok, worst, nbad = close_rel(hp[k], screen[k], 1e-3, 1e-4)
        assert ok, (k, worst, nbad)
    grads = oracle.preprocess_backward(params, sh, cam, gp["n_touched"], screen)
    ours = run.grads_np()
    for k in grads:
        ok, worst, nbad = close_rel(ours[k], grads[k].reshape(ours[k].shape), 1e-3, 1e-4)
        assert ok, (k, worst, nbad)
    run.rast.close()
