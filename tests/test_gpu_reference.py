"""The CUDA path against the reference's OWN kernels on identical inputs.

oracle/_ref/libtgs_ref.so is Adversarr/tinygs's fastgs_ours (fp32) and
fastgs_ours_fp16 rasterizers plus its L1 and fused-SSIM losses, compiled
unchanged from their sources (oracle/build_ref.py) and driven through their
own raw entry points.  Both run on the same device arrays, so any difference
is a difference of the kernels.

What is compared, and how tightly:
  * tile counts per Gaussian: bit-exact.  The two builds are both fast-math
    and round the 2D conic differently in the last bits for a share of the
    Gaussians (FMA contraction and reciprocal choices differ between the two
    kernels); a tile decision that sits on its threshold can flip.  None
    flips at 10k-50k Gaussians; at 3M (cfg2) a handful do, each by one tile,
    and the budget below is 1e-5 of the Gaussians.
  * instance lists, tile ranges, bucket offsets: bit-exact on every tile no
    flipped Gaussian touches, with the reference's equal-depth ties (ordered
    by atomic arrival, fastgs_ours/kernels_forward.cuh:407-410) put in index
    order, the deterministic order of this build.
  * images: fp16 within 2e-3 on every pixel; fp32 within 1e-5 outside the
    tiles of a flip or of a depth tie, with at most 1e-5 of those pixels
    above it (conic last-bit differences moving an alpha across 1/255) and
    none above 4e-3 (one Gaussian's contribution at that threshold).
  * per-pixel contributor counts: exact outside flipped / tied tiles (fp16:
    at most 1e-4 of the pixels, where a record one half ulp apart moves the
    transmittance stop).
  * fused L1 + SSIM against the reference's L1Loss then FusedSSIMLoss:
    loss map and gradient image within a few ulps of their largest entry
    (fp16: one half ulp of it, at least two ulps of the smallest subnormal).
  * backward, fp32 path: every parameter gradient (sh_rest included) within
    1e-3 relative (+1e-4 of the array's maximum for entries near zero), for
    Gaussians away from flipped / tied tiles.
  * backward, fp16 path: the reference accumulates in half2 with f16x2
    atomics (fastgs_ours_fp16/kernels_backward.cuh:1359-1387) and is itself
    order dependent; this build evaluates the same formula in fp32.  The
    relative L2 error against the reference must stay within 2e-2 (the
    reference's own run-to-run spread is printed beside it).

The reference's fp32 path itself stops working at 100k Gaussians and above
on B200 (its per-tile instance ranges come out inverted; the harness checks
them before its blend and refuses), so the fp32 comparisons run at <= 50k;
the full-size comparison is cfg2, the fp16 path the benchmark measures.
"""
import numpy as np
import pytest
import torch

from tinygs_b200 import runtime as rt
from tinygs_b200 import scenes

from gpu_helpers import GpuRun, close_rel, scene

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def refpy():
    from oracle import refpy as R

    if not R.available():
        pytest.skip("oracle/_ref/libtgs_ref.so not built (built from the reference sources by oracle/build_ref.py)")
    R.load()
    return R


CASES = [("cfg0", None, False), ("cfg0", None, True), ("cfg1", 20000, False), ("cfg1", 20000, True),
         ("cfg1", 50000, False), ("cfg2", None, True)]
IDS = [f"{c}-{n or 'full'}-{'fp16' if f else 'fp32'}" for c, n, f in CASES]


class Pair:
    """One forward (and backward) of this build and of the reference on the
    same Gaussians, camera and gradient image."""

    def __init__(self, R, name, n, fp16):
        cfg, params, sh, cam = scene(name, n=n)
        self.fp16, self.cam = fp16, cam
        self.run = GpuRun(params, sh, cam, fp16).forward()
        assert self.run.counts.overflow == 0
        self.N, self.W, self.H = self.run.n, self.run.W, self.run.H
        self.gw, self.gh = (self.W + 15) // 16, (self.H + 15) // 16
        self.T = self.gw * self.gh
        self.ref = R.RefRasterizer()
        self.ref_image = torch.zeros_like(self.run.image)
        self.V, self.I, self.B = self.ref.forward(self.run.g, cam, self.ref_image, fp16)
        self.R = R

    def close(self):
        self.ref.close()
        self.run.rast.close()

    # reference state in this build's formats
    def ref_bins(self):
        R, N = self.R, self.N
        keys = self.ref.copy(R.INST_KEYS, np.uint32 if self.fp16 else np.uint16, self.I).astype(np.int64)
        prims = self.ref.copy(R.INST_PRIMS, np.uint32, self.I).astype(np.int64)
        sp = self.ref.copy(R.SORTED_PRIMS, np.uint32, self.V).astype(np.int64)
        sk = self.ref.copy(R.SORTED_DEPTH_KEYS, np.uint32, self.V).astype(np.int64)
        depth = np.zeros(N, np.int64)
        depth[sp] = sk
        # the reference's list is ordered by (tile, depth); equal depths keep
        # their atomic arrival order
        comp = keys * (1 << 33) + depth[prims]
        assert np.all(np.diff(comp) >= 0)
        tie = np.zeros(self.T, bool)
        dup = np.nonzero(np.diff(comp) == 0)[0]
        tie[keys[dup]] = True
        order = np.lexsort((prims, depth[prims], keys))
        return {"tile": keys[order], "prim": prims[order], "tie_tiles": tie,
                "ranges": self.ref.copy(R.TILE_RANGES, np.uint32, 2 * self.T).reshape(self.T, 2),
                "bucket_offsets": self.ref.copy(R.BUCKET_OFFSETS, np.uint32, self.T)}


def _excluded_tiles(p, flipped, ours, refb):
    """Tiles touched by a flipped Gaussian (in either list) or holding a
    depth tie in the reference's list."""
    bad = refb["tie_tiles"].copy()
    if flipped.size:
        f = np.isin(ours["inst_prim"], flipped)
        bad[ours["inst_tile"][f].astype(np.int64)] = True
        f = np.isin(refb["prim"], flipped)
        bad[refb["tile"][f]] = True
    return bad


def _tile_pixels(p, tiles):
    """Mask over the tiled image plane of the pixels of the given 16x16 tiles."""
    tw = (p.W + 7) // 8
    pl = rt.image_numel(p.W, p.H) // 3
    idx = np.arange(pl)
    blk = idx >> 6
    by, bx = blk // tw, blk % tw
    y = by * 8 + ((idx >> 3) & 7)
    x = bx * 8 + (idx & 7)
    t = (y // 16) * p.gw + (x // 16)
    return tiles[np.minimum(t, p.T - 1)] & (y < ((p.H + 7) // 8 * 8)) & (x < ((p.W + 7) // 8 * 8))


@pytest.mark.parametrize("name,n,fp16", CASES, ids=IDS)
def test_forward_matches_reference_kernels(refpy, cuda_lib, name, n, fp16):
    p = Pair(refpy, name, n, fp16)
    try:
        ours_p, ours_b, fs = p.run.prims(), p.run.bins(), p.run.fwd_state()
        rn = p.ref.copy(refpy.N_TOUCHED, np.uint32, p.N)
        flipped = np.nonzero(rn != ours_p["n_touched"])[0]
        budget = 0 if p.N <= 100_000 else int(1e-5 * p.N)
        assert flipped.size <= budget, f"{flipped.size} tile counts differ (budget {budget})"
        assert np.abs(rn[flipped].astype(np.int64) - ours_p["n_touched"][flipped].astype(np.int64)).max(
            initial=0) <= 1
        refb = p.ref_bins()
        bad = _excluded_tiles(p, flipped, ours_b, refb)
        if flipped.size == 0:
            assert p.V == int((ours_p["n_touched"] > 0).sum())
            np.testing.assert_array_equal(ours_b["inst_tile"].astype(np.int64), refb["tile"])
            np.testing.assert_array_equal(ours_b["inst_prim"].astype(np.int64), refb["prim"])
            np.testing.assert_array_equal(ours_b["ranges"], refb["ranges"])
            np.testing.assert_array_equal(ours_b["bucket_offsets"], refb["bucket_offsets"])
        else:
            # per-tile lists equal on every tile no flipped Gaussian touches
            our_cnt = ours_b["ranges"][:, 1].astype(np.int64) - ours_b["ranges"][:, 0]
            ref_cnt = refb["ranges"][:, 1].astype(np.int64) - refb["ranges"][:, 0]
            good = ~bad
            np.testing.assert_array_equal(our_cnt[good], ref_cnt[good])
            ours_keep = good[ours_b["inst_tile"].astype(np.int64)]
            ref_keep = good[refb["tile"]]
            np.testing.assert_array_equal(ours_b["inst_prim"][ours_keep].astype(np.int64), refb["prim"][ref_keep])
        # images
        a = p.run.image.float().cpu().numpy()
        b = p.ref_image.float().cpu().numpy()
        err = np.abs(a - b)
        if fp16:
            assert err.max() <= 2e-3, err.max()
        else:
            skip = np.tile(_tile_pixels(p, bad), 3)
            e = err[~skip]
            assert (e > 1e-5).mean() <= 1e-5, (int((e > 1e-5).sum()), e.max())
            assert e.max() <= 4e-3, e.max()
        pl = rt.image_numel(p.W, p.H) // 3
        rc = p.ref.copy(refpy.N_CONTRIB, np.uint16 if fp16 else np.uint32, pl).astype(np.int64)
        keep = ~_tile_pixels(p, bad)
        moved = fs["n_contrib"].astype(np.int64)[keep] != rc[keep]
        if fp16:
            # a fp16 record one half ulp apart moves the T < 1e-4 stop of a
            # pixel by a few Gaussians (1304 of 2.2M records at cfg2)
            assert moved.mean() <= 1e-4, int(moved.sum())
        else:
            assert not moved.any(), int(moved.sum())
    finally:
        p.close()


@pytest.mark.parametrize("name,n,fp16", CASES, ids=IDS)
def test_loss_and_backward_match_reference_kernels(refpy, cuda_lib, name, n, fp16):
    p = Pair(refpy, name, n, fp16)
    try:
        W, H = p.W, p.H
        tgt = torch.from_numpy(scenes.target_image(W, H, 11).reshape(-1)).to(p.run.dt).cuda()
        # loss: the fused L1 + SSIM against the reference's two losses
        lo, go = torch.zeros_like(p.run.image), torch.zeros_like(p.run.image)
        loss = rt.FusedLoss(W, H)
        loss.evaluate(p.run.image, tgt, lo, go, W, H, grad_scaler=10.0)
        lr, gr = torch.zeros_like(p.run.image), torch.zeros_like(p.run.image)
        refpy.l1(fp16, W, H, p.run.image, tgt, lr, gr, 8.0)
        p.ref.ssim(fp16, W, H, p.run.image, tgt, lr, gr, 2.0)
        torch.cuda.synchronize()
        loss.close()
        for x, y in ((lo, lr), (go, gr)):
            x, y = x.double().cpu().numpy(), y.double().cpu().numpy()
            # fp32: a few ulps of the largest entry; fp16: one half ulp of
            # it, and at least two ulps of the smallest half subnormal
            tol = max(2.0 ** -10 * float(np.abs(y).max()), 2.0 ** -23) if fp16 else 1e-6 * float(np.abs(y).max())
            assert np.abs(x - y).max() <= tol, (np.abs(x - y).max(), tol)
        # backward on the loss gradient, through both rasterizers
        gimg = go.float().cpu().numpy()
        p.run.backward(gimg)
        g_ref = p.run.g.zeros_like()
        p.ref.backward(p.run.g, p.cam, p.ref_image, go, g_ref, fp16)
        torch.cuda.synchronize()
        ours, theirs = p.run.grads_np(), g_ref.to_numpy()
        if not fp16:
            rn = p.ref.copy(refpy.N_TOUCHED, np.uint32, p.N)
            ours_b = p.run.bins()
            refb = p.ref_bins()
            bad = _excluded_tiles(p, np.nonzero(rn != p.run.prims()["n_touched"])[0], ours_b, refb)
            near = np.zeros(p.N, bool)
            near[ours_b["inst_prim"][bad[ours_b["inst_tile"].astype(np.int64)]]] = True
            for k in ours:
                ok, worst, nbad = close_rel(ours[k][~near], theirs[k][~near], 1e-3, 1e-4)
                assert ok, (k, worst, nbad)
        else:
            g2 = p.run.g.zeros_like()
            p.ref.backward(p.run.g, p.cam, p.ref_image, go, g2, fp16)
            torch.cuda.synchronize()
            again = g2.to_numpy()
            rels, nonfinite = {}, {}
            for k in ours:
                assert np.isfinite(ours[k]).all(), k
                nonfinite[k] = int((~np.isfinite(theirs[k])).sum())
                norm = np.linalg.norm(theirs[k].ravel())
                if nonfinite[k] or not norm > 0:
                    print(f"fp16 backward {name}-{n}: {k}: reference has {nonfinite[k]} non-finite entries")
                    continue
                rel = np.linalg.norm((ours[k] - theirs[k]).ravel()) / norm
                spread = np.linalg.norm((again[k] - theirs[k]).ravel()) / norm
                rels[k] = rel
                print(f"fp16 backward {name}-{n}: {k} rel L2 vs reference {rel:.2e}, reference run to run {spread:.2e}")
            if p.N <= 100_000:
                assert not any(nonfinite.values()), nonfinite
                for k, rel in rels.items():
                    assert rel <= 2e-2, (k, rel)
            else:
                # At 1920 x 1080 the per-pixel gradients (~1e-6, x255 in the
                # reference's scaled half arithmetic) fall into the half
                # subnormal range: the reference's half2 sums lose precision
                # and overflow into inf/NaN for some Gaussians.  Both are
                # compared with the CPU oracle's fp32 evaluation of the same
                # formula from this build's forward state: this build must be
                # within 2e-3 of it, and closer to it than the reference on
                # every array.
                from oracle import pyoracle as O

                O.load()
                fs = p.run.fwd_state()
                screen = O.blend_backward(p.run.prims(), p.run.bins(), fs, go.cpu().numpy(), p.cam, fp16)
                exact = O.preprocess_backward(p.run.params, p.run.sh, p.cam, p.run.prims()["n_touched"], screen)
                for k in ours:
                    e = exact[k].reshape(ours[k].shape)
                    ne = max(float(np.linalg.norm(e.ravel())), 1e-30)
                    mine = float(np.linalg.norm((ours[k] - e).ravel())) / ne
                    fin = np.isfinite(theirs[k])
                    ref_err = float(np.linalg.norm(np.where(fin, theirs[k] - e, 0).ravel())) / ne
                    print(f"fp16 backward {name}: {k}: rel L2 vs fp32 evaluation, this build {mine:.2e}, "
                          f"reference {ref_err:.2e} (+{nonfinite[k]} non-finite)")
                    assert mine <= 2e-3, (k, mine)
                    assert mine < ref_err or nonfinite[k] > 0, (k, mine, ref_err)
    finally:
        p.close()


def test_adam_matches_reference_simple_adam(refpy, cuda_lib):
    """tgs_adam_step against the reference's own SimpleAdam::step
    (simple_adam.cu:457-580, compiled unchanged) on the same parameters and
    gradients, two steps in a row (the second exercises the moments and the
    bias corrections), 100,003 Gaussians so every array has a ragged tail,
    max_grad_1 = 0.3 as in the benchmark configurations."""
    n, sh = 100_003, 3
    params = scenes.gaussian_params(n, sh, "normal", 5)
    g = rt.GaussianSet.from_numpy(params, sh)
    gr = g.zeros_like()
    ours = rt.SimpleAdam(g, gr, rt.AdamParams(max_grad_1=0.3))
    ref = refpy.RefAdam(n, sh, {"max_grad_1": 0.3})
    try:
        for name in rt.SEGMENTS:
            ref.param(name).copy_(g.views[name].reshape(-1))
        rng = np.random.default_rng(9)
        for step in range(2):
            for name in rt.SEGMENTS:
                v = torch.from_numpy(rng.standard_normal(g.views[name].numel()).astype(np.float32) * 3.0).cuda()
                gr.views[name].copy_(v.view_as(gr.views[name]))
                ref.grad(name).copy_(v)
            ours.step(0.1)
            ref.step(0.1)
            torch.cuda.synchronize()
            for name in rt.SEGMENTS:
                a = g.views[name].reshape(-1).cpu().numpy()
                b = ref.param(name).cpu().numpy()
                np.testing.assert_allclose(a, b, rtol=2e-6, atol=1e-9, err_msg=f"step {step} {name}")
    finally:
        ref.close()
