"""Gradient routing of the multi-GPU step on one GPU: with two inboxes in
local memory, tgs_raster_backward_routed stores every Gaussian's gradients
into the inbox of the rank whose slice holds it (slot = the calling rank),
equal to the plain backward's gradients of that slice."""
import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import GpuRun, close_rel, scene
from tinygs_b200 import _abi
from tinygs_b200 import dp as dpm
from tinygs_b200 import runtime as rt

pytestmark = pytest.mark.gpu

WIDTHS = {"means": 3, "opacities": 1, "rotations": 4, "scales": 3, "sh0": 3, "sh_rest": 45}


def _slot(buf: torch.Tensor, slot: int, slice_pad: int, rows: int) -> dict:
    base = slot * 59 * slice_pad
    out, off = {}, 0
    for k, w in WIDTHS.items():
        out[k] = buf[base + off: base + off + w * slice_pad].view(slice_pad, w)[:rows].cpu().numpy()
        off += w * slice_pad
    return out


@pytest.mark.parametrize("rank", [0, 1])
def test_routed_backward_fills_the_owners_inboxes(rank):
    cfg, params, sh, cam = scene("cfg1", n=10_001)
    run = GpuRun(params, sh, cam, False).forward()
    g = np.random.default_rng(5).normal(0, 1e-3, run.image.numel()).astype(np.float32)
    run.backward(g, accumulate=False)
    plain = run.grads_np()
    n, world = run.n, 2
    lo = [dpm.dp_slice_begin(n, world, r) for r in range(world + 1)]
    slice_pad = (max(lo[r + 1] - lo[r] for r in range(world)) + 3) // 4 * 4
    inboxes = [torch.full((world * 59 * slice_pad,), float("nan"), device="cuda") for _ in range(world)]
    # the blend backward accumulates the screen-space gradients that the
    # forward zeroes: a second backward needs a second forward
    run.forward()
    run.rast.backward_routed(run.ctx, [b.data_ptr() for b in inboxes], slice_pad, world, rank)
    torch.cuda.synchronize()
    for s in range(world):
        got = _slot(inboxes[s], rank, slice_pad, lo[s + 1] - lo[s])
        for k in WIDTHS:
            ref = plain[k].reshape(n, -1)[lo[s]:lo[s + 1]]
            # two blend-backward runs: float-atomic order noise only
            ok, worst, nbad = close_rel(got[k], ref, 1e-3, 1e-5)
            assert ok, (s, k, worst, nbad)
        # the other slot of that inbox is untouched
        other = _slot(inboxes[s], 1 - rank, slice_pad, lo[s + 1] - lo[s])
        assert np.isnan(other["means"]).all()
