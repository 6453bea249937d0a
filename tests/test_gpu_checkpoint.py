"""Checkpoint and resume (tgs_checkpoint_save / _info / _load through
tinygs_b200.checkpoint): the saved state comes back bit for bit into fresh
objects, the resumed run continues as the uninterrupted one does, and
damaged, truncated or oversized files are refused without touching the
destination arrays."""
import ctypes

import numpy as np
import pytest
import torch

from tinygs_b200 import _abi
from tinygs_b200 import checkpoint as ck
from tinygs_b200 import runtime as rt
from tinygs_b200 import scenes

pytestmark = pytest.mark.gpu

N0, CAP = 3000, 12000


class Run:
    """A small densifying training run (cfg0 scene, SH0, fp32)."""

    def __init__(self, params=None):
        cfg0 = scenes.CONFIGS["cfg0"]
        self.params0 = scenes.gaussian_params(N0, 0, cfg0.means, 5) if params is None else params
        self.cam = scenes.cameras(cfg0)[0]
        W, H = self.cam["width"], self.cam["height"]
        self.W, self.H = W, H
        self.g = rt.GaussianSet.from_numpy(self.params0, 0, capacity=CAP)
        self.grads = self.g.zeros_like()
        self.opt = rt.SimpleAdam(self.g, self.grads, rt.AdamParams(max_grad_1=0.3))
        self.dens = rt.Densifier(self.g, self.grads, self.opt,
                                 rt.DensifyParams(refine_every=2, start_refine=2, end_refine=20,
                                                  duplicate_grad_threshold=1e-6, reset_every=1000))
        self.rast = rt.FastGSB200Rasterizer(CAP, W, H)
        self.img = torch.zeros(rt.image_numel(W, H), device="cuda")
        self.gimg, self.lmap = torch.zeros_like(self.img), torch.zeros_like(self.img)
        self.tgt = torch.from_numpy(scenes.target_image(W, H, 3).reshape(-1)).cuda()
        self.loss = rt.FusedLoss(W, H)
        self.step_no = 0

    def step(self):
        ctx = rt.RasterizeContext(fwd_input=self.cam, fwd_output_image=self.img, grad_output_image=self.gimg,
                                  gaussians_grad=self.grads, grad_scaler=10.0,
                                  densification_info=self.dens.densification_info)
        self.gimg.zero_()
        self.lmap.zero_()
        self.rast.set_gaussians(self.g)
        self.rast.forward(ctx)
        self.loss.evaluate(self.img, self.tgt, self.lmap, self.gimg, self.W, self.H, grad_scaler=10.0)
        ctx.accumulate = False
        self.rast.backward(ctx)
        self.opt.step(0.1)
        self.dens.step(ctx)
        self.step_no += 1

    def state(self):
        torch.cuda.synchronize()
        return {"n": self.g.n, "params": self.g.to_numpy(), "m": self.opt.exp_avg.to_numpy(),
                "v": self.opt.exp_avg_sq.to_numpy(), "dens": self.dens.densification_info.cpu().numpy(),
                "adam": self.opt.global_steps, "strategy": self.dens.step_count,
                "rng": (self.dens.rng.state, self.dens.rng.inc)}

    def close(self):
        self.rast.close()
        self.loss.close()
        self.dens.close()


def _equal(a, b):
    assert a["n"] == b["n"] and a["adam"] == b["adam"] and a["strategy"] == b["strategy"] and a["rng"] == b["rng"]
    for key in ("params", "m", "v"):
        for name in a[key]:
            np.testing.assert_array_equal(a[key][name], b[key][name])
    np.testing.assert_array_equal(a["dens"], b["dens"])


def test_round_trip_and_continuation(tmp_path):
    path = tmp_path / "run.ckpt"
    a = Run()
    for _ in range(3):  # past the first refine: the count has moved
        a.step()
    saved = a.state()
    assert saved["n"] != N0
    ck.save_checkpoint(path, a.g, a.opt, a.dens, step=a.step_no)
    assert not (tmp_path / "run.ckpt.tmp").exists()
    info = ck.checkpoint_info(path)
    assert (info.n, info.sh_degree, info.has_moments, info.has_densification) == (saved["n"], 0, True, True)
    assert (info.step, info.adam_step, info.strategy_step) == (3, saved["adam"], saved["strategy"])
    assert (info.rng_state, info.rng_inc) == saved["rng"]

    # a fresh run (other initial parameters, so nothing matches by accident)
    b = Run(params=scenes.gaussian_params(N0, 0, scenes.CONFIGS["cfg0"].means, 77))
    b.step_no = ck.load_checkpoint(path, b.g, b.opt, b.dens)
    assert b.step_no == 3
    _equal(b.state(), saved)

    # both continue: through the next refine (strategy step 4) the counts
    # stay equal and the parameters agree up to the float-atomic order noise
    # of the blend backward
    for _ in range(3):
        a.step()
        b.step()
    sa, sb = a.state(), b.state()
    assert sa["n"] == sb["n"] and sa["adam"] == sb["adam"] and sa["strategy"] == sb["strategy"]
    assert sa["rng"] == sb["rng"]
    for name in sa["params"]:
        x, y = sa["params"][name], sb["params"][name]
        close = np.abs(x - y) <= 1e-6 + 1e-5 * np.abs(x)
        assert close.mean() > 0.999, (name, close.mean())
    a.close()
    b.close()


def test_refused_files_leave_arrays_untouched(tmp_path):
    path = tmp_path / "run.ckpt"
    a = Run()
    a.step()
    ck.save_checkpoint(path, a.g, a.opt, a.dens, step=1)
    raw = path.read_bytes()
    b = Run(params=scenes.gaussian_params(N0, 0, scenes.CONFIGS["cfg0"].means, 78))
    before = b.state()

    def refused(data, code, name):
        p = tmp_path / name
        p.write_bytes(data)
        with pytest.raises(_abi.TgsError) as e:
            ck.load_checkpoint(p, b.g, b.opt, b.dens)
        assert e.value.status == code
        _equal(b.state(), before)

    refused(raw[:-9], _abi.TGS_ERR_INVALID_ARGUMENT, "truncated.ckpt")
    flipped = bytearray(raw)
    flipped[200] ^= 0x40
    refused(bytes(flipped), _abi.TGS_ERR_INVALID_ARGUMENT, "flipped.ckpt")
    refused(raw + b"\0", _abi.TGS_ERR_INVALID_ARGUMENT, "longer.ckpt")
    refused(b"NOTACKPT" + raw[8:], _abi.TGS_ERR_INVALID_ARGUMENT, "foreign.ckpt")

    # a parameters-only checkpoint cannot fill the moments
    ck.save_checkpoint(tmp_path / "params.ckpt", a.g)
    refused((tmp_path / "params.ckpt").read_bytes(), _abi.TGS_ERR_UNSUPPORTED, "params_only.ckpt")
    # ... but restores the parameters alone
    small = rt.GaussianSet(0, 0, capacity=CAP)
    ck.load_checkpoint(tmp_path / "params.ckpt", small)
    assert small.n == a.g.n
    np.testing.assert_array_equal(small.to_numpy()["means"], a.g.to_numpy()["means"])

    # capacity below the saved count
    tiny = rt.GaussianSet(0, 0, capacity=a.g.n - 1)
    lib = _abi.load_library()
    p = tiny.abi()
    rc = lib.tgs_checkpoint_load(bytes(path), tiny.capacity, ctypes.byref(p), None, None, None, None,
                                 torch.cuda.current_stream().cuda_stream)
    assert rc == _abi.TGS_ERR_CAPACITY
    assert lib.tgs_checkpoint_info(bytes(tmp_path / "missing.ckpt"), None, None, None, None) == \
        _abi.TGS_ERR_INVALID_ARGUMENT
    a.close()
    b.close()
