"""Helpers shared by the GPU parity tests: run the CUDA path through the C ABI
and read its intermediate state back in the oracle's formats."""
from __future__ import annotations

import numpy as np
import torch

from tinygs_b200 import runtime as rt
from tinygs_b200 import scenes


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


class GpuRun:
    """One forward (and optionally backward) of the CUDA rasterizer."""

    def __init__(self, params: dict, sh_degree: int, cam: dict, fp16: bool, max_instances: int = 0):
        self.params, self.sh, self.cam, self.fp16 = params, sh_degree, cam, fp16
        self.n = params["means"].shape[0]
        self.W, self.H = int(cam["width"]), int(cam["height"])
        self.g = rt.GaussianSet.from_numpy(params, sh_degree)
        self.grads = self.g.zeros_like()
        self.rast = rt.FastGSB200Rasterizer(max(self.n, 1), self.W, self.H, max_instances)
        self.rast.set_gaussians(self.g)
        self.dt = torch.float16 if fp16 else torch.float32
        numel = rt.image_numel(self.W, self.H)
        self.image = torch.zeros(numel, dtype=self.dt, device="cuda")
        self.alpha = torch.zeros(numel // 3, dtype=self.dt, device="cuda")
        self.grad_image = torch.zeros(numel, dtype=self.dt, device="cuda")
        self.ctx = rt.RasterizeContext(fwd_input=cam, fwd_output_image=self.image, grad_output_image=self.grad_image,
                                       gaussians_grad=self.grads, alpha=self.alpha)

    def forward(self):
        self.rast.forward(self.ctx)
        torch.cuda.synchronize()
        self.counts = self.rast.counts()
        return self

    def backward(self, grad_image: np.ndarray, accumulate: bool = True):
        self.grad_image.copy_(torch.from_numpy(np.ascontiguousarray(grad_image)).to(self.dt))
        self.ctx.accumulate = accumulate
        self.rast.backward(self.ctx)
        torch.cuda.synchronize()
        return self

    # ---- intermediate state in oracle formats
    def prims(self) -> dict:
        n = self.n
        r = self.rast
        out = {"n_touched": to_np(r.debug_array(0, torch.int32, n)).view(np.uint32),
               "bounds": to_np(r.debug_array(9, torch.int16, 4 * n)).view(np.uint16).reshape(n, 4),
               "mean2d": to_np(r.debug_array(5, torch.float32, 2 * n)).reshape(n, 2),
               "depth_key": to_np(r.debug_array(14, torch.int32, n)).view(np.uint32)}
        if self.fp16:
            out["prim_info"] = to_np(r.debug_array(8, torch.uint8, 16 * n)).reshape(n, 16)
        else:
            out["conic_opacity"] = to_np(r.debug_array(6, torch.float32, 4 * n)).reshape(n, 4)
            out["color"] = to_np(r.debug_array(7, torch.float32, 3 * n)).reshape(n, 3)
        vis = out["n_touched"] > 0
        # entries of culled Gaussians are not written by the kernels
        out["mean2d"][~vis] = 0
        out["bounds"][~vis] = 0
        out["depth_key"][~vis] = 0
        return out

    def bins(self) -> dict:
        c = self.counts
        gw, gh = (self.W + 15) // 16, (self.H + 15) // 16
        r = self.rast
        ni = int(c.n_instances)
        ranges = to_np(r.debug_array(3, torch.int32, 2 * gw * gh)).view(np.uint32).reshape(gw * gh, 2)
        # tiles are not stored per instance: tile t owns [ranges[t,0], ranges[t,1])
        tiles = np.zeros(ni, np.uint32)
        for t in np.nonzero(ranges[:, 1] > ranges[:, 0])[0]:
            tiles[ranges[t, 0]:ranges[t, 1]] = t
        return {"inst_tile": tiles,
                "inst_prim": to_np(r.debug_array(2, torch.int32, ni)).view(np.uint32),
                "ranges": ranges,
                "bucket_offsets": to_np(r.debug_array(13, torch.int32, gw * gh)).view(np.uint32),
                "n_instances": ni, "n_buckets": int(c.n_buckets), "n_visible": int(c.n_visible),
                "sorted_visible": to_np(r.debug_array(10, torch.int32, int(c.n_visible))).view(np.uint32)}

    def fwd_state(self) -> dict:
        c = self.counts
        gw, gh = (self.W + 15) // 16, (self.H + 15) // 16
        pl = rt.image_numel(self.W, self.H) // 3
        r = self.rast
        nb = int(c.n_buckets)
        if self.fp16:
            ncon = to_np(r.debug_array(4, torch.int16, pl)).view(np.uint16)
            ckpt = to_np(r.debug_array(15, torch.int16, nb * 256 * 4)).view(np.uint16)
            tmax = to_np(r.debug_array(12, torch.int32, gw * gh)).view(np.uint32).astype(np.uint16)
        else:
            ncon = to_np(r.debug_array(4, torch.int32, pl)).view(np.uint32)
            ckpt = to_np(r.debug_array(15, torch.float32, nb * 256 * 4))
            tmax = to_np(r.debug_array(12, torch.int32, gw * gh)).view(np.uint32)
        if ckpt.size == 0:
            ckpt = np.zeros(256 * 4, ckpt.dtype)
        return {"image": to_np(self.image), "alpha": to_np(self.alpha), "n_contrib": ncon, "tile_max": tmax,
                "ckpt": np.ascontiguousarray(ckpt)}

    def helpers(self) -> dict:
        h = to_np(self.rast.debug_array(11, torch.float32, 12 * self.n)).reshape(self.n, 12)
        vis = to_np(self.rast.debug_array(0, torch.int32, self.n)) > 0
        h = h.copy()
        h[~vis] = 0
        return {"grad_mean2d": h[:, 0:2], "absgrad_mean2d": h[:, 2:4], "grad_conic": h[:, 4:7],
                "grad_opacity": h[:, 7], "grad_color": h[:, 8:11]}

    def grads_np(self) -> dict:
        return self.grads.to_numpy()


def scene(name: str, n: int | None = None, sh_degree: int | None = None, view: int = 0):
    cfg = scenes.CONFIGS[name]
    n = cfg.n if n is None else n
    sh = cfg.sh_degree if sh_degree is None else sh_degree
    params = scenes.gaussian_params(n, sh, cfg.means, cfg.seed)
    cam = scenes.cameras(cfg)[view]
    return cfg, params, sh, cam


def close_rel(a, b, rtol=1e-3, floor_frac=1e-4):
    """|a-b| <= rtol*|b| + floor_frac*max|b|, elementwise; returns (ok, worst)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    scale = max(float(np.abs(b).max()) if b.size else 0.0, 1e-30)
    err = np.abs(a - b)
    lim = rtol * np.abs(b) + floor_frac * scale
    bad = err > lim
    worst = float((err / np.maximum(lim, 1e-30)).max()) if err.size else 0.0
    return (not bad.any()), worst, int(bad.sum())
