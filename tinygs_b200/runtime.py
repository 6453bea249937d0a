"""Python mirror of the reference's plugin interfaces over the C ABI.

PyTorch is used only for device memory and streams; every computation goes
through ``libtgs_b200.so``.  Names and argument meaning follow the reference:

  GaussianSet            GPUGaussian3d (tinygs/include/tinygs/core/gpu_gaussian.hpp)
  RasterizeContext       tinygs/include/tinygs/rasterizer/rasterizer.hpp:9-29
  FastGSB200Rasterizer   RasterizerBase::forward/backward (rasterizer.hpp:38-58)
  L1Loss, FusedSSIMLoss  LossBase::evaluate(ctx, scale) (loss/loss.hpp:15-28)
  SimpleAdam             OptimizerBase::step(scale, stream) (optim/optim.hpp:39-92)

Errors surface as exceptions (the reference throws std::runtime_error);
the C ABI underneath returns status codes.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _abi
from ._abi import (TgsAdamConfig, TgsCamera, TgsDensifyConfig, TgsGaussians, TgsPcg32, TgsRasterCaps, TgsRasterCounts,
                   check, load_library)

SEGMENTS = ("means", "opacities", "rotations", "scales", "sh0", "sh_rest")
WIDTHS = {"means": 3, "opacities": 1, "rotations": 4, "scales": 3, "sh0": 3, "sh_rest": 45}
FLOATS_PER_GAUSSIAN = sum(WIDTHS.values())  # 59


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream_handle(stream) -> int | None:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


class GaussianSet:
    """One SoA set of Gaussian arrays (parameters, gradients or a moment) in a
    single device allocation: 59 floats per Gaussian, segments padded to a
    multiple of four Gaussians so every segment starts 16-byte aligned."""

    def __init__(self, n: int, sh_degree: int, device="cuda", storage: torch.Tensor | None = None,
                 capacity: int | None = None):
        self.n = int(n)
        self.sh_degree = int(sh_degree)
        self.capacity = max(self.n, int(capacity) if capacity is not None else self.n)
        npad = (self.capacity + 3) // 4 * 4
        self.npad = npad
        total = FLOATS_PER_GAUSSIAN * npad
        self.storage = storage if storage is not None else torch.zeros(total, dtype=torch.float32, device=device)
        self.full: dict[str, torch.Tensor] = {}
        off = 0
        for name in SEGMENTS:
            w = WIDTHS[name]
            self.full[name] = self.storage[off:off + w * npad].view(npad, w)
            off += w * npad
        self.views: dict[str, torch.Tensor] = {}
        self.resize(self.n)

    def resize(self, n: int) -> None:
        """Live count within the capacity (densification moves it)."""
        if not 0 <= n <= self.capacity:
            raise ValueError(f"{n} Gaussians do not fit a capacity of {self.capacity}")
        self.n = int(n)
        for name in SEGMENTS:
            self.views[name] = self.full[name][: self.n]

    def __getattr__(self, name):
        views = self.__dict__.get("views")
        if views is not None and name in views:
            return views[name]
        raise AttributeError(name)

    @classmethod
    def from_numpy(cls, arrays: dict[str, np.ndarray], sh_degree: int, device="cuda",
                   capacity: int | None = None) -> "GaussianSet":
        n = arrays["means"].shape[0]
        g = cls(n, sh_degree, device, capacity=capacity)
        g.copy_from_numpy(arrays)
        return g

    def copy_from_numpy(self, arrays: dict[str, np.ndarray]) -> None:
        for name in SEGMENTS:
            a = np.asarray(arrays[name], dtype=np.float32).reshape(self.n, WIDTHS[name])
            self.views[name].copy_(torch.from_numpy(a))

    def to_numpy(self) -> dict[str, np.ndarray]:
        out = {}
        for name in SEGMENTS:
            v = self.views[name].detach().cpu().numpy()
            out[name] = v.reshape(self.n, 15, 3) if name == "sh_rest" else (v[:, 0] if name == "opacities" else v)
        return out

    def zeros_like(self) -> "GaussianSet":
        return GaussianSet(self.n, self.sh_degree, self.storage.device, capacity=self.capacity)

    def abi(self) -> TgsGaussians:
        s = TgsGaussians()
        for name in SEGMENTS:
            setattr(s, name, self.full[name].data_ptr() if self.capacity > 0 else None)
        s.n = self.n
        s.sh_degree = self.sh_degree
        return s

    # ---- row operations (GPUGaussian3d::reorder / remove / append,
    # tinygs/src/core/gpu_gaussian.cu:117-171, 273-311)
    def _replace_with(self, other: "GaussianSet", n: int) -> None:
        self.storage.copy_(other.storage)
        self.resize(n)

    def reorder(self, idx: torch.Tensor, stream=None) -> None:
        """Row i <- row idx[i] (idx: int32/uint32 device tensor of n)."""
        tmp = GaussianSet(self.n, self.sh_degree, self.storage.device, capacity=self.capacity)
        src, dst = self.abi(), tmp.abi()
        check(load_library().tgs_arena_gather(ctypes.byref(src), ctypes.byref(dst), idx.data_ptr(), self.n,
                                              _stream_handle(stream)), "tgs_arena_gather")
        self._replace_with(tmp, self.n)

    def remove(self, keep: torch.Tensor, stream=None) -> int:
        """Keeps the rows with keep[i] != 0 (uint8 device tensor of n), in
        order; returns the new count (one host synchronisation)."""
        lib = load_library()
        ws_bytes = ctypes.c_size_t()
        check(lib.tgs_arena_compact_workspace_bytes(self.n, ctypes.byref(ws_bytes)), "workspace")
        ws = torch.empty(max(int(ws_bytes.value), 1), dtype=torch.uint8, device=self.storage.device)
        n_kept = torch.zeros(1, dtype=torch.int32, device=self.storage.device)
        tmp = GaussianSet(self.n, self.sh_degree, self.storage.device, capacity=self.capacity)
        src, dst = self.abi(), tmp.abi()
        check(lib.tgs_arena_compact(ctypes.byref(src), ctypes.byref(dst), keep.data_ptr(), self.n, ws.data_ptr(),
                                    ws.numel(), n_kept.data_ptr(), _stream_handle(stream)), "tgs_arena_compact")
        kept = int(n_kept.item())
        self._replace_with(tmp, kept)
        return kept

    def append(self, count: int) -> None:
        """count zero rows at the end (within the capacity)."""
        n = self.n
        self.resize(n + int(count))
        for name in SEGMENTS:
            self.full[name][n:n + int(count)].zero_()

    def fill_rows(self, rows: torch.Tensor, value: float = 0.0, segment: int = -1, stream=None) -> None:
        s = self.abi()
        check(load_library().tgs_arena_fill_rows(ctypes.byref(s), rows.data_ptr(), rows.numel(), float(value),
                                                  int(segment), _stream_handle(stream)), "tgs_arena_fill_rows")


def psnr(pred: torch.Tensor, target: torch.Tensor, width: int, height: int, stream=None) -> torch.Tensor:
    """PsnrMetric::evaluate (tinygs/src/loss/psnr.cu:72-128) left on the
    device: a float32 tensor [MSE, PSNR] (tgs_metric_psnr; no host sync)."""
    out = torch.empty(2, dtype=torch.float32, device=pred.device)
    ws = torch.empty(1, dtype=torch.float64, device=pred.device)
    dtype = _abi.TGS_FLOAT16 if pred.dtype == torch.float16 else _abi.TGS_FLOAT32
    check(load_library().tgs_metric_psnr(dtype, int(width), int(height), _ptr(pred), _ptr(target), _ptr(ws),
                                         _ptr(out), _stream_handle(stream)), "tgs_metric_psnr")
    return out


def morton_order(g: GaussianSet, stream=None) -> torch.Tensor:
    """The reference's Morton order of the Gaussians' means
    (tinygs/src/orchestrator.cu:26-100): int32 device tensor perm with row i
    of the reordered set = row perm[i] (tgs_morton_order)."""
    lib = load_library()
    n = g.n
    ws_bytes = ctypes.c_size_t()
    check(lib.tgs_morton_workspace_bytes(n, ctypes.byref(ws_bytes)), "tgs_morton_workspace_bytes")
    ws = torch.empty(int(ws_bytes.value), dtype=torch.uint8, device=g.storage.device)
    perm = torch.empty(max(n, 1), dtype=torch.int32, device=g.storage.device)
    check(lib.tgs_morton_order(g.full["means"].data_ptr(), n, ws.data_ptr(), ws.numel(), perm.data_ptr(),
                               _stream_handle(stream)), "tgs_morton_order")
    return perm[:n]


def reorder_gaussians(params: GaussianSet, grads: GaussianSet | None = None, optimizer=None,
                      densification_info: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Orchestrator::reorder_gaussians (tinygs/src/orchestrator.cu:1038-1060):
    Morton-sorts the Gaussians and applies the same permutation to the
    gradients, the optimizer's moments and the densification records.
    Returns the permutation."""
    perm = morton_order(params, stream)
    params.reorder(perm, stream)
    if grads is not None:
        grads.reorder(perm, stream)
    if optimizer is not None:
        optimizer.reorder(perm, stream)
    if densification_info is not None and params.n > 0:
        tmp = torch.empty_like(densification_info[: params.n])
        check(load_library().tgs_dens_gather(densification_info.data_ptr(), tmp.data_ptr(), perm.data_ptr(),
                                             params.n, _stream_handle(stream)), "tgs_dens_gather")
        densification_info[: params.n].copy_(tmp)
    return perm


def make_camera(cam: dict) -> TgsCamera:
    c = TgsCamera()
    c.width, c.height = int(cam["width"]), int(cam["height"])
    c.fx, c.fy, c.cx, c.cy = float(cam["fx"]), float(cam["fy"]), float(cam["cx"]), float(cam["cy"])
    c.near_plane, c.far_plane = float(cam.get("near", 0.01)), float(cam.get("far", 100.0))
    w = np.asarray(cam["w2c"], dtype=np.float32).reshape(16)
    for k in range(16):
        c.w2c[k] = float(w[k])
    return c


def image_numel(width: int, height: int, channels: int = 3) -> int:
    return channels * ((width + 7) // 8 * 8) * ((height + 7) // 8 * 8)


@dataclass
class RasterizeContext:
    """Mirror of tinygs::RasterizeContext (rasterizer.hpp:9-29)."""
    stream: object = None
    grad_scaler: float = 1.0
    fwd_input: dict | None = None          # camera: width, height, fx, fy, cx, cy, near, far, w2c
    fwd_output_image: torch.Tensor | None = None
    grad_output_image: torch.Tensor | None = None
    gaussians_grad: GaussianSet | None = None
    densification_info: torch.Tensor | None = None  # [n][4] float32
    alpha: torch.Tensor | None = None
    accumulate: bool = True


class FastGSB200Rasterizer:
    """RasterizerBase implementation backed by the sm_100a kernels."""

    def __init__(self, max_gaussians: int, max_width: int, max_height: int, max_instances: int = 0,
                 data_type: str = "float32"):
        self.lib = load_library()
        caps = TgsRasterCaps(int(max_gaussians), int(max_width), int(max_height), int(max_instances))
        h = ctypes.c_void_p()
        check(self.lib.tgs_raster_create(ctypes.byref(caps), ctypes.byref(h)), "tgs_raster_create")
        self.handle = h
        self.caps = caps
        self.gaussians: GaussianSet | None = None
        self.data_type = data_type

    def close(self):
        if getattr(self, "handle", None) is not None and self.handle.value:
            self.lib.tgs_raster_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_gaussians(self, g: GaussianSet) -> None:
        self.gaussians = g

    def _dtype(self, img: torch.Tensor) -> int:
        if img.dtype == torch.float32:
            return _abi.TGS_FLOAT32
        if img.dtype == torch.float16:
            return _abi.TGS_FLOAT16
        raise RuntimeError(f"unsupported image dtype {img.dtype}")

    def forward(self, ctx: RasterizeContext) -> None:
        if self.gaussians is None:
            raise RuntimeError("Gaussians not set")
        g = self.gaussians.abi()
        cam = make_camera(ctx.fwd_input)
        check(self.lib.tgs_raster_forward(self.handle, ctypes.byref(g), ctypes.byref(cam),
                                          self._dtype(ctx.fwd_output_image), _ptr(ctx.fwd_output_image),
                                          _ptr(ctx.alpha), _ptr(ctx.densification_info),
                                          _stream_handle(ctx.stream)), "tgs_raster_forward")

    def backward(self, ctx: RasterizeContext) -> None:
        if self.gaussians is None or ctx.gaussians_grad is None:
            raise RuntimeError("Gaussians or gradient gaussians not set")
        g = self.gaussians.abi()
        gg = ctx.gaussians_grad.abi()
        cam = make_camera(ctx.fwd_input)
        check(self.lib.tgs_raster_backward(self.handle, ctypes.byref(g), ctypes.byref(cam),
                                           self._dtype(ctx.fwd_output_image), _ptr(ctx.fwd_output_image),
                                           _ptr(ctx.grad_output_image), ctypes.byref(gg),
                                           1 if ctx.accumulate else 0, _ptr(ctx.densification_info),
                                           _stream_handle(ctx.stream)), "tgs_raster_backward")

    def backward_routed(self, ctx: RasterizeContext, inbox_ptrs: list[int], slice_pad: int, world: int,
                        rank: int) -> None:
        """Backward (overwrite mode) storing each Gaussian's gradients into its
        owner's gradient inbox, slot `rank` (tgs_raster_backward_routed)."""
        g = self.gaussians.abi()
        cam = make_camera(ctx.fwd_input)
        arr = (ctypes.c_void_p * world)(*inbox_ptrs)
        check(self.lib.tgs_raster_backward_routed(self.handle, ctypes.byref(g), ctypes.byref(cam),
                                                  self._dtype(ctx.fwd_output_image), _ptr(ctx.fwd_output_image),
                                                  _ptr(ctx.grad_output_image), arr, int(slice_pad), world, rank,
                                                  _ptr(ctx.densification_info), _stream_handle(ctx.stream)),
              "tgs_raster_backward_routed")

    # ---- owner-split data parallelism (tgs_raster_preprocess_views & co.)
    def share(self) -> bytes:
        """The handle's device memory as a CUDA IPC handle (64 bytes)."""
        h = _abi.TgsIpcHandle()
        check(self.lib.tgs_raster_share(self.handle, ctypes.byref(h)), "tgs_raster_share")
        return bytes(h.bytes)

    def arena(self) -> int:
        p = ctypes.c_void_p()
        check(self.lib.tgs_raster_arena(self.handle, ctypes.byref(p)), "tgs_raster_arena")
        return p.value

    def attach_views(self, arenas: list[int], rank: int) -> None:
        arr = (ctypes.c_void_p * len(arenas))(*arenas)
        check(self.lib.tgs_raster_attach_views(self.handle, arr, len(arenas), rank), "tgs_raster_attach_views")

    def preprocess_views(self, params: GaussianSet, cams: list[dict], dtype: int, first: int, last: int,
                         dens: torch.Tensor | None = None, stream=None) -> None:
        g = params.abi()
        cs = (TgsCamera * len(cams))(*[make_camera(c) for c in cams])
        check(self.lib.tgs_raster_preprocess_views(self.handle, ctypes.byref(g), cs, dtype, int(first), int(last),
                                                   _ptr(dens), _stream_handle(stream)), "tgs_raster_preprocess_views")

    def forward_gathered(self, n: int, cam: dict, image: torch.Tensor, alpha: torch.Tensor | None = None,
                         stream=None) -> None:
        c = make_camera(cam)
        check(self.lib.tgs_raster_forward_gathered(self.handle, int(n), ctypes.byref(c), self._dtype(image),
                                                   _ptr(image), _ptr(alpha), _stream_handle(stream)),
              "tgs_raster_forward_gathered")

    def backward_screen(self, cam: dict, image: torch.Tensor, grad_image: torch.Tensor, absgrad: bool = False,
                        stream=None) -> None:
        c = make_camera(cam)
        check(self.lib.tgs_raster_backward_screen(self.handle, ctypes.byref(c), self._dtype(image), _ptr(image),
                                                  _ptr(grad_image), 1 if absgrad else 0, _stream_handle(stream)),
              "tgs_raster_backward_screen")

    def backward_views_adam(self, params: GaussianSet, cams: list[dict], first: int, last: int,
                            grads: GaussianSet | None,
                            exp_avg: GaussianSet, exp_avg_sq: GaussianSet, cfg: "AdamParams", step: int,
                            gradient_scale: float, dens: torch.Tensor | None = None, stream=None) -> None:
        p, m, v = params.abi(), exp_avg.abi(), exp_avg_sq.abi()
        gr = grads.abi() if grads is not None else None
        cs = (TgsCamera * len(cams))(*[make_camera(c) for c in cams])
        c = cfg.abi()
        check(self.lib.tgs_raster_backward_views_adam(self.handle, ctypes.byref(p), cs, int(first), int(last),
                                                      ctypes.byref(gr) if gr is not None else None,
                                                      ctypes.byref(m), ctypes.byref(v),
                                                      ctypes.byref(c), int(step), float(gradient_scale), _ptr(dens),
                                                      _stream_handle(stream)), "tgs_raster_backward_views_adam")

    def set_stage_timing(self, enable: bool) -> None:
        check(self.lib.tgs_raster_set_stage_timing(self.handle, 1 if enable else 0), "tgs_raster_set_stage_timing")

    def stage_times(self) -> list[float]:
        """ms of [preprocess, binning, blend forward, blend backward,
        per-Gaussian backward (+Adam when fused)] of the last forward/backward."""
        out = (ctypes.c_float * 5)()
        check(self.lib.tgs_raster_stage_times(self.handle, out), "tgs_raster_stage_times")
        return list(out)

    def counts(self, stream=None) -> TgsRasterCounts:
        c = TgsRasterCounts()
        check(self.lib.tgs_raster_counts(self.handle, ctypes.byref(c), _stream_handle(stream)), "tgs_raster_counts")
        return c

    def debug_buffer(self, which: int) -> tuple[int, int]:
        p = ctypes.c_void_p()
        n = ctypes.c_size_t()
        check(self.lib.tgs_raster_debug_buffer(self.handle, which, ctypes.byref(p), ctypes.byref(n)),
              "tgs_raster_debug_buffer")
        return p.value, n.value

    def debug_array(self, which: int, dtype: torch.dtype, count: int) -> torch.Tensor:
        """Copy the first `count` elements of an internal buffer (tests only)."""
        ptr, nbytes = self.debug_buffer(which)
        elem = torch.tensor([], dtype=dtype).element_size()
        if count * elem > nbytes:
            raise ValueError("debug buffer smaller than requested")
        if count == 0:
            return torch.empty(0, dtype=dtype, device="cuda")
        typestr = {torch.float32: "<f4", torch.float16: "<f2", torch.int32: "<i4", torch.int16: "<i2",
                   torch.uint8: "|u1"}[dtype]
        view = _DeviceView(ptr, count, typestr)
        return torch.as_tensor(view, device="cuda").clone()


class _DeviceView:
    """Minimal __cuda_array_interface__ exporter for a raw device pointer."""

    def __init__(self, ptr: int, count: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (count,), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class FusedLoss:
    """The reference's default loss mix (configs/default.json:30-39):
    0.8 * L1 + 0.2 * (1 - SSIM), each term scaled by grad_scaler, evaluated
    in one call that accumulates into `loss` and `grad` like
    LossBase::evaluate and also reduces the step's loss to a device scalar."""

    def __init__(self, max_width: int, max_height: int, w_l1: float = 0.8, w_ssim: float = 0.2):
        self.lib = load_library()
        h = ctypes.c_void_p()
        check(self.lib.tgs_loss_create(int(max_width), int(max_height), ctypes.byref(h)), "tgs_loss_create")
        self.handle = h
        self.w_l1, self.w_ssim = w_l1, w_ssim

    def set_accumulate(self, accumulate: bool) -> None:
        """False: evaluate() writes every element of the padded loss map and
        gradient (what the accumulating mode leaves in zeroed buffers), so no
        per-step zeroing is needed (tgs_loss_set_accumulate)."""
        check(self.lib.tgs_loss_set_accumulate(self.handle, 1 if accumulate else 0), "tgs_loss_set_accumulate")

    def close(self):
        if getattr(self, "handle", None) is not None and self.handle.value:
            self.lib.tgs_loss_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _dtype(t: torch.Tensor) -> int:
        return _abi.TGS_FLOAT16 if t.dtype == torch.float16 else _abi.TGS_FLOAT32

    def evaluate(self, pred, target, loss_map, grad, width, height, grad_scaler=1.0, loss_sum=None, stream=None):
        check(self.lib.tgs_loss_l1_ssim(self.handle, self._dtype(pred), int(width), int(height), _ptr(pred),
                                        _ptr(target), _ptr(loss_map), _ptr(grad),
                                        float(self.w_l1 * grad_scaler), float(self.w_ssim * grad_scaler),
                                        _ptr(loss_sum), _stream_handle(stream)), "tgs_loss_l1_ssim")

    def evaluate_l1(self, pred, target, loss_map, grad, width, height, scale, stream=None):
        check(self.lib.tgs_loss_l1(self._dtype(pred), int(width), int(height), _ptr(pred), _ptr(target),
                                   _ptr(loss_map), _ptr(grad), float(scale), _stream_handle(stream)), "tgs_loss_l1")

    def evaluate_ssim(self, pred, target, loss_map, grad, width, height, scale, stream=None):
        check(self.lib.tgs_loss_fused_ssim(self.handle, self._dtype(pred), int(width), int(height), _ptr(pred),
                                           _ptr(target), _ptr(loss_map), _ptr(grad), float(scale),
                                           _stream_handle(stream)), "tgs_loss_fused_ssim")


@dataclass
class AdamParams:
    """GaussianOptimizationParams + SimpleAdamParameters (optim.hpp:8-37,
    simple_adam.hpp:8-27) with the reference defaults."""
    beta1: float = 0.9
    beta2: float = 0.999
    epsilon: float = 1e-8
    max_grad_1: float = 1.0
    means_lr: float = 1.6e-4
    shs_lr: float = 2.5e-3
    opacities_lr: float = 5.0e-2
    scales_lr: float = 5.0e-3
    rotations_lr: float = 1.0e-3
    opacities_l1: float = 0.0
    scales_l1: float = 0.0
    scene_scale: float = 1.0
    global_lr: float = 1.0
    decay_reduction_mean: bool = True

    def abi(self) -> TgsAdamConfig:
        return TgsAdamConfig(self.beta1, self.beta2, self.epsilon, self.max_grad_1, self.means_lr, self.shs_lr,
                             self.opacities_lr, self.scales_lr, self.rotations_lr, self.opacities_l1,
                             self.scales_l1, self.scene_scale, self.global_lr, 1 if self.decay_reduction_mean else 0)


class SimpleAdam:
    """OptimizerBase::step over a GaussianSet; owns the two moment sets."""

    def __init__(self, params: GaussianSet, grads: GaussianSet, cfg: AdamParams | None = None):
        self.lib = load_library()
        self.params, self.grads = params, grads
        self.cfg = cfg or AdamParams()
        self.exp_avg = params.zeros_like()
        self.exp_avg_sq = params.zeros_like()
        self.global_steps = 0

    def fused_backward_step(self, rast: "FastGSB200Rasterizer", ctx: RasterizeContext, scale: float,
                            write_grads: bool = False) -> None:
        """rast.backward(ctx) with accumulate=False followed by step(scale),
        in one pass over the Gaussians (tgs_raster_backward_adam)."""
        self.global_steps += 1
        p, m, v = self.params.abi(), self.exp_avg.abi(), self.exp_avg_sq.abi()
        g = self.grads.abi() if write_grads else None
        cam = make_camera(ctx.fwd_input)
        cfg = self.cfg.abi()
        check(self.lib.tgs_raster_backward_adam(rast.handle, ctypes.byref(p), ctypes.byref(cam),
                                                rast._dtype(ctx.fwd_output_image), _ptr(ctx.fwd_output_image),
                                                _ptr(ctx.grad_output_image), ctypes.byref(g) if g else None,
                                                ctypes.byref(m), ctypes.byref(v), ctypes.byref(cfg),
                                                self.global_steps, float(scale), _ptr(ctx.densification_info),
                                                _stream_handle(ctx.stream)), "tgs_raster_backward_adam")

    # ---- OptimizerBase row hooks (tinygs/include/tinygs/optim/optim.hpp:61-76,
    # SimpleAdam: tinygs/src/optim/simple_adam.cu:841-1099)
    def remove(self, keep: torch.Tensor, stream=None) -> int:
        """Compacts both moments to the kept rows."""
        self.exp_avg.remove(keep, stream)
        return self.exp_avg_sq.remove(keep, stream)

    def duplicate(self, indices=None, new_indices=None, count: int = 0) -> None:
        """New Gaussians get zero moments (the reference only grows its
        moment vectors to the new size; the indices are unused)."""
        for m in (self.exp_avg, self.exp_avg_sq):
            m.append(count)

    def reset(self, indices: torch.Tensor, stream=None) -> None:
        """Zeroes both moments of the given rows."""
        for m in (self.exp_avg, self.exp_avg_sq):
            m.fill_rows(indices, 0.0, -1, stream)

    def reset_opacity(self, stream=None) -> None:
        """Zeroes the opacity moments of every row."""
        rows = torch.arange(self.params.n, dtype=torch.int32, device=self.params.storage.device)
        for m in (self.exp_avg, self.exp_avg_sq):
            m.fill_rows(rows, 0.0, 1, stream)

    def reorder(self, idx: torch.Tensor, stream=None) -> None:
        for m in (self.exp_avg, self.exp_avg_sq):
            m.reorder(idx, stream)

    def step(self, scale: float, stream=None, zero_grads: bool = False) -> None:
        self.global_steps += 1
        p, g, m, v = self.params.abi(), self.grads.abi(), self.exp_avg.abi(), self.exp_avg_sq.abi()
        cfg = self.cfg.abi()
        check(self.lib.tgs_adam_step(ctypes.byref(p), ctypes.byref(g), ctypes.byref(m), ctypes.byref(v),
                                     ctypes.byref(cfg), self.global_steps, float(scale), 1 if zero_grads else 0,
                                     _stream_handle(stream)), "tgs_adam_step")


@dataclass
class DensifyParams:
    """StrategyParams (tinygs/include/tinygs/strategy/strategy.hpp:9-29)."""
    pruning_opacity_threshold: float = 0.005
    pruning_scale_threshold: float = 0.1
    max_screen_size: float = 10.0
    duplicate_grad_threshold: float = 0.0002
    duplicate_scale_threshold: float = 0.01
    absgrad: bool = False
    refine_every: int = 100
    start_refine: int = 500
    end_refine: int = 15_000
    max_num_gaussians: int = 10_000_000
    reset_every: int = 3_000
    seed: int = 42

    def abi(self, scene_scale: float, grad_scaler: float, width: int, height: int) -> TgsDensifyConfig:
        c = TgsDensifyConfig()
        c.duplicate_grad_threshold = self.duplicate_grad_threshold
        c.duplicate_scale_threshold = self.duplicate_scale_threshold
        c.pruning_opacity_threshold = self.pruning_opacity_threshold
        c.pruning_scale_threshold = self.pruning_scale_threshold
        c.max_screen_size = self.max_screen_size
        c.scene_scale = scene_scale
        c.grad_scaler = grad_scaler
        c.absgrad = 1 if self.absgrad else 0
        c.refine_every, c.start_refine, c.end_refine = self.refine_every, self.start_refine, self.end_refine
        c.reset_every = self.reset_every
        c.image_width, c.image_height = int(width), int(height)
        c.max_num_gaussians = self.max_num_gaussians
        return c


class Densifier:
    """DefaultStrategy (tinygs/src/strategy/default.cu:17-69) over GaussianSets
    allocated with spare capacity: step() runs once per training step after
    the optimizer, refines / resets when the step number asks, and moves the
    live count of the parameters, gradients and both Adam moments."""

    def __init__(self, params: GaussianSet, grads: GaussianSet | None, optimizer: SimpleAdam,
                 cfg: DensifyParams | None = None, scene_scale: float = 1.0):
        self.lib = load_library()
        self.params, self.grads, self.optimizer = params, grads, optimizer
        self.cfg = cfg or DensifyParams()
        self.scene_scale = float(scene_scale)
        self.capacity = params.capacity
        h = ctypes.c_void_p()
        check(self.lib.tgs_densify_create(self.capacity, ctypes.byref(h)), "tgs_densify_create")
        self.handle = h
        self.rng = TgsPcg32()
        self.lib.tgs_pcg32_seed(ctypes.byref(self.rng), self.cfg.seed, 1)
        # densification_info records (counter, grad, absgrad, max radius)
        self.dens_storage = torch.zeros((self.capacity, 4), dtype=torch.float32, device=params.storage.device)
        self.step_count = 0

    @property
    def densification_info(self) -> torch.Tensor:
        return self.dens_storage[: self.params.n]

    def step(self, ctx: RasterizeContext) -> int:
        """One strategy step; returns the new number of Gaussians."""
        cam = ctx.fwd_input
        cfg = self.cfg.abi(self.scene_scale, ctx.grad_scaler, int(cam["width"]), int(cam["height"]))
        n = ctypes.c_int64(self.params.n)
        p, m, v = self.params.abi(), self.optimizer.exp_avg.abi(), self.optimizer.exp_avg_sq.abi()
        g = self.grads.abi() if self.grads is not None else None
        check(self.lib.tgs_densify_step(self.handle, ctypes.byref(p), ctypes.byref(g) if g else None,
                                        ctypes.byref(m), ctypes.byref(v), self.dens_storage.data_ptr(),
                                        ctypes.byref(cfg), self.step_count, ctypes.byref(self.rng),
                                        ctypes.byref(n), _stream_handle(ctx.stream)), "tgs_densify_step")
        self.step_count += 1
        for s in (self.params, self.grads, self.optimizer.exp_avg, self.optimizer.exp_avg_sq):
            if s is not None:
                s.resize(n.value)
        return n.value

    def close(self) -> None:
        if self.handle:
            self.lib.tgs_densify_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
