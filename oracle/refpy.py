"""ctypes front end of oracle/_ref/libtgs_ref.so: the reference's own CUDA
kernels (Adversarr/tinygs fastgs_ours/, fastgs_ours_fp16/, loss/l1.cu,
loss/fused_ssim.cu) built unchanged by oracle/build_ref.py.

TEST INFRASTRUCTURE ONLY -- imported by tests/ (as the checker) and by
bench.py's reference arm (which times the reference's own step).  Runs the
reference on device memory the caller owns (torch tensors), so the product
and the reference see the same bytes.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int32, c_int64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_ref" / "libtgs_ref.so"

N_TOUCHED, SORTED_PRIMS, SORTED_DEPTH_KEYS, INST_KEYS, INST_PRIMS, TILE_RANGES, BUCKET_OFFSETS = range(7)
TILE_MAX_CONTRIB, N_CONTRIB, MEAN2D, CONIC_OPACITY, COLOR, BOUNDS, CKPT = range(7, 14)
GRAD_MEAN2D, ABSGRAD_MEAN2D, GRAD_CONIC, GRAD_COLOR, PRIM_INFO_GRAD, ALPHA, BUCKET_TILE = range(14, 21)


class RefCamera(ctypes.Structure):
    _fields_ = [("width", c_int32), ("height", c_int32), ("fx", c_float), ("fy", c_float), ("cx", c_float),
                ("cy", c_float), ("near_plane", c_float), ("far_plane", c_float), ("w2c", c_float * 16)]


class RefGaussians(ctypes.Structure):
    _fields_ = [("means", c_void_p), ("opacities", c_void_p), ("rotations", c_void_p), ("scales", c_void_p),
                ("sh0", c_void_p), ("sh_rest", c_void_p), ("n", c_int64), ("sh_degree", c_int32)]


_lib = None


def available() -> bool:
    return LIB.exists()


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            raise FileNotFoundError(f"{LIB} is not built (python oracle/build_ref.py, where the reference is present)")
        lib = ctypes.CDLL(str(LIB))
        lib.tgsref_copy.restype = c_int64
        lib.tgsref_last_error.restype = ctypes.c_char_p
        _lib = lib
    return _lib


def _check(st: int, what: str) -> None:
    if st != 0:
        raise RuntimeError(f"{what}: {st} {load().tgsref_last_error().decode(errors='replace')}")


def camera(cam: dict) -> RefCamera:
    c = RefCamera()
    c.width, c.height = int(cam["width"]), int(cam["height"])
    c.fx, c.fy, c.cx, c.cy = float(cam["fx"]), float(cam["fy"]), float(cam["cx"]), float(cam["cy"])
    c.near_plane, c.far_plane = float(cam.get("near", 0.01)), float(cam.get("far", 100.0))
    w = np.asarray(cam["w2c"], dtype=np.float32).reshape(16)
    for k in range(16):
        c.w2c[k] = float(w[k])
    return c


def gaussians(gset) -> RefGaussians:
    """A tinygs_b200.runtime.GaussianSet (same SoA layout as the reference's
    GPUGaussian3d arrays) as the harness's pointer struct."""
    s = RefGaussians()
    for name in ("means", "opacities", "rotations", "scales", "sh0", "sh_rest"):
        setattr(s, name, gset.full[name].data_ptr())
    s.n, s.sh_degree = gset.n, gset.sh_degree
    return s


def _stream(stream) -> int:
    import torch

    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


class RefRasterizer:
    """The reference rasterizer of one precision on one handle."""

    def __init__(self):
        self.lib = load()
        h = c_void_p()
        _check(self.lib.tgsref_create(ctypes.byref(h)), "tgsref_create")
        self.h = h
        self.counts = (0, 0, 0)
        self.fp16 = False

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            self.lib.tgsref_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, gset, cam: dict, image, fp16: bool, dens=None, stream=None):
        self.fp16 = bool(fp16)
        self.cam = camera(cam)
        self.g = gaussians(gset)
        counts = (c_int32 * 3)()
        _check(self.lib.tgsref_forward(self.h, int(fp16), ctypes.byref(self.g), ctypes.byref(self.cam),
                                       c_void_p(image.data_ptr()), c_void_p(dens.data_ptr() if dens is not None else 0),
                                       c_void_p(_stream(stream)), counts), "tgsref_forward")
        self.counts = (counts[0], counts[1], counts[2])
        return self.counts

    def backward(self, gset, cam: dict, image, grad_image, grads, fp16: bool, dens=None, stream=None):
        g, gr = gaussians(gset), gaussians(grads)
        _check(self.lib.tgsref_backward(self.h, int(fp16), ctypes.byref(g), ctypes.byref(camera(cam)),
                                        c_void_p(image.data_ptr()), c_void_p(grad_image.data_ptr()),
                                        ctypes.byref(gr), c_void_p(dens.data_ptr() if dens is not None else 0),
                                        c_void_p(_stream(stream))), "tgsref_backward")

    def copy(self, which: int, dtype, count: int) -> np.ndarray:
        out = np.zeros(max(int(count), 0), dtype=dtype)
        if out.nbytes == 0:
            return out
        got = self.lib.tgsref_copy(self.h, int(which), out.ctypes.data_as(c_void_p), c_int64(out.nbytes))
        if got < 0:
            raise RuntimeError(f"tgsref_copy({which}) failed")
        return out[: got // out.itemsize]

    def ssim(self, fp16, width, height, pred, target, loss, grad, scale, stream=None):
        _check(self.lib.tgsref_ssim(self.h, int(fp16), int(width), int(height), c_void_p(pred.data_ptr()),
                                    c_void_p(target.data_ptr()), c_void_p(loss.data_ptr()),
                                    c_void_p(grad.data_ptr()), c_float(scale), c_void_p(_stream(stream))),
               "tgsref_ssim")


def l1(fp16, width, height, pred, target, loss, grad, scale, stream=None):
    _check(load().tgsref_l1(int(fp16), int(width), int(height), c_void_p(pred.data_ptr()),
                            c_void_p(target.data_ptr()), c_void_p(loss.data_ptr()), c_void_p(grad.data_ptr()),
                            c_float(scale), c_void_p(_stream(stream))), "tgsref_l1")


class RefAdam:
    """The reference's SimpleAdam over its own parameter and gradient
    containers (thrust vectors of n Gaussians, the reference's SoA layout)."""

    SEGMENTS = ("means", "opacities", "rotations", "scales", "sh0", "sh_rest")
    WIDTHS = {"means": 3, "opacities": 1, "rotations": 4, "scales": 3, "sh0": 3, "sh_rest": 45}

    def __init__(self, n: int, sh_degree: int, config: dict | None = None):
        import json

        self.lib = load()
        self.n = int(n)
        h = c_void_p()
        cfg = json.dumps(config or {}).encode()
        _check(self.lib.tgsref_adam_create(c_int64(self.n), c_int32(sh_degree), ctypes.c_char_p(cfg),
                                           ctypes.byref(h)), "tgsref_adam_create")
        self.h = h
        self.params, self.grads = RefGaussians(), RefGaussians()
        _check(self.lib.tgsref_adam_arrays(self.h, ctypes.byref(self.params), ctypes.byref(self.grads)),
               "tgsref_adam_arrays")

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            self.lib.tgsref_adam_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _view(self, s: RefGaussians, name: str):
        import torch

        from tinygs_b200.runtime import _DeviceView

        count = self.n * self.WIDTHS[name]
        return torch.as_tensor(_DeviceView(getattr(s, name), count, "<f4"), device="cuda")

    def param(self, name: str):
        """Device tensor view of a parameter array (flat, float32)."""
        return self._view(self.params, name)

    def grad(self, name: str):
        return self._view(self.grads, name)

    def step(self, gradient_scale: float, stream=None) -> None:
        _check(self.lib.tgsref_adam_step(self.h, c_float(gradient_scale), c_void_p(_stream(stream))),
               "tgsref_adam_step")
