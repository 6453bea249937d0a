"""ctypes binding of ``include/tgs_abi.h``.

This module only describes the C structs and function prototypes and loads
``libtgs_b200.so``; it never falls back to anything else.  Loading the library
does not touch the GPU (the CUDA runtime is linked statically and initialised
lazily), so the export check runs on machines without one.
"""
from __future__ import annotations

import ctypes
import re
from ctypes import POINTER, c_char_p, c_float, c_int32, c_int64, c_size_t, c_uint32, c_uint64, c_void_p
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libtgs_b200.so"
HEADER = PKG.parent / "include" / "tgs_abi.h"

TGS_OK = 0
TGS_ERR_INVALID_ARGUMENT = 1
TGS_ERR_CUDA = 2
TGS_ERR_CAPACITY = 3
TGS_ERR_OUT_OF_MEMORY = 4
TGS_ERR_NO_FORWARD = 5
TGS_ERR_UNSUPPORTED = 6
TGS_ERR_DEVICE_TIMEOUT = 7

TGS_FLOAT32 = 0
TGS_FLOAT16 = 1
TGS_UINT8 = 2
TGS_IMAGE_TILED_CHW = 0
TGS_IMAGE_HWC = 1
TGS_NOALLOC_MAX_PIXELS = 262144


class TgsGaussians(ctypes.Structure):
    _fields_ = [("means", c_void_p), ("opacities", c_void_p), ("rotations", c_void_p), ("scales", c_void_p),
                ("sh0", c_void_p), ("sh_rest", c_void_p), ("n", c_int64), ("sh_degree", c_int32),
                ("_pad", c_int32)]


class TgsCamera(ctypes.Structure):
    _fields_ = [("width", c_int32), ("height", c_int32), ("fx", c_float), ("fy", c_float), ("cx", c_float),
                ("cy", c_float), ("near_plane", c_float), ("far_plane", c_float), ("w2c", c_float * 16)]


class TgsRasterCaps(ctypes.Structure):
    _fields_ = [("max_gaussians", c_int64), ("max_width", c_int32), ("max_height", c_int32),
                ("max_instances", c_int64)]


class TgsRasterCounts(ctypes.Structure):
    _fields_ = [("n_visible", c_uint32), ("n_instances", c_uint32), ("n_buckets", c_uint32),
                ("overflow", c_uint32)]


class TgsAdamConfig(ctypes.Structure):
    _fields_ = [("beta1", c_float), ("beta2", c_float), ("epsilon", c_float), ("max_grad_1", c_float),
                ("means_lr", c_float), ("shs_lr", c_float), ("opacities_lr", c_float), ("scales_lr", c_float),
                ("rotations_lr", c_float), ("opacities_l1", c_float), ("scales_l1", c_float),
                ("scene_scale", c_float), ("global_lr", c_float), ("decay_reduction_mean", c_int32)]


class TgsDensifyConfig(ctypes.Structure):
    _fields_ = [("duplicate_grad_threshold", c_float), ("duplicate_scale_threshold", c_float),
                ("pruning_opacity_threshold", c_float), ("pruning_scale_threshold", c_float),
                ("max_screen_size", c_float), ("scene_scale", c_float), ("grad_scaler", c_float),
                ("absgrad", c_int32), ("refine_every", c_int32), ("start_refine", c_int32),
                ("end_refine", c_int32), ("reset_every", c_int32), ("image_width", c_int32),
                ("image_height", c_int32), ("_pad", c_int32), ("max_num_gaussians", c_int64)]


class TgsPcg32(ctypes.Structure):
    _fields_ = [("state", c_uint64), ("inc", c_uint64)]


class TgsTrainState(ctypes.Structure):
    _fields_ = [("step", c_uint64), ("adam_step", c_uint64), ("strategy_step", c_uint64), ("rng", TgsPcg32)]


class TgsIpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]

    def raw(self) -> bytes:
        return ctypes.string_at(ctypes.addressof(self), ctypes.sizeof(self))

    @classmethod
    def from_raw(cls, data: bytes) -> "TgsIpcHandle":
        h = cls()
        ctypes.memmove(ctypes.addressof(h), data, min(len(data), ctypes.sizeof(h)))
        return h


_P = c_void_p
PROTOTYPES = {
    "tgs_raster_create": (c_int32, [POINTER(TgsRasterCaps), POINTER(c_void_p)]),
    "tgs_raster_destroy": (c_int32, [_P]),
    "tgs_raster_workspace_bytes": (c_int32, [_P, POINTER(c_size_t)]),
    "tgs_raster_forward": (c_int32, [_P, POINTER(TgsGaussians), POINTER(TgsCamera), c_int32, _P, _P, _P, _P]),
    "tgs_raster_backward": (c_int32, [_P, POINTER(TgsGaussians), POINTER(TgsCamera), c_int32, _P, _P,
                                      POINTER(TgsGaussians), c_int32, _P, _P]),
    "tgs_raster_backward_adam": (c_int32, [_P, POINTER(TgsGaussians), POINTER(TgsCamera), c_int32, _P, _P,
                                           POINTER(TgsGaussians), POINTER(TgsGaussians), POINTER(TgsGaussians),
                                           POINTER(TgsAdamConfig), c_uint32, c_float, _P, _P]),
    "tgs_raster_counts": (c_int32, [_P, POINTER(TgsRasterCounts), _P]),
    "tgs_raster_set_stage_timing": (c_int32, [_P, c_int32]),
    "tgs_raster_stage_times": (c_int32, [_P, POINTER(c_float)]),
    "tgs_raster_debug_buffer": (c_int32, [_P, c_int32, POINTER(c_void_p), POINTER(c_size_t)]),
    "tgs_loss_l1": (c_int32, [c_int32, c_int32, c_int32, _P, _P, _P, _P, c_float, _P]),
    "tgs_loss_create": (c_int32, [c_int32, c_int32, POINTER(c_void_p)]),
    "tgs_loss_destroy": (c_int32, [_P]),
    "tgs_loss_fused_ssim": (c_int32, [_P, c_int32, c_int32, c_int32, _P, _P, _P, _P, c_float, _P]),
    "tgs_loss_l1_ssim": (c_int32, [_P, c_int32, c_int32, c_int32, _P, _P, _P, _P, c_float, c_float, _P, _P]),
    "tgs_loss_l1_ssim_noalloc": (c_int32, [c_int32, c_int32, c_int32, _P, _P, _P, _P, c_float, c_float, _P, _P]),
    "tgs_adam_step": (c_int32, [POINTER(TgsGaussians), POINTER(TgsGaussians), POINTER(TgsGaussians),
                                POINTER(TgsGaussians), POINTER(TgsAdamConfig), c_uint32, c_float, c_int32, _P]),
    "tgs_gaussians_zero": (c_int32, [POINTER(TgsGaussians), _P]),
    "tgs_pcg32_seed": (None, [POINTER(TgsPcg32), c_uint64, c_uint64]),
    "tgs_shared_alloc": (c_int32, [c_size_t, POINTER(c_void_p), POINTER(TgsIpcHandle)]),
    "tgs_shared_free": (c_int32, [_P]),
    "tgs_shared_open": (c_int32, [POINTER(TgsIpcHandle), POINTER(c_void_p)]),
    "tgs_shared_close": (c_int32, [_P]),
    "tgs_raster_backward_routed": (c_int32, [_P, POINTER(TgsGaussians), POINTER(TgsCamera), c_int32, _P, _P,
                                             POINTER(c_void_p), c_int64, c_int32, c_int32, _P, _P]),
    "tgs_dp_inbox_adam": (c_int32, [POINTER(TgsGaussians), _P, c_int64, c_int32, c_int32, POINTER(TgsGaussians),
                                    POINTER(TgsGaussians), POINTER(TgsAdamConfig), c_uint32, c_float, _P]),
    "tgs_dp_reduce_adam_multicast": (c_int32, [POINTER(TgsGaussians), POINTER(TgsGaussians), POINTER(TgsGaussians),
                                               c_int32, c_int32, POINTER(TgsGaussians), POINTER(TgsGaussians),
                                               POINTER(TgsAdamConfig), c_uint32, c_float, _P]),
    "tgs_dp_reduce_adam": (c_int32, [POINTER(TgsGaussians), POINTER(TgsGaussians), c_int32, c_int32,
                                     POINTER(TgsGaussians), POINTER(TgsGaussians), POINTER(TgsAdamConfig), c_uint32,
                                     c_float, _P]),
    "tgs_densify_create": (c_int32, [c_int64, POINTER(c_void_p)]),
    "tgs_densify_destroy": (c_int32, [_P]),
    "tgs_densify_step": (c_int32, [_P, POINTER(TgsGaussians), POINTER(TgsGaussians), POINTER(TgsGaussians),
                                   POINTER(TgsGaussians), _P, POINTER(TgsDensifyConfig), c_int32, POINTER(TgsPcg32),
                                   POINTER(c_int64), _P]),
    "tgs_arena_gather": (c_int32, [POINTER(TgsGaussians), POINTER(TgsGaussians), _P, c_int64, _P]),
    "tgs_arena_compact_workspace_bytes": (c_int32, [c_int64, POINTER(c_size_t)]),
    "tgs_arena_keep_index": (c_int32, [_P, c_int64, _P, c_size_t, _P, _P, _P]),
    "tgs_arena_compact": (c_int32, [POINTER(TgsGaussians), POINTER(TgsGaussians), _P, c_int64, _P, c_size_t, _P,
                                    _P]),
    "tgs_arena_fill_rows": (c_int32, [POINTER(TgsGaussians), _P, c_int64, c_float, c_int32, _P]),
    "tgs_dens_gather": (c_int32, [_P, _P, _P, c_int64, _P]),
    "tgs_morton_workspace_bytes": (c_int32, [c_int64, POINTER(c_size_t)]),
    "tgs_morton_order": (c_int32, [_P, c_int64, _P, c_size_t, _P, _P]),
    "tgs_metric_psnr": (c_int32, [c_int32, c_int32, c_int32, _P, _P, _P, _P, _P]),
    "tgs_image_from_u8": (c_int32, [_P, c_int32, c_int32, c_int32, c_int32, _P, c_int32, _P]),
    "tgs_image_resize_u8": (c_int32, [_P, c_int32, c_int32, c_int32, _P, c_int32, c_int32, c_int32, _P, _P]),
    "tgs_image_blur_state_init": (c_int32, [_P, c_int64, c_uint64, _P]),
    "tgs_checkpoint_save": (c_int32, [c_char_p, POINTER(TgsGaussians), POINTER(TgsGaussians), POINTER(TgsGaussians),
                                      _P, POINTER(TgsTrainState), _P]),
    "tgs_checkpoint_info": (c_int32, [c_char_p, POINTER(c_int64), POINTER(c_int32), POINTER(c_uint32),
                                      POINTER(TgsTrainState)]),
    "tgs_checkpoint_load": (c_int32, [c_char_p, c_int64, POINTER(TgsGaussians), POINTER(TgsGaussians),
                                      POINTER(TgsGaussians), _P, POINTER(TgsTrainState), _P]),
    "tgs_raster_share": (c_int32, [_P, POINTER(TgsIpcHandle)]),
    "tgs_raster_arena": (c_int32, [_P, POINTER(c_void_p)]),
    "tgs_raster_attach_views": (c_int32, [_P, POINTER(c_void_p), c_int32, c_int32]),
    "tgs_raster_preprocess_views": (c_int32, [_P, POINTER(TgsGaussians), POINTER(TgsCamera), c_int32, c_int64,
                                              c_int64, _P, _P]),
    "tgs_raster_forward_gathered": (c_int32, [_P, c_int64, POINTER(TgsCamera), c_int32, _P, _P, _P]),
    "tgs_raster_backward_screen": (c_int32, [_P, POINTER(TgsCamera), c_int32, _P, _P, c_int32, _P]),
    "tgs_raster_backward_views_adam": (c_int32, [_P, POINTER(TgsGaussians), POINTER(TgsCamera), c_int64, c_int64,
                                                 POINTER(TgsGaussians), POINTER(TgsGaussians), POINTER(TgsGaussians),
                                                 POINTER(TgsAdamConfig), c_uint32, c_float, _P, _P]),
    "tgs_status_string": (c_char_p, [c_int32]),
    "tgs_loss_set_accumulate": (c_int32, [c_void_p, c_int32]),
    "tgs_version": (c_char_p, []),
}

_lib = None


def header_symbols(header: Path = HEADER) -> list[str]:
    """Names of every function ``include/tgs_abi.h`` declares."""
    text = header.read_text()
    return sorted(set(re.findall(r"TGS_API\s+[\w\s\*]*?\b(tgs_\w+)\s*\(", text)))


def load_library(path: Path | str | None = None) -> ctypes.CDLL:
    """Load libtgs_b200.so and attach the prototypes.  Raises if it is missing:
    there is no fallback implementation."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"{p} is missing; build it with `python -m tinygs_b200.build` "
                           "(tinygs_b200 has no non-CUDA fallback)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


class TgsError(RuntimeError):
    def __init__(self, status: int, where: str):
        lib = _lib
        msg = lib.tgs_status_string(status).decode() if lib is not None else str(status)
        super().__init__(f"{where}: {msg} (status {status})")
        self.status = status


def check(status: int, where: str) -> None:
    if status != TGS_OK:
        raise TgsError(status, where)
