"""numpy/ctypes front end of the CPU oracle (oracle/tgs_oracle.c).

TEST INFRASTRUCTURE ONLY -- imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline leg as the checker.  Parity status: pinned to the
reference's own kernels for the rasterizer and the losses through the golden
vectors in tests/golden/ (made by tests/golden/make_reference_golden.py from
oracle/_ref, the reference's CUDA sources built unchanged); the optimizer
and densification restatements are pinned by formula and published-vector
tests only (the reference ships no golden vectors for this path).
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int32, c_int64, c_uint8, c_uint16, c_uint32, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libtgs_oracle.so"


class OrcCamera(ctypes.Structure):
    _fields_ = [("width", c_int32), ("height", c_int32), ("fx", c_float), ("fy", c_float), ("cx", c_float),
                ("cy", c_float), ("near_plane", c_float), ("far_plane", c_float), ("w2c", c_float * 16)]


class OrcPrimitives(ctypes.Structure):
    _fields_ = [("n_touched", c_void_p), ("bounds", c_void_p), ("mean2d", c_void_p), ("conic_opacity", c_void_p),
                ("color", c_void_p), ("depth_key", c_void_p), ("fragile", c_void_p), ("prim_info", c_void_p)]


_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB.exists():
        from .build_oracle import build
        build()
    _lib = ctypes.CDLL(str(LIB))
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle buffers must be C-contiguous"
    return a.ctypes.data_as(c_void_p)


def set_fragile_f16(rel: float) -> None:
    """Width of the fp16 path's fragile band around the tile-test threshold
    (relative to max(|threshold|, 1)); rel <= 0 restores the default."""
    lib = load()
    lib.orc_set_fragile_f16.argtypes = [c_float]
    lib.orc_set_fragile_f16(float(rel))


def threads() -> int:
    return int(os.environ.get("TGS_ORACLE_THREADS", os.cpu_count() or 1))


def camera(cam: dict) -> OrcCamera:
    c = OrcCamera()
    c.width, c.height = int(cam["width"]), int(cam["height"])
    c.fx, c.fy, c.cx, c.cy = float(cam["fx"]), float(cam["fy"]), float(cam["cx"]), float(cam["cy"])
    c.near_plane, c.far_plane = float(cam.get("near", 0.01)), float(cam.get("far", 100.0))
    w = np.asarray(cam["w2c"], dtype=np.float32).reshape(16)
    for k in range(16):
        c.w2c[k] = float(w[k])
    return c


def grid(cam: dict) -> tuple[int, int]:
    return (int(cam["width"]) + 15) // 16, (int(cam["height"]) + 15) // 16


def plane(cam: dict) -> int:
    return ((int(cam["width"]) + 7) // 8 * 8) * ((int(cam["height"]) + 7) // 8 * 8)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def preprocess(params: dict, sh_degree: int, cam: dict, fp16: bool, dens: np.ndarray | None = None) -> dict:
    lib = load()
    n = params["means"].shape[0]
    out = {"n_touched": np.zeros(n, np.uint32), "bounds": np.zeros((n, 4), np.uint16),
           "mean2d": np.zeros((n, 2), np.float32), "conic_opacity": np.zeros((n, 4), np.float32),
           "color": np.zeros((n, 3), np.float32), "depth_key": np.zeros(n, np.uint32),
           "fragile": np.zeros(n, np.uint8), "prim_info": np.zeros((n, 16), np.uint8) if fp16 else None}
    prim = OrcPrimitives(*[_p(out[k]) for k in ("n_touched", "bounds", "mean2d", "conic_opacity", "color",
                                                "depth_key", "fragile", "prim_info")])
    c = camera(cam)
    arrs = [_f32(params[k]) for k in ("means", "opacities", "rotations", "scales", "sh0", "sh_rest")]
    lib.orc_preprocess(c_int64(n), *[_p(a) for a in arrs], c_int32(sh_degree), ctypes.byref(c), c_int32(int(fp16)),
                       ctypes.byref(prim), _p(dens), c_int32(threads()))
    out["_keep"] = (arrs, prim)
    return out


def prim_struct(prims: dict):
    """OrcPrimitives over the arrays of a primitives dict (oracle- or
    GPU-produced); returns the struct and the arrays it points into."""
    keys = ("n_touched", "bounds", "mean2d", "conic_opacity", "color", "depth_key", "fragile", "prim_info")
    dtypes = {"n_touched": np.uint32, "bounds": np.uint16, "mean2d": np.float32, "conic_opacity": np.float32,
              "color": np.float32, "depth_key": np.uint32, "fragile": np.uint8, "prim_info": np.uint8}
    arrs = []
    for k in keys:
        a = prims.get(k)
        arrs.append(None if a is None else np.ascontiguousarray(a, dtype=dtypes[k]))
    return OrcPrimitives(*[_p(a) for a in arrs]), arrs


def count_tiles(prims: dict, cam: dict, fp16: bool, band: float = 0.0):
    """Per-Gaussian touched-tile counts recomputed from the screen-space
    records in `prims` (the decision create_instances repeats).  With
    band > 0, returns (counts, fragile) where fragile flags a tile test
    within `band` of its threshold (relative to max(|threshold|, 1))."""
    lib = load()
    st, keep = prim_struct(prims)
    n = prims["n_touched"].shape[0]
    out = np.zeros(n, np.uint32)
    fr = np.zeros(n, np.uint8)
    c = camera(cam)
    lib.orc_count_tiles(c_int64(n), ctypes.byref(st), ctypes.byref(c), c_int32(int(fp16)), _p(out), _p(fr),
                        c_float(band), c_int32(threads()))
    return (out, fr) if band > 0 else out


def pixel_fragile(cam: dict, band: float):
    """Starts recording blend decisions within `band` (relative) of their
    thresholds; returns the per-pixel flag array the next blend forwards
    fill.  pixel_fragile_off() stops it."""
    buf = np.zeros(plane(cam), np.uint8)
    load().orc_set_pixel_fragile(_p(buf), c_float(band))
    return buf


def pixel_fragile_off() -> None:
    load().orc_set_pixel_fragile(None, c_float(0.0))


def binning(prims: dict, cam: dict, fp16: bool, cap: int | None = None) -> dict:
    lib = load()
    lib.orc_binning.restype = c_int64
    n = prims["n_touched"].shape[0]
    total = int(prims["n_touched"].astype(np.int64).sum())
    cap = total if cap is None else cap
    gw, gh = grid(cam)
    inst_tile = np.zeros(max(cap, 1), np.uint32)
    inst_prim = np.zeros(max(cap, 1), np.uint32)
    ranges = np.zeros((gw * gh, 2), np.uint32)
    sorted_vis = np.zeros(max(n, 1), np.uint32)
    nvis = c_uint32(0)
    c = camera(cam)
    prim, _refs = prim_struct(prims)
    ni = lib.orc_binning(c_int64(n), ctypes.byref(prim), ctypes.byref(c), c_int32(int(fp16)), _p(inst_tile),
                         _p(inst_prim), c_int64(cap), _p(ranges), _p(sorted_vis), ctypes.byref(nvis))
    if ni < 0:
        raise RuntimeError("oracle binning capacity exceeded")
    offs = np.zeros(gw * gh, np.uint32)
    lib.orc_bucket_offsets.restype = c_int64
    nb = lib.orc_bucket_offsets(_p(ranges), c_int32(gw * gh), _p(offs))
    return {"inst_tile": inst_tile[:ni], "inst_prim": inst_prim[:ni], "ranges": ranges, "n_instances": int(ni),
            "sorted_visible": sorted_vis[: nvis.value], "n_visible": int(nvis.value),
            "bucket_offsets": offs, "n_buckets": int(nb)}


def blend_forward(prims: dict, bins: dict, cam: dict, fp16: bool) -> dict:
    lib = load()
    c = camera(cam)
    gw, gh = grid(cam)
    pl = plane(cam)
    nb = max(bins["n_buckets"], 1)
    inst_prim = np.ascontiguousarray(bins["inst_prim"]) if bins["n_instances"] else np.zeros(1, np.uint32)
    if fp16:
        image = np.zeros(3 * pl, np.uint16)
        alpha = np.zeros(pl, np.uint16)
        ncon = np.zeros(pl, np.uint16)
        tmax = np.zeros(gw * gh, np.uint16)
        ckpt = np.zeros(nb * 256 * 4, np.uint16)
        lib.orc_blend_forward_f16(ctypes.byref(c), _p(bins["ranges"]), _p(inst_prim), _p(prims["mean2d"]),
                                  _p(prims["prim_info"]), _p(image), _p(alpha), _p(ncon), _p(tmax),
                                  _p(bins["bucket_offsets"]), _p(ckpt), c_int32(threads()))
        return {"image": image.view(np.float16), "alpha": alpha.view(np.float16), "n_contrib": ncon,
                "tile_max": tmax, "ckpt": ckpt}
    image = np.zeros(3 * pl, np.float32)
    alpha = np.zeros(pl, np.float32)
    ncon = np.zeros(pl, np.uint32)
    tmax = np.zeros(gw * gh, np.uint32)
    ckpt = np.zeros(nb * 256 * 4, np.float32)
    lib.orc_blend_forward_f32(ctypes.byref(c), _p(bins["ranges"]), _p(inst_prim), _p(prims["mean2d"]),
                              _p(prims["conic_opacity"]), _p(prims["color"]), _p(image), _p(alpha), _p(ncon),
                              _p(tmax), _p(bins["bucket_offsets"]), _p(ckpt), c_int32(threads()))
    return {"image": image, "alpha": alpha, "n_contrib": ncon, "tile_max": tmax, "ckpt": ckpt}


def blend_backward(prims: dict, bins: dict, fwd: dict, grad_image: np.ndarray, cam: dict, fp16: bool) -> dict:
    """Per-Gaussian screen-space gradients (the blend backward's outputs)."""
    lib = load()
    c = camera(cam)
    n = prims["n_touched"].shape[0]
    gm = np.zeros((n, 2), np.float32)
    ag = np.zeros((n, 2), np.float32)
    go = np.zeros(n, np.float32)
    gc = np.zeros((n, 3), np.float32)
    inst_prim = np.ascontiguousarray(bins["inst_prim"]) if bins["n_instances"] else np.zeros(1, np.uint32)
    if fp16:
        gconic = np.zeros((n, 3), np.float32)
        lib.orc_blend_backward_f16(ctypes.byref(c), c_int64(n), _p(bins["ranges"]), _p(inst_prim),
                                   _p(prims["mean2d"]), _p(prims["prim_info"]),
                                   _p(np.ascontiguousarray(fwd["image"]).view(np.uint16)),
                                   _p(np.ascontiguousarray(grad_image, dtype=np.float16).view(np.uint16)),
                                   _p(fwd["tile_max"]), _p(bins["bucket_offsets"]), _p(fwd["ckpt"]), _p(gm), _p(ag),
                                   _p(gconic), _p(go), _p(gc), c_int32(threads()))
    else:
        gsoa = np.zeros((3, n), np.float32)
        lib.orc_blend_backward_f32(ctypes.byref(c), c_int64(n), _p(bins["ranges"]), _p(inst_prim),
                                   _p(prims["mean2d"]), _p(prims["conic_opacity"]), _p(prims["color"]),
                                   _p(fwd["image"]), _p(_f32(grad_image)), _p(fwd["n_contrib"]), _p(fwd["tile_max"]),
                                   _p(bins["bucket_offsets"]), _p(fwd["ckpt"]), _p(gm), _p(ag), _p(gsoa), _p(go),
                                   _p(gc), c_int32(threads()))
        gconic = np.ascontiguousarray(gsoa.T)
    return {"grad_mean2d": gm, "absgrad_mean2d": ag, "grad_conic": gconic, "grad_opacity": go, "grad_color": gc}


def preprocess_backward(params: dict, sh_degree: int, cam: dict, n_touched: np.ndarray, screen: dict,
                        grads: dict | None = None, dens: np.ndarray | None = None) -> dict:
    """Parameter gradients from the screen-space ones; accumulates into
    `grads` (zeros if None).  The opacity gradient passes straight through."""
    lib = load()
    n = params["means"].shape[0]
    if grads is None:
        grads = {"means": np.zeros((n, 3), np.float32), "opacities": np.zeros(n, np.float32),
                 "rotations": np.zeros((n, 4), np.float32), "scales": np.zeros((n, 3), np.float32),
                 "sh0": np.zeros((n, 3), np.float32), "sh_rest": np.zeros((n, 15, 3), np.float32)}
    c = camera(cam)
    keep = [_f32(params[k]) for k in ("means", "rotations", "scales", "sh_rest")]
    conic = np.ascontiguousarray(screen["grad_conic"], dtype=np.float32)
    lib.orc_preprocess_backward(c_int64(n), *[_p(a) for a in keep], c_int32(sh_degree), ctypes.byref(c),
                                _p(np.ascontiguousarray(n_touched, dtype=np.uint32)),
                                _p(_f32(screen["grad_mean2d"])), _p(conic), c_int32(0),
                                _p(_f32(screen["absgrad_mean2d"])), _p(_f32(screen["grad_color"])),
                                _p(grads["means"]), _p(grads["rotations"]), _p(grads["scales"]), _p(grads["sh0"]),
                                _p(grads["sh_rest"]), _p(dens), c_int32(threads()))
    touched = np.asarray(n_touched) > 0
    grads["opacities"][touched] += screen["grad_opacity"][touched]
    return grads


def l1(pred, target, loss_map, grad, width, height, scale):
    lib = load()
    if pred.dtype == np.float16:
        lib.orc_l1_f16(c_int32(width), c_int32(height), _p(pred.view(np.uint16)), _p(target.view(np.uint16)),
                       _p(None if loss_map is None else loss_map.view(np.uint16)),
                       _p(None if grad is None else grad.view(np.uint16)), c_float(scale))
    else:
        lib.orc_l1_f32(c_int32(width), c_int32(height), _p(pred), _p(target), _p(loss_map), _p(grad), c_float(scale))


def ssim(pred, target, loss_map, grad, width, height, scale):
    lib = load()
    if pred.dtype == np.float16:
        lib.orc_ssim_f16(c_int32(width), c_int32(height), _p(pred.view(np.uint16)), _p(target.view(np.uint16)),
                         _p(None if loss_map is None else loss_map.view(np.uint16)),
                         _p(None if grad is None else grad.view(np.uint16)), c_float(scale), c_int32(threads()))
    else:
        lib.orc_ssim_f32(c_int32(width), c_int32(height), _p(pred), _p(target), _p(loss_map), _p(grad),
                         c_float(scale), c_int32(threads()))


def adam(theta, grad, m, v, lr, beta1, beta2, eps, gscale, bc1, bc2_sqrt, max_g, decay_kind=0, decay=0.0):
    lib = load()
    lib.orc_adam(c_int64(theta.size), _p(theta), _p(_f32(grad)), _p(m), _p(v), c_float(lr), c_float(beta1),
                 c_float(beta2), c_float(eps), c_float(gscale), c_float(bc1), c_float(bc2_sqrt), c_float(max_g),
                 c_int32(decay_kind), c_float(decay))


def adam_step(params: dict, grads: dict, m: dict, v: dict, cfg, step: int, gradient_scale: float) -> None:
    """SimpleAdam::step_adam on numpy dicts (in place), simple_adam.cu:457-580."""
    bc1 = np.float32(1.0 - cfg.beta1 ** step)
    bc2 = np.float32(np.sqrt(1.0 - cfg.beta2 ** step))
    n = params["means"].shape[0]
    gs = 1.0 / n if cfg.decay_reduction_mean else 1.0
    table = [("means", cfg.means_lr * cfg.scene_scale * cfg.global_lr, 0, 0.0),
             ("opacities", cfg.opacities_lr * cfg.global_lr, 1, cfg.opacities_l1 * gs),
             ("rotations", cfg.rotations_lr * cfg.global_lr, 0, 0.0),
             ("scales", cfg.scales_lr * cfg.global_lr, 2, cfg.scales_l1 * gs),
             ("sh0", cfg.shs_lr * cfg.global_lr, 0, 0.0),
             ("sh_rest", np.float32(cfg.shs_lr) * np.float32(0.05) * np.float32(cfg.global_lr), 0, 0.0)]
    for name, lr, kind, decay in table:
        adam(params[name], grads[name], m[name], v[name], np.float32(lr), cfg.beta1, cfg.beta2, cfg.epsilon,
             gradient_scale, bc1, bc2, cfg.max_grad_1, kind if decay != 0.0 else 0, decay)


def render(params: dict, sh_degree: int, cam: dict, fp16: bool) -> dict:
    prims = preprocess(params, sh_degree, cam, fp16)
    bins = binning(prims, cam, fp16)
    fwd = blend_forward(prims, bins, cam, fp16)
    return {"prims": prims, "bins": bins, "fwd": fwd}


def train_step(params: dict, sh_degree: int, cam: dict, target: np.ndarray, fp16: bool, adam_cfg=None,
               moments=None, step: int = 1, grad_scaler: float = 10.0, w_l1: float = 0.8,
               w_ssim: float = 0.2, do_adam: bool = True) -> dict:
    """One Orchestrator::train_step (orchestrator.cu:335-439) on the CPU:
    forward, 0.8 L1 + 0.2 (1-SSIM) scaled by grad_scaler, backward, Adam with
    gradient scale 1/grad_scaler.  Mutates params (and moments) in place."""
    W, H = int(cam["width"]), int(cam["height"])
    r = render(params, sh_degree, cam, fp16)
    img = r["fwd"]["image"]
    dt = np.float16 if fp16 else np.float32
    loss_map = np.zeros(img.shape, dt)
    grad_img = np.zeros(img.shape, dt)
    l1(img, target.astype(dt), loss_map, grad_img, W, H, w_l1 * grad_scaler)
    ssim(img, target.astype(dt), loss_map, grad_img, W, H, w_ssim * grad_scaler)
    screen = blend_backward(r["prims"], r["bins"], r["fwd"], grad_img, cam, fp16)
    grads = preprocess_backward(params, sh_degree, cam, r["prims"]["n_touched"], screen)
    out = {"render": r, "loss_map": loss_map, "grad_image": grad_img, "screen": screen, "grads": grads}
    if do_adam:
        from types import SimpleNamespace
        cfg = adam_cfg or SimpleNamespace(beta1=0.9, beta2=0.999, epsilon=1e-8, max_grad_1=0.3, means_lr=1.6e-4,
                                          shs_lr=2.5e-3, opacities_lr=5e-2, scales_lr=5e-3, rotations_lr=1e-3,
                                          opacities_l1=0.0, scales_l1=0.0, scene_scale=1.0, global_lr=1.0,
                                          decay_reduction_mean=True)
        if moments is None:
            moments = ({k: np.zeros_like(v) for k, v in params.items()}, {k: np.zeros_like(v) for k, v in params.items()})
        adam_step(params, grads, moments[0], moments[1], cfg, step, 1.0 / grad_scaler)
        out["moments"] = moments
    return out


# ------------------------------------------------------------ densification

class OrcPcg32(ctypes.Structure):
    _fields_ = [("state", ctypes.c_uint64), ("inc", ctypes.c_uint64)]


class OrcSet(ctypes.Structure):
    _fields_ = [("means", c_void_p), ("opacities", c_void_p), ("rotations", c_void_p), ("scales", c_void_p),
                ("sh0", c_void_p), ("sh_rest", c_void_p)]


class OrcDensifyConfig(ctypes.Structure):
    _fields_ = [("duplicate_grad_threshold", c_float), ("duplicate_scale_threshold", c_float),
                ("pruning_opacity_threshold", c_float), ("pruning_scale_threshold", c_float),
                ("max_screen_size", c_float), ("scene_scale", c_float), ("grad_scaler", c_float),
                ("absgrad", c_int32), ("refine_every", c_int32), ("start_refine", c_int32),
                ("end_refine", c_int32), ("reset_every", c_int32), ("image_width", c_int32),
                ("image_height", c_int32), ("_pad", c_int32), ("max_num_gaussians", c_int64)]


SEGMENT_WIDTHS = {"means": 3, "opacities": 1, "rotations": 4, "scales": 3, "sh0": 3, "sh_rest": 45}


def _densify_protos(lib):
    lib.orc_pcg32_seed.argtypes = [POINTER(OrcPcg32), ctypes.c_uint64, ctypes.c_uint64]
    lib.orc_pcg32_next_uint.restype = c_uint32
    lib.orc_pcg32_next_uint.argtypes = [POINTER(OrcPcg32)]
    lib.orc_pcg32_next_float.restype = c_float
    lib.orc_pcg32_next_float.argtypes = [POINTER(OrcPcg32)]
    lib.orc_pcg32_advance.argtypes = [POINTER(OrcPcg32), ctypes.c_uint64]
    lib.orc_random_logistic.argtypes = [POINTER(OrcPcg32), c_int64, c_void_p]
    lib.orc_densify_step.restype = c_int64
    lib.orc_densify_step.argtypes = [c_int64, c_int64, OrcSet, OrcSet, OrcSet, OrcSet, c_void_p,
                                     POINTER(OrcDensifyConfig), c_int32, POINTER(OrcPcg32)]
    return lib


def pcg32(seed: int, seq: int = 1) -> OrcPcg32:
    lib = _densify_protos(load())
    r = OrcPcg32()
    lib.orc_pcg32_seed(ctypes.byref(r), seed, seq)
    return r


def pcg32_next_uint(r: OrcPcg32, count: int) -> np.ndarray:
    lib = _densify_protos(load())
    return np.array([lib.orc_pcg32_next_uint(ctypes.byref(r)) for _ in range(count)], np.uint32)


def pcg32_advance(r: OrcPcg32, delta: int) -> None:
    _densify_protos(load()).orc_pcg32_advance(ctypes.byref(r), delta)


def random_logistic(r: OrcPcg32, n: int) -> np.ndarray:
    lib = _densify_protos(load())
    out = np.zeros(max(n, 1), np.float32)
    lib.orc_random_logistic(ctypes.byref(r), n, _p(out))
    return out[:n]


def densify_config(**kw) -> OrcDensifyConfig:
    c = OrcDensifyConfig(duplicate_grad_threshold=2e-4, duplicate_scale_threshold=0.01,
                         pruning_opacity_threshold=0.005, pruning_scale_threshold=0.1, max_screen_size=10.0,
                         scene_scale=1.0, grad_scaler=10.0, absgrad=0, refine_every=100, start_refine=500,
                         end_refine=15000, reset_every=3000, image_width=1280, image_height=720,
                         max_num_gaussians=10_000_000)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def _set_of(arrays: dict | None) -> OrcSet:
    s = OrcSet()
    if arrays is not None:
        for k in SEGMENT_WIDTHS:
            setattr(s, k, arrays[k].ctypes.data)
    return s


def alloc_set(capacity: int, init: dict | None = None) -> dict:
    """Arrays of `capacity` Gaussians (the first rows copied from `init`)."""
    out = {k: np.zeros((capacity, w), np.float32) for k, w in SEGMENT_WIDTHS.items()}
    if init is not None:
        for k, w in SEGMENT_WIDTHS.items():
            a = np.asarray(init[k], np.float32).reshape(-1, w)
            out[k][: a.shape[0]] = a
    return out


def densify_step(n: int, params: dict, grads: dict | None, m: dict, v: dict, dens: np.ndarray,
                 cfg: OrcDensifyConfig, step: int, rng: OrcPcg32) -> int:
    """DefaultStrategy::step_impl on capacity-sized arrays (in place); returns
    the new count (-1 when the growth would pass the capacity)."""
    lib = _densify_protos(load())
    cap = params["means"].shape[0]
    return int(lib.orc_densify_step(n, cap, _set_of(params), _set_of(grads), _set_of(m), _set_of(v),
                                    _p(dens), ctypes.byref(cfg), step, ctypes.byref(rng)))


def morton_order(means: np.ndarray) -> np.ndarray:
    """The reference's Morton order of the means (orchestrator.cu:26-100)."""
    lib = load()
    m = np.ascontiguousarray(means, dtype=np.float32).reshape(-1, 3)
    perm = np.zeros(max(m.shape[0], 1), np.uint32)
    lib.orc_morton_order(c_int64(m.shape[0]), _p(m), _p(perm))
    return perm[: m.shape[0]]
