"""Seeded synthetic scenes standing in for the reference's scenes.

No public dataset is named for this path and the reference's competition
scenes are absent, so the configurations of the benchmark are generated here
with the shapes and distributions the benchmark specifies (numpy PCG64,
fixed seeds, so every run and every machine sees the same data):

  cfg0  10k Gaussians, SH0, fp32, 256x256, fx=fy=300, camera at distance 3
  cfg1  500k, SH3, fp32, 1280x720, fx=fy=1000
  cfg2  3M, SH3, fp16 rasterizer, 1920x1080, fx=fy=1200, 60-view orbit r=4
  cfg3  1M (densifies towards 3M), SH3, fp32, 1280x720, 60-view orbit
  cfg4  6M, SH3, fp16, 1920x1080, 8 orbit views per step (one per GPU)

Parameter distributions: means U[-1,1]^3 (cfg0) or N(0, 1.5^2 I) (others);
log-scales N(-4, 0.5); quaternions N(0, I4) normalised, stored (w,x,y,z);
opacity logits N(0, 1); DC colour U[0,1] stored as (rgb-0.5)/C0 with
C0 = 0.28209479177387814; higher SH bands N(0, 0.1) (zero for SH0).
Cameras use the OpenCV convention (x right, y down, z forward).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

SH_C0 = 0.28209479177387814


@dataclass
class SceneConfig:
    name: str
    n: int
    sh_degree: int
    dtype: str  # "float32" | "float16" (rasterizer image type)
    width: int
    height: int
    focal: float
    cam_distance: float
    means: str  # "uniform" | "normal"
    views: int = 1
    seed: int = 0
    extra: dict = field(default_factory=dict)


CONFIGS = {
    "cfg0": SceneConfig("cfg0", 10_000, 0, "float32", 256, 256, 300.0, 3.0, "uniform", 1, 1000),
    "cfg1": SceneConfig("cfg1", 500_000, 3, "float32", 1280, 720, 1000.0, 4.0, "normal", 60, 1001),
    "cfg2": SceneConfig("cfg2", 3_000_000, 3, "float16", 1920, 1080, 1200.0, 4.0, "normal", 60, 1002),
    "cfg3": SceneConfig("cfg3", 1_000_000, 3, "float32", 1280, 720, 1000.0, 4.0, "normal", 60, 1003,
                        {"max_gaussians": 3_000_000, "refine_every": 100, "grad_threshold": 2e-4,
                         "prune_opacity": 0.005, "iterations": 3000}),
    "cfg4": SceneConfig("cfg4", 6_000_000, 3, "float16", 1920, 1080, 1200.0, 4.0, "normal", 8, 1004),
}


def gaussian_params(n: int, sh_degree: int, means: str, seed: int) -> dict[str, np.ndarray]:
    """Parameter arrays in the reference's SoA layout (float32, C order)."""
    rng = np.random.default_rng(seed)
    if means == "uniform":
        m = rng.uniform(-1.0, 1.0, size=(n, 3))
    else:
        m = rng.normal(0.0, 1.5, size=(n, 3))
    scales = rng.normal(-4.0, 0.5, size=(n, 3))
    q = rng.normal(0.0, 1.0, size=(n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    opac = rng.normal(0.0, 1.0, size=(n,))
    rgb = rng.uniform(0.0, 1.0, size=(n, 3))
    sh0 = (rgb - 0.5) / SH_C0
    rest = np.zeros((n, 15, 3))
    if sh_degree > 0:
        nb = (sh_degree + 1) ** 2 - 1
        rest[:, :nb, :] = rng.normal(0.0, 0.1, size=(n, nb, 3))
    f = np.float32
    return {"means": m.astype(f), "opacities": opac.astype(f), "rotations": q.astype(f),
            "scales": scales.astype(f), "sh0": sh0.astype(f), "sh_rest": rest.astype(f)}


def look_at_w2c(position, target=(0.0, 0.0, 0.0)) -> np.ndarray:
    """Row-major world-to-camera matrix of a camera at `position` looking at
    `target`, OpenCV axes (x right, y down, z forward), world y pointing down."""
    c = np.asarray(position, dtype=np.float64)
    z = np.asarray(target, dtype=np.float64) - c
    z /= np.linalg.norm(z)
    down = np.array([0.0, 1.0, 0.0])
    x = np.cross(down, z)
    if np.linalg.norm(x) < 1e-8:
        x = np.array([1.0, 0.0, 0.0])
    x /= np.linalg.norm(x)
    y = np.cross(z, x)
    R = np.stack([x, y, z])
    w2c = np.eye(4)
    w2c[:3, :3] = R
    w2c[:3, 3] = -R @ c
    return w2c.astype(np.float32)


def orbit_w2c(n_views: int, radius: float, seed: int, elevation: float = 0.35) -> list[np.ndarray]:
    """`n_views` cameras on a ring of the given radius around the origin, in a
    seeded order."""
    rng = np.random.default_rng(seed + 7)
    order = rng.permutation(n_views)
    out = []
    for k in order:
        th = 2.0 * np.pi * k / n_views
        pos = (radius * np.cos(th), -elevation * radius, radius * np.sin(th))
        out.append(look_at_w2c(pos))
    return out


def camera_dict(cfg: SceneConfig, w2c: np.ndarray, near: float = 0.01, far: float = 100.0) -> dict:
    return {"width": cfg.width, "height": cfg.height, "fx": cfg.focal, "fy": cfg.focal,
            "cx": cfg.width / 2.0, "cy": cfg.height / 2.0, "near": near, "far": far,
            "w2c": np.asarray(w2c, dtype=np.float32).reshape(16)}


def cameras(cfg: SceneConfig) -> list[dict]:
    if cfg.views == 1:
        return [camera_dict(cfg, look_at_w2c((0.0, 0.0, -cfg.cam_distance)))]
    return [camera_dict(cfg, w) for w in orbit_w2c(cfg.views, cfg.cam_distance, cfg.seed)]


def padded_hw(width: int, height: int) -> tuple[int, int]:
    return (height + 7) // 8 * 8, (width + 7) // 8 * 8


def target_image(width: int, height: int, seed: int, dtype=np.float32) -> np.ndarray:
    """Seeded U[0,1] target in the tiled CHW layout (values only, so any
    layout of U[0,1] noise is the same distribution; padding is zero)."""
    hp, wp = padded_hw(width, height)
    rng = np.random.default_rng(seed)
    img = rng.uniform(0.0, 1.0, size=(3, hp, wp)).astype(np.float32)
    img[:, height:, :] = 0.0
    img[:, :, width:] = 0.0
    return to_tiled(img).astype(dtype)


def to_tiled(img_chw: np.ndarray) -> np.ndarray:
    """[C][Hp][Wp] row-major -> the reference's 8x8-tiled CHW flat layout."""
    c, hp, wp = img_chw.shape
    t = img_chw.reshape(c, hp // 8, 8, wp // 8, 8).transpose(0, 1, 3, 2, 4)
    return np.ascontiguousarray(t).reshape(c, hp * wp)


def from_tiled(flat: np.ndarray, width: int, height: int) -> np.ndarray:
    """Inverse of to_tiled; returns [C][H][W] (padding dropped)."""
    hp, wp = padded_hw(width, height)
    c = flat.size // (hp * wp)
    t = np.asarray(flat).reshape(c, hp // 8, wp // 8, 8, 8).transpose(0, 1, 3, 2, 4)
    return np.ascontiguousarray(t).reshape(c, hp, wp)[:, :height, :width]
