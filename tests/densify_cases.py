"""Seeded inputs for the densification tests: parameters, moments, gradients
and densification statistics whose values keep every decision (grow,
split or clone, each prune test) far from its threshold, so that the CUDA
path and the oracle take the same decisions whatever their last-bit
arithmetic differences."""
from __future__ import annotations

import numpy as np

WIDTHS = {"means": 3, "opacities": 1, "rotations": 4, "scales": 3, "sh0": 3, "sh_rest": 45}


def make_case(n: int, seed: int = 7, grad_scaler: float = 10.0):
    rng = np.random.default_rng(seed)
    f = np.float32
    params = {
        "means": rng.normal(0, 1, (n, 3)).astype(f),
        # logit -7 (sigmoid 0.0009, pruned) or around 0 (kept); threshold 0.005 ~ logit -5.29
        "opacities": np.where(rng.random(n) < 0.15, -7.0, rng.normal(0.0, 1.0, n)).astype(f).reshape(n, 1),
        "rotations": rng.normal(0, 1, (n, 4)).astype(f),
        # exp(-6) = 0.0025 (clone), exp(-3) = 0.05 (split), exp(-1) = 0.37 (large in world space)
        "scales": np.stack([rng.choice([-6.0, -3.0, -1.0], size=n, p=[0.5, 0.4, 0.1]) + rng.normal(0, 0.1, n)
                            for _ in range(3)], 1).astype(f),
        "sh0": rng.normal(0, 0.5, (n, 3)).astype(f),
        "sh_rest": rng.normal(0, 0.1, (n, 45)).astype(f),
    }
    degenerate = rng.random(n) < 0.02
    params["rotations"][degenerate] = 0.0
    moments = [{k: rng.normal(0, 1e-3, (n, w)).astype(f) for k, w in WIDTHS.items()} for _ in range(2)]
    moments[1] = {k: np.abs(v) for k, v in moments[1].items()}
    grads = {k: rng.normal(0, 1e-2, (n, w)).astype(f) for k, w in WIDTHS.items()}
    # densification records: counter, accumulated |grad|, accumulated absgrad, max radius
    thr = 2e-4 * grad_scaler
    counter = rng.integers(0, 6, n).astype(f)
    ratio = np.where(rng.random(n) < 0.3, 3.0, 0.3) * thr  # well above or below the threshold
    dens = np.zeros((n, 4), f)
    dens[:, 0] = counter
    dens[:, 1] = ratio * np.maximum(counter, 1.0)
    dens[:, 2] = dens[:, 1] * 1.5
    dens[:, 3] = np.where(rng.random(n) < 0.1, 500.0, 20.0)  # screen radius in pixels
    return params, moments, grads, dens
