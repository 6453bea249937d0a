"""Self-checks of the CPU oracle (no GPU).

The reference ships no golden vectors for this path, so the oracle is pinned
here against independent restatements: an exhaustive IEEE binary16 check, a
float64 numpy renderer of the reference's own two-Gaussian scene
(examples/single_gs.cpp:46-66), an independent numpy SSIM, finite
differences of its own forward, and the Adam formula.
"""
import math

import numpy as np
import pytest

from tinygs_b200 import scenes

C0 = 0.28209479177387814


def test_half_conversion_exhaustive(oracle):
    lib = oracle.load()
    import ctypes

    lib.orc_h2f.restype = ctypes.c_float
    lib.orc_h2f.argtypes = [ctypes.c_uint16]
    lib.orc_f2h.restype = ctypes.c_uint16
    lib.orc_f2h.argtypes = [ctypes.c_float]
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([lib.orc_h2f(int(b)) for b in bits[::7]], np.float32)
    r = ref[::7]
    same = (got == r) | (np.isnan(got) & np.isnan(r))
    assert same.all()
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.normal(0, 1, 3000), rng.normal(0, 3e4, 500), rng.uniform(-1e-4, 1e-4, 500),
                         np.array([65504.0, 65519.99, 65520.0, 1e-8, -0.0, 2.0 ** -24, 3 * 2.0 ** -25])])
    xs = xs.astype(np.float32)
    with np.errstate(over="ignore"):
        exp = xs.astype(np.float16).view(np.uint16)
    got = np.array([lib.orc_f2h(float(x)) for x in xs], np.uint16)
    np.testing.assert_array_equal(got, exp)


def test_tiled_layout_matches_reference_formula():
    w, h = 40, 24
    img = np.arange(3 * h * w, dtype=np.float32).reshape(3, h, w)
    flat = scenes.to_tiled(img)
    tw = (w + 7) // 8
    for (y, x) in [(0, 0), (7, 7), (8, 0), (13, 37), (23, 39)]:
        idx = ((y >> 3) * tw + (x >> 3)) * 64 + (y & 7) * 8 + (x & 7)  # common.hpp:389-408
        assert flat[1, idx] == img[1, y, x]
    np.testing.assert_array_equal(scenes.from_tiled(flat, w, h), img)


# --------------------------------------------------------------- KAT

def _single_gs_scene():
    """examples/single_gs.cpp:46-66 with its default arguments."""
    o1 = o2 = 0.6
    s1 = s2 = 0.1
    q1 = np.array([-1.0, 0.0, 1.0, 1.0]) * 3.0
    q2 = np.array([1.0, 1.0, 0.0, -1.0]) * 3.0
    params = {
        "means": np.array([[0.0, 0.0, 0.0], [0.5, 0.3, 0.1]], np.float32),
        "scales": np.array([[s1, -s1, 0.3 * s1], [s2, -s2, 0.3 * s2]], np.float32),
        "rotations": np.stack([q1, q2]).astype(np.float32),
        "opacities": np.array([o1, o2], np.float32),
        "sh0": np.array([[0.0, 0.0, 1.0], [1.0, 0.0, 0.0]], np.float32),
        "sh_rest": np.zeros((2, 15, 3), np.float32),
    }
    W, H = 480, 360
    w2c = np.eye(4, dtype=np.float32)
    w2c[2, 3] = 3.0
    cam = {"width": W, "height": H, "fx": 375.0, "fy": 375.0, "cx": W / 2.0, "cy": H / 2.0, "near": 0.001,
           "far": 10000.0, "w2c": w2c.reshape(16)}
    return params, cam


def _numpy_render(params, cam, pixels):
    """Independent float64 evaluation of the projected Gaussians (EWA with
    the 0.3 px dilation, frustum-clamped Jacobian) composited front to back,
    at the given pixel centres."""
    w2c = np.asarray(cam["w2c"], np.float64).reshape(4, 4)
    R, t = w2c[:3, :3], w2c[:3, 3]
    fx, fy, cx, cy, W, H = cam["fx"], cam["fy"], cam["cx"], cam["cy"], cam["width"], cam["height"]
    prims = []
    for i in range(params["means"].shape[0]):
        m = params["means"][i].astype(np.float64)
        pc = R @ m + t
        q = params["rotations"][i].astype(np.float64)
        q = q / np.linalg.norm(q)
        r, x, y, z = q
        Rq = np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - r * z), 2 * (x * z + r * y)],
                       [2 * (x * y + r * z), 1 - 2 * (x * x + z * z), 2 * (y * z - r * x)],
                       [2 * (x * z - r * y), 2 * (y * z + r * x), 1 - 2 * (x * x + y * y)]])
        S = np.diag(np.exp(params["scales"][i].astype(np.float64)))
        Sig = Rq @ S @ S @ Rq.T
        tx = np.clip(pc[0] / pc[2], (-0.15 * W - cx) / fx, (1.15 * W - cx) / fx) * pc[2]
        ty = np.clip(pc[1] / pc[2], (-0.15 * H - cy) / fy, (1.15 * H - cy) / fy) * pc[2]
        J = np.array([[fx / pc[2], 0, -fx * tx / pc[2] ** 2], [0, fy / pc[2], -fy * ty / pc[2] ** 2]])
        cov = J @ R @ Sig @ R.T @ J.T + 0.3 * np.eye(2)
        conic = np.linalg.inv(cov)
        mean2d = np.array([fx * pc[0] / pc[2] + cx, fy * pc[1] / pc[2] + cy])
        op = 1 / (1 + math.exp(-float(params["opacities"][i])))
        col = np.maximum(0.5 + C0 * params["sh0"][i].astype(np.float64), 0.0)
        prims.append((pc[2], mean2d, conic, op, col))
    prims.sort(key=lambda p: p[0])
    out = []
    for (px, py) in pixels:
        T, C = 1.0, np.zeros(3)
        for _, m2, conic, op, col in prims:
            d = m2 - np.array([px + 0.5, py + 0.5])
            power = 0.5 * d @ conic @ d
            a = min(op * math.exp(-power), 0.999)
            if a < 1 / 255:
                continue
            C += T * a * col
            T *= 1 - a
        out.append((C, 1 - T))
    return out


def test_kat_single_gs_scene(oracle):
    params, cam = _single_gs_scene()
    r = oracle.render(params, 0, cam, False)
    assert r["bins"]["n_visible"] == 2
    img = scenes.from_tiled(r["fwd"]["image"], cam["width"], cam["height"])
    alpha = scenes.from_tiled(r["fwd"]["alpha"][None, :], cam["width"], cam["height"])[0]
    rng = np.random.default_rng(1)
    pix = [(240, 180), (239, 179), (300, 210)] + [(int(x), int(y)) for x, y in
                                                  zip(rng.integers(200, 340, 40), rng.integers(140, 240, 40))]
    ref = _numpy_render(params, cam, pix)
    for (x, y), (c, a) in zip(pix, ref):
        np.testing.assert_allclose(img[:, y, x], c, atol=2e-5, rtol=1e-4)
        assert abs(alpha[y, x] - a) < 2e-5
    # the centre pixel sees the first Gaussian's blue-ish colour
    assert img[2, 180, 240] > img[0, 180, 240]


def test_fp16_render_close_to_fp32(oracle):
    cfg = scenes.CONFIGS["cfg0"]
    p = scenes.gaussian_params(4000, 0, cfg.means, 7)
    cam = scenes.cameras(cfg)[0]
    a = oracle.render(p, 0, cam, False)["fwd"]["image"]
    b = oracle.render(p, 0, cam, True)["fwd"]["image"].astype(np.float32)
    # uint8 colour quantisation and fp16 compositing: a few 1/255 steps
    assert np.abs(a - b).max() < 0.05
    assert np.abs(a - b).mean() < 2e-3


# ----------------------------------------------------- binning properties

def test_oracle_binning_properties(oracle):
    cfg = scenes.CONFIGS["cfg0"]
    p = scenes.gaussian_params(cfg.n, 0, cfg.means, cfg.seed)
    cam = scenes.cameras(cfg)[0]
    prims = oracle.preprocess(p, 0, cam, False)
    bins = oracle.binning(prims, cam, False)
    tiles, prim = bins["inst_tile"], bins["inst_prim"]
    assert bins["n_instances"] == int(prims["n_touched"].sum())
    assert np.all(np.diff(tiles.astype(np.int64)) >= 0)
    same = tiles[1:] == tiles[:-1]
    d = prims["depth_key"]
    assert np.all((d[prim[:-1]] <= d[prim[1:]]) | ~same)
    per = np.bincount(prim, minlength=cfg.n)
    np.testing.assert_array_equal(per, prims["n_touched"])


# ------------------------------------------------------------ SSIM

def _gauss_window():
    x = np.arange(11) - 5
    g = np.exp(-(x ** 2) / (2 * 1.5 ** 2))
    return g / g.sum()


def _conv2(img, g):
    pad = np.pad(img, 5)
    h = sum(g[k] * pad[:, k:k + img.shape[1]] for k in range(11))
    return sum(g[k] * h[k:k + img.shape[0], :] for k in range(11))


def _ssim_numpy(x, y):
    g = _gauss_window()
    mu1, mu2 = _conv2(x, g), _conv2(y, g)
    s1 = _conv2(x * x, g) - mu1 ** 2
    s2 = _conv2(y * y, g) - mu2 ** 2
    s12 = _conv2(x * y, g) - mu1 * mu2
    C1, C2 = 1e-4, 9e-4
    return ((2 * mu1 * mu2 + C1) * (2 * s12 + C2)) / ((mu1 ** 2 + mu2 ** 2 + C1) * (s1 + s2 + C2))


def test_ssim_oracle_matches_numpy_and_finite_differences(oracle):
    w, h = 24, 16
    rng = np.random.default_rng(3)
    x = rng.uniform(0, 1, (3, h, w)).astype(np.float16).astype(np.float32)  # exact in fp16
    y = rng.uniform(0, 1, (3, h, w)).astype(np.float16).astype(np.float32)
    xt, yt = scenes.to_tiled(x), scenes.to_tiled(y)
    loss = np.zeros_like(xt)
    grad = np.zeros_like(xt)
    s = 1.0
    oracle.ssim(np.ascontiguousarray(xt), np.ascontiguousarray(yt), loss, grad, w, h, s)
    L = scenes.from_tiled(loss, w, h)
    for c in range(3):
        ref = (1 - _ssim_numpy(x[c].astype(np.float64), y[c].astype(np.float64))) / (w * h)
        np.testing.assert_allclose(L[c], ref, atol=2e-6)
    G = scenes.from_tiled(grad, w, h)
    # finite differences of the total SSIM loss (fp64 numpy model)
    for (c, yy, xx) in [(0, 5, 7), (1, 0, 0), (2, 15, 23), (1, 8, 12)]:
        e = 1e-4
        xp, xm = x.astype(np.float64).copy(), x.astype(np.float64).copy()
        xp[c, yy, xx] += e
        xm[c, yy, xx] -= e
        fp = (1 - _ssim_numpy(xp[c], y[c].astype(np.float64))).sum() / (w * h)
        fm = (1 - _ssim_numpy(xm[c], y[c].astype(np.float64))).sum() / (w * h)
        fd = (fp - fm) / (2 * e)
        assert abs(G[c, yy, xx] - fd) <= 1e-3 * abs(fd) + 1e-7, (c, yy, xx, G[c, yy, xx], fd)


def test_l1_oracle(oracle):
    w, h = 16, 8
    rng = np.random.default_rng(4)
    p = rng.uniform(-0.2, 1.2, 3 * w * h).astype(np.float32)
    t = rng.uniform(0, 1, 3 * w * h).astype(np.float32)
    loss, grad = np.zeros_like(p), np.zeros_like(p)
    oracle.l1(p, t, loss, grad, w, h, 3.0)
    s = 3.0 / (3 * w * h)
    np.testing.assert_allclose(loss, np.abs(np.clip(p, 0, 1) - t) * s, rtol=1e-6)
    np.testing.assert_allclose(grad, np.sign(np.clip(p, 0, 1) - t) * s, rtol=1e-6)


# ------------------------------------------------ gradients by FD

def _tiny_scene(n=12, seed=0):
    rng = np.random.default_rng(seed)
    p = {"means": rng.uniform(-0.5, 0.5, (n, 3)).astype(np.float32),
         "scales": rng.normal(-2.0, 0.2, (n, 3)).astype(np.float32),
         "rotations": rng.normal(0, 1, (n, 4)).astype(np.float32),
         "opacities": rng.normal(1.0, 0.5, n).astype(np.float32),
         "sh0": rng.normal(0, 1, (n, 3)).astype(np.float32),
         "sh_rest": rng.normal(0, 0.3, (n, 15, 3)).astype(np.float32)}
    cam = {"width": 48, "height": 32, "fx": 40.0, "fy": 40.0, "cx": 24.0, "cy": 16.0, "near": 0.01, "far": 100.0,
           "w2c": scenes.look_at_w2c((0.3, -0.2, -2.5)).reshape(16)}
    return p, cam


def test_backward_is_the_derivative_of_the_forward(oracle):
    """The restated backward against central differences of the restated
    forward for a random linear functional of the image.  The forward is
    piecewise (alpha < 1/255 cut, early termination, integer tile bounds), so
    the check runs the oracle's smooth variant of it (every tile touched, no
    cut, no termination), of which the reference's backward is the exact
    derivative; opacities stay below the 0.999 alpha cap."""
    lib = oracle.load()
    lib.orc_set_smooth_forward(1)
    try:
        for seed in (0, 1):
            p, cam = _tiny_scene(seed=seed)
            sh = 2
            rng = np.random.default_rng(9)
            base = oracle.render(p, sh, cam, False)
            wgt = rng.normal(0, 1, base["fwd"]["image"].shape).astype(np.float32)

            def f(pp):
                return float(np.dot(oracle.render(pp, sh, cam, False)["fwd"]["image"].astype(np.float64), wgt))

            screen = oracle.blend_backward(base["prims"], base["bins"], base["fwd"], wgt, cam, False)
            grads = oracle.preprocess_backward(p, sh, cam, base["prims"]["n_touched"], screen)
            w2c = np.asarray(cam["w2c"], np.float64).reshape(4, 4)

            def depth_order(pp):
                return np.argsort(pp["means"].astype(np.float64) @ w2c[2, :3], kind="stable")

            for name in ("means", "scales", "rotations", "opacities", "sh0", "sh_rest"):
                skip = []
                fd = np.zeros_like(p[name], dtype=np.float64)
                flat = p[name].reshape(-1)
                for k in range(flat.size):
                    if name == "sh_rest" and (k // 3) % 15 >= 8:
                        continue  # degree 2: eight active higher bands
                    pp = {kk: v.copy() for kk, v in p.items()}
                    pp[name].reshape(-1)[k] += 1e-3
                    order_p = depth_order(pp)
                    fp = f(pp)
                    pp[name].reshape(-1)[k] -= 2e-3
                    if name == "means" and not np.array_equal(order_p, depth_order(pp)):
                        skip.append(k)  # the step reorders two Gaussians in depth
                        continue
                    fd.reshape(-1)[k] = (fp - f(pp)) / 2e-3
                a = grads[name].astype(np.float64)
                if name == "rotations":
                    # the reference divides the raw-quaternion gradient by
                    # |q|^3 where the derivative has |q|^2
                    # (fastgs_ours/kernels_backward.cuh:328-332): it is the
                    # derivative scaled by 1/|q|, equal for unit quaternions
                    a = a * np.linalg.norm(p["rotations"].astype(np.float64), axis=1, keepdims=True)
                a = a.ravel()
                b = fd.ravel()
                a[skip] = 0.0
                b[skip] = 0.0
                assert len(skip) <= 2
                rel = np.linalg.norm(a - b) / np.linalg.norm(b)
                assert rel < 2e-2, (seed, name, rel)
    finally:
        lib.orc_set_smooth_forward(0)


# ----------------------------------------------------------- Adam

def test_adam_oracle_formula(oracle):
    from types import SimpleNamespace
    rng = np.random.default_rng(2)
    n = 50
    mk = lambda: {"means": rng.normal(size=(n, 3)).astype(np.float32), "opacities": rng.normal(size=n).astype(np.float32),
                  "rotations": rng.normal(size=(n, 4)).astype(np.float32),
                  "scales": rng.normal(size=(n, 3)).astype(np.float32),
                  "sh0": rng.normal(size=(n, 3)).astype(np.float32),
                  "sh_rest": rng.normal(size=(n, 15, 3)).astype(np.float32)}
    p, g = mk(), mk()
    cfg = SimpleNamespace(beta1=0.9, beta2=0.999, epsilon=1e-8, max_grad_1=0.3, means_lr=1e-3, shs_lr=2e-3,
                          opacities_lr=3e-3, scales_lr=4e-3, rotations_lr=5e-3, opacities_l1=0.0, scales_l1=0.0,
                          scene_scale=1.5, global_lr=1.0, decay_reduction_mean=True)
    m = {k: np.zeros_like(v) for k, v in p.items()}
    v = {k: np.zeros_like(x) for k, x in p.items()}
    ref = {k: x.astype(np.float64).copy() for k, x in p.items()}
    mr = {k: np.zeros_like(x, dtype=np.float64) for k, x in p.items()}
    vr = {k: np.zeros_like(x, dtype=np.float64) for k, x in p.items()}
    lrs = {"means": 1e-3 * 1.5, "opacities": 3e-3, "rotations": 5e-3, "scales": 4e-3, "sh0": 2e-3, "sh_rest": 1e-4}
    for step in (1, 2):
        oracle.adam_step(p, g, m, v, cfg, step, 0.5)
        for k in ref:
            gg = np.clip(0.5 * g[k].astype(np.float64), -0.3, 0.3)
            mr[k] = 0.9 * mr[k] + 0.1 * gg
            vr[k] = 0.999 * vr[k] + 0.001 * gg * gg
            mh = mr[k] / (1 - 0.9 ** step)
            den = np.sqrt(vr[k]) / np.sqrt(1 - 0.999 ** step) + 1e-8
            ref[k] -= mh * lrs[k] / den
    for k in ref:
        np.testing.assert_allclose(p[k], ref[k], rtol=1e-5, atol=1e-6, err_msg=k)


def _morton_numpy(means):
    """Independent numpy restatement of the reference's Morton order
    (orchestrator.cu:26-100), float32 arithmetic throughout."""
    m = np.asarray(means, np.float32)
    lo, hi = m.min(0), m.max(0)
    d = (hi - lo).astype(np.float32)
    inv = (np.float32(1.0) / np.where(d < np.float32(1e-8), np.float32(1e-8), d)).astype(np.float32)
    u = np.clip(((m - lo).astype(np.float32) * inv).astype(np.float32), np.float32(0), np.float32(1))
    q = (u * np.float32(1023.0)).astype(np.float32).astype(np.uint32)
    code = np.zeros(m.shape[0], np.uint64)
    for b in range(10):
        for c in range(3):
            code |= ((q[:, c].astype(np.uint64) >> np.uint64(b)) & np.uint64(1)) << np.uint64(3 * b + c)
    return np.argsort(code, kind="stable").astype(np.uint32)


def test_oracle_morton_order_matches_numpy(oracle):
    rng = np.random.default_rng(3)
    means = rng.normal(0, 1.5, (20000, 3)).astype(np.float32)
    means[100:200] = means[100]  # equal codes keep index order
    np.testing.assert_array_equal(oracle.morton_order(means), _morton_numpy(means))
    flat = means.copy()
    flat[:, 2] = 0.25  # a degenerate axis: extent clamped to 1e-8
    np.testing.assert_array_equal(oracle.morton_order(flat), _morton_numpy(flat))
    assert oracle.morton_order(means[:1]).tolist() == [0]
    assert oracle.morton_order(np.zeros((0, 3), np.float32)).size == 0
