"""Host side of the image data path, no GPU: the loaders' PCG32 and
permutation against the C oracle's PCG32, and the numpy restatement of the
data-path kernels (oracle/image_oracle.py) against itself where two routes
exist."""
import numpy as np

from oracle import image_oracle as io
from oracle import pyoracle
from tinygs_b200 import dataloader as dl
from tinygs_b200 import scenes


def test_host_pcg32_matches_oracle():
    for seed in (0, 1, 12345, 2**63 + 7):
        a = dl.Pcg32(seed, 1)
        r = pyoracle.pcg32(seed, 1)
        np.testing.assert_array_equal(np.array([a.next_uint() for _ in range(500)], np.uint32),
                                      pyoracle.pcg32_next_uint(r, 500))


def test_bounded_draws_and_permutation():
    rng = dl.Pcg32(7, 1)
    draws = [rng.next_uint(b) for b in (1, 2, 3, 7, 1000, 2**31 + 1) for _ in range(50)]
    assert all(d >= 0 for d in draws)
    for n in (1, 2, 10, 251):
        p = dl.permutation(dl.Pcg32(3, 1), n)
        assert sorted(p) == list(range(n))
    # the same seed, the same sequence of epochs
    a, b = dl.Pcg32(5, 1), dl.Pcg32(5, 1)
    assert [dl.permutation(a, 9) for _ in range(3)] == [dl.permutation(b, 9) for _ in range(3)]


def test_blur_state_init_is_the_pcg32_stream():
    n = 300
    st = io.blur_state_init(n, seed=0)
    r = pyoracle.pcg32(0, 1)
    outs = pyoracle.pcg32_next_uint(r, 2 * n).astype(np.uint64)
    np.testing.assert_array_equal(st, (outs[0::2] << np.uint64(32)) | outs[1::2])


def test_hwc_reorder_round_trip():
    rng = np.random.default_rng(0)
    for (w, h, c) in ((37, 21, 3), (16, 8, 4), (9, 17, 3)):
        img = rng.integers(0, 256, (h, w, c), dtype=np.uint8)
        t = io.hwc_to_tiled(img, w, h, "u8")
        back = scenes.from_tiled(t.reshape(-1), w, h)
        np.testing.assert_array_equal(back, img[:, :, :3].transpose(2, 0, 1))
        # padding is zero
        assert int(t.sum()) == int(img[:, :, :3].astype(np.int64).sum())


def test_nearest_resize_identity_and_halving():
    rng = np.random.default_rng(1)
    w, h = 24, 16
    src = io.hwc_to_tiled(rng.integers(0, 256, (h, w, 3), dtype=np.uint8), w, h, "u8")
    same, _ = io.resize(src, w, h, 3, w, h, "u8")
    np.testing.assert_array_equal(same, src)
    half, _ = io.resize(src, w, h, 3, w // 2, h // 2, "u8")
    full = scenes.from_tiled(src.reshape(-1), w, h)
    np.testing.assert_array_equal(scenes.from_tiled(half.reshape(-1), w // 2, h // 2), full[:, ::2, ::2])


def test_convert_values():
    v = np.arange(256, dtype=np.uint8)
    f = io.convert(v, "f32")
    assert f.dtype == np.float32 and f[0] == 0 and abs(float(f[255]) - 1.0) < 1e-7
    h = io.convert(v, "f16")
    assert h.dtype == np.float16
    np.testing.assert_array_equal(h, f.astype(np.float16))
