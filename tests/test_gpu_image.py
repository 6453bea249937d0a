"""The image data path on the GPU (tgs_image_from_u8, tgs_image_resize_u8,
tgs_image_blur_state_init and the loaders of tinygs_b200.dataloader) against
the numpy restatement of the reference's data-loader kernels
(oracle/image_oracle.py): bit-exact for every dtype, layout and size,
odd sizes and padding included."""
import numpy as np
import pytest
import torch

from oracle import image_oracle as io
from tinygs_b200 import _abi
from tinygs_b200 import dataloader as dl
from tinygs_b200._abi import check, load_library

pytestmark = pytest.mark.gpu

DT = {"f32": (_abi.TGS_FLOAT32, torch.float32), "f16": (_abi.TGS_FLOAT16, torch.float16),
      "u8": (_abi.TGS_UINT8, torch.uint8)}


def _np(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy()


@pytest.mark.parametrize("dtype", ["f32", "f16", "u8"])
@pytest.mark.parametrize("w,h,c", [(37, 21, 3), (1920, 1080, 3), (64, 40, 4)])
def test_tiled_conversion(dtype, w, h, c):
    rng = np.random.default_rng(w * h + c)
    plane = io.pad8(w) * io.pad8(h)
    src = rng.integers(0, 256, c * plane, dtype=np.uint8)
    d_src = torch.from_numpy(src).cuda()
    code, tdt = DT[dtype]
    out = torch.full((c * plane,), 7, dtype=tdt, device="cuda")
    check(load_library().tgs_image_from_u8(d_src.data_ptr(), _abi.TGS_IMAGE_TILED_CHW, c, w, h, out.data_ptr(),
                                           code, torch.cuda.current_stream().cuda_stream), "tgs_image_from_u8")
    np.testing.assert_array_equal(_np(out), io.convert(src, dtype))


@pytest.mark.parametrize("dtype", ["f32", "f16", "u8"])
@pytest.mark.parametrize("w,h,c", [(37, 21, 3), (1281, 719, 3), (300, 17, 4), (8, 8, 3)])
def test_hwc_reorder(dtype, w, h, c):
    rng = np.random.default_rng(w + 7 * h + c)
    img = rng.integers(0, 256, (h, w, c), dtype=np.uint8)
    d_src = torch.from_numpy(img.reshape(-1).copy()).cuda()
    code, tdt = DT[dtype]
    out = torch.full((3 * io.pad8(w) * io.pad8(h),), 7, dtype=tdt, device="cuda")
    check(load_library().tgs_image_from_u8(d_src.data_ptr(), _abi.TGS_IMAGE_HWC, c, w, h, out.data_ptr(), code,
                                           torch.cuda.current_stream().cuda_stream), "tgs_image_from_u8")
    np.testing.assert_array_equal(_np(out), io.hwc_to_tiled(img, w, h, dtype).reshape(-1))


def test_blur_state_init():
    n = 3 * 64 * 40
    st = dl.blur_state(n, seed=0)
    np.testing.assert_array_equal(_np(st).view(np.uint64)[:n], io.blur_state_init(n, 0))
    st9 = dl.blur_state(100, seed=9)
    np.testing.assert_array_equal(_np(st9).view(np.uint64)[:100], io.blur_state_init(100, 9))


@pytest.mark.parametrize("dtype", ["f32", "f16"])
@pytest.mark.parametrize("blur", [False, True])
@pytest.mark.parametrize("src_wh,dst_wh", [((100, 60), (50, 30)), ((100, 60), (37, 23)), ((64, 48), (160, 96)),
                                           ((1920, 1080), (960, 540))])
def test_resize(dtype, blur, src_wh, dst_wh):
    (sw, sh), (dw, dh) = src_wh, dst_wh
    rng = np.random.default_rng(sw + dw)
    img = rng.integers(0, 256, (sh, sw, 3), dtype=np.uint8)
    src = io.hwc_to_tiled(img, sw, sh, "u8").reshape(-1)
    d_src = torch.from_numpy(src.copy()).cuda()
    code, tdt = DT[dtype]
    n_out = 3 * io.pad8(dw) * io.pad8(dh)
    out = torch.full((n_out,), 7, dtype=tdt, device="cuda")
    state = dl.blur_state(n_out, seed=0) if blur else None
    ref_state = io.blur_state_init(n_out, 0) if blur else None
    lib = load_library()
    for _ in range(2 if blur else 1):  # twice: the states advance in place
        check(lib.tgs_image_resize_u8(d_src.data_ptr(), sw, sh, 3, out.data_ptr(), code, dw, dh,
                                      None if state is None else state.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream), "tgs_image_resize_u8")
        ref, ref_state = io.resize(src, sw, sh, 3, dw, dh, dtype, ref_state)
        np.testing.assert_array_equal(_np(out), ref.reshape(-1))
        if blur:
            np.testing.assert_array_equal(_np(state).view(np.uint64), ref_state)


def test_rejects_bad_arguments():
    lib = load_library()
    buf = torch.zeros(3 * 64, dtype=torch.uint8, device="cuda")
    out = torch.zeros(3 * 64, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.tgs_image_from_u8(buf.data_ptr(), 5, 3, 8, 8, out.data_ptr(), 0, s) == _abi.TGS_ERR_INVALID_ARGUMENT
    assert lib.tgs_image_from_u8(buf.data_ptr(), 0, 2, 8, 8, out.data_ptr(), 0, s) == _abi.TGS_ERR_INVALID_ARGUMENT
    assert lib.tgs_image_from_u8(buf.data_ptr() + 1, 0, 3, 8, 8, out.data_ptr(), 0, s) == \
        _abi.TGS_ERR_INVALID_ARGUMENT
    assert lib.tgs_image_from_u8(None, 0, 3, 8, 8, out.data_ptr(), 0, s) == _abi.TGS_ERR_INVALID_ARGUMENT
    assert lib.tgs_image_resize_u8(buf.data_ptr(), 8, 8, 3, out.data_ptr(), _abi.TGS_UINT8, 4, 4, None, s) == \
        _abi.TGS_ERR_INVALID_ARGUMENT
    assert lib.tgs_image_resize_u8(buf.data_ptr(), 0, 8, 3, out.data_ptr(), 0, 4, 4, None, s) == \
        _abi.TGS_ERR_INVALID_ARGUMENT


def _dataset(n=5, w=200, h=120, layout=_abi.TGS_IMAGE_HWC):
    rng = np.random.default_rng(11)
    if layout == _abi.TGS_IMAGE_HWC:
        imgs = [rng.integers(0, 256, (h, w, 3), dtype=np.uint8) for _ in range(n)]
    else:
        imgs = [io.hwc_to_tiled(rng.integers(0, 256, (h, w, 3), dtype=np.uint8), w, h, "u8") for _ in range(n)]
    cams = [{"fx": 100.0 + k, "fy": 100.0, "cx": w / 2, "cy": h / 2, "w2c": np.eye(4, dtype=np.float32)}
            for k in range(n)]
    return dl.ImageDataset(imgs, cams, w, h, layout=layout)


def _expected(ds, i, dtype):
    if ds.layout == _abi.TGS_IMAGE_HWC:
        return io.hwc_to_tiled(ds.images[i], ds.width, ds.height, dtype).reshape(-1)
    return io.convert(ds.images[i], dtype).reshape(-1)


@pytest.mark.parametrize("layout", [_abi.TGS_IMAGE_HWC, _abi.TGS_IMAGE_TILED_CHW])
def test_simple_loader_order_and_images(layout):
    ds = _dataset(layout=layout)
    loader = dl.SimpleDataLoader(ds, _abi.TGS_FLOAT16, seed=0)
    rng = dl.Pcg32(0, 1)
    order = [i for _ in range(3) for i in dl.permutation(rng, len(ds))]
    for k in range(12):
        b = loader.next()
        assert b.index == order[k]
        assert b.camera["fx"] == ds.cameras[b.index]["fx"] and b.camera["width"] == ds.width
        np.testing.assert_array_equal(_np(b.image), _expected(ds, b.index, "f16"))


def test_async_loader_order_images_and_slot_reuse():
    ds = _dataset(n=7)
    loader = dl.AsyncDataLoader(ds, _abi.TGS_FLOAT32, seed=3, prefetch_factor=3)
    rng = dl.Pcg32(3, 1)
    dl.permutation(rng, len(ds))  # the constructor's draw; the first epoch is the reset's
    order = [i for _ in range(3) for i in dl.permutation(rng, len(ds))]
    stream = torch.cuda.Stream()
    seen = []
    try:
        for k in range(20):
            b = loader.next(stream)
            with torch.cuda.stream(stream):
                got = b.image.clone()  # the consumer's read, ordered after the conversion
                torch.cuda._sleep(200_000)  # keeps the slot busy while the prefetcher wants it
            stream.synchronize()
            seen.append(b.index)
            np.testing.assert_array_equal(_np(got), _expected(ds, b.index, "f32"))
    finally:
        loader.close()
    assert seen == order[:20]


def test_loader_resize():
    ds = _dataset(n=3, w=120, h=80)
    loader = dl.SimpleDataLoader(ds, _abi.TGS_FLOAT32, seed=0)
    loader.set_output_shape(60, 40)  # a new permutation, as the reference's reset
    state = io.blur_state_init(3 * 64 * 40, 0)  # the prefix the 60x40 output indexes
    rng = dl.Pcg32(0, 1)
    dl.permutation(rng, 3)
    order = dl.permutation(rng, 3)
    for k in range(3):
        b = loader.next()
        assert b.index == order[k] and b.camera["width"] == 60
        src = io.hwc_to_tiled(ds.images[b.index], 120, 80, "u8").reshape(-1)
        ref, state = io.resize(src, 120, 80, 3, 60, 40, "f32", state)
        np.testing.assert_array_equal(_np(b.image), ref.reshape(-1))
