"""numpy restatement of the reference's image data path.

TEST INFRASTRUCTURE ONLY -- imported by tests/ as the checker of
tinygs_b200/csrc/image.cu.  Parity status: unpinned against the reference's
own code (its data-loader kernels are file-static in a translation unit that
needs its dataset and logging headers; the harness under oracle/ref/ does not
build it).  The arithmetic is restated line by line from the cited sources;
PCG32 is checked against the C oracle's restatement, which the
densification tests pin.

Layout: channel planes of 8x8 tiles, tiles row-major, pixels in a tile
row-major (include/tinygs/common.hpp:367-413), planes padded to multiples
of 8 in both directions.
"""
from __future__ import annotations

import numpy as np

U8_SCALE = np.float32(1.0) / np.float32(255.0)  # CHAR_TO_FLOAT, dataloader.cu:19
_MULT = np.uint64(0x5851F42D4C957F2D)


def pad8(x: int) -> int:
    return (x + 7) // 8 * 8


def tiled_index(y: np.ndarray, x: np.ndarray, tiles_w: int) -> np.ndarray:
    """get_linear_index_tiled (common.hpp:404-408)."""
    y = np.asarray(y, np.int64)
    x = np.asarray(x, np.int64)
    return (((y >> 3) * tiles_w + (x >> 3)) << 6) + ((y & 7) << 3) + (x & 7)


def convert(v: np.ndarray, dtype: str) -> np.ndarray:
    """convert_u8_float / convert_u8_half (dataloader.cu:26-104):
    1/255 * v in float32, then rounded to nearest half for fp16."""
    if dtype == "u8":
        return v.astype(np.uint8)
    f = U8_SCALE * v.astype(np.float32)
    return f.astype(np.float16) if dtype == "f16" else f


def hwc_to_tiled(img: np.ndarray, width: int, height: int, dtype: str) -> np.ndarray:
    """PngFolderDataset's HWC -> tiled CHW reorder (dataset/png_folder.cpp:
    60-69; RGB kept, alpha dropped), padding zero, then convert()."""
    hp, wp = pad8(height), pad8(width)
    out = np.zeros((3, hp * wp), np.uint8)
    yy, xx = np.meshgrid(np.arange(height), np.arange(width), indexing="ij")
    idx = tiled_index(yy, xx, wp // 8)
    for c in range(3):
        out[c, idx.reshape(-1)] = img[:, :, c].reshape(-1)
    return convert(out, dtype)


def _seeded(initstate: np.ndarray) -> tuple[np.ndarray, np.uint64]:
    """pcg32(initstate, 1) (pcg32.hpp:45-56), vectorised over states."""
    inc = np.uint64(3)
    state = np.zeros_like(initstate)
    state = state * _MULT + inc
    state = state + initstate
    state = state * _MULT + inc
    return state, inc


def _next(state: np.ndarray, inc: np.uint64) -> tuple[np.ndarray, np.ndarray]:
    """pcg32::next_uint (pcg32.hpp:59-65)."""
    old = state
    state = old * _MULT + inc
    xs = (((old >> np.uint64(18)) ^ old) >> np.uint64(27)).astype(np.uint32)
    rot = (old >> np.uint64(59)).astype(np.uint32)
    out = (xs >> rot) | (xs << ((np.uint32(0) - rot) & np.uint32(31)))
    return state, out


def blur_state_init(n: int, seed: int = 0) -> np.ndarray:
    """DataLoaderBase::reset's states (dataloader.cu:361-378): one
    pcg32(seed, 1) stream, element i = (output 2i << 32) | output 2i+1."""
    with np.errstate(over="ignore"):
        state, inc = _seeded(np.array([seed], np.uint64))
        outs = np.empty(2 * n, np.uint32)
        for k in range(2 * n):
            state, o = _next(state, inc)
            outs[k] = o[0]
    return (outs[0::2].astype(np.uint64) << np.uint64(32)) | outs[1::2].astype(np.uint64)


def _src_coord(x: np.ndarray, src: int, dst: int) -> np.ndarray:
    """min((uint32_t)((float)x * (float)src / (float)dst), src - 1)."""
    f = (x.astype(np.float32) * np.float32(src)) / np.float32(dst)
    return np.minimum(f.astype(np.uint32), np.uint32(src - 1))


def resize(src: np.ndarray, src_w: int, src_h: int, channels: int, dst_w: int, dst_h: int, dtype: str,
           state: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray | None]:
    """resize_nn_u8_to_float_tiled (dataloader.cu:107-120; state None) or
    resize_u8_to_{float,half}_tiled_stochastic_blur (:122-186).  src: u8
    [channels][padded src plane]; returns ([channels][padded dst plane] with
    zero padding, the advanced states)."""
    src = src.reshape(channels, -1)
    hp, wp = pad8(dst_h), pad8(dst_w)
    out = np.zeros((channels, hp * wp), np.uint8)
    yy, xx = np.meshgrid(np.arange(dst_h, dtype=np.uint32), np.arange(dst_w, dtype=np.uint32), indexing="ij")
    yy, xx = yy.reshape(-1), xx.reshape(-1)
    di = tiled_index(yy, xx, wp // 8)
    sx, sy = _src_coord(xx, src_w, dst_w), _src_coord(yy, src_h, dst_h)
    stw = pad8(src_w) // 8
    new_state = None if state is None else state.copy()
    for c in range(channels):
        if state is None:
            out[c, di] = src[c, tiled_index(sy, sx, stw)]
            continue
        span_x = _src_coord(xx + np.uint32(1), src_w, dst_w) - sx + np.uint32(1)
        span_y = _src_coord(yy + np.uint32(1), src_h, dst_h) - sy + np.uint32(1)
        o = c * hp * wp + di
        with np.errstate(over="ignore"):
            st, inc = _seeded(state[o].astype(np.uint64))
            st, rx = _next(st, inc)
            st, ry = _next(st, inc)
        dx, dy = rx % span_x, ry % span_y
        out[c, di] = src[c, tiled_index(sy + dy, sx + dx, stw)]
        new_state[o] = st
    return convert(out, dtype), new_state
