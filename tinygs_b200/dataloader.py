"""Data path of the training loop: host images to device targets.

Mirror of the reference's data loaders (tinygs/include/tinygs/dataloader/
dataloader.hpp, simple.hpp, async.hpp; tinygs/src/dataloader/*): a dataset
of 8-bit images with cameras, a permutation drawn with PCG32 (Fisher-Yates,
reshuffled at every epoch), and ``next()`` returning the camera of the view
and its target image on the device in the rasterizer's tiled layout
(float32 or float16).  The conversion, the HWC -> tiled reorder and the
resize run as CUDA kernels of ``libtgs_b200.so`` (tgs_image_from_u8,
tgs_image_resize_u8); there is no CPU fallback.

Differences in mechanism (results are the same): the reference copies every
image through one device scratch buffer under a mutex and synchronises the
prefetch stream after each transfer (dataloader.cu:218-339).  Here each of
the ``prefetch_factor`` ring slots has its own pinned host staging buffer
and device scratch, so the prefetch thread never waits for a copy it did not
need; the consumer stream waits for a slot's conversion with an event, and a
slot is reused only after an event recorded on the consumer stream when the
next batch was taken, so the GPU never waits on the host and the host never
waits on the GPU outside the prefetch thread.
"""
from __future__ import annotations

import queue
import threading
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _abi
from ._abi import check, load_library
from .runtime import _stream_handle


# ------------------------------------------------------------------ PCG32

_MULT = 0x5851F42D4C957F2D
_MASK64 = (1 << 64) - 1


class Pcg32:
    """The reference's pcg32 (include/tinygs/random/pcg32.hpp): O'Neill's
    PCG-XSH-RR with a 64-bit LCG state; used on the host for the view
    permutation (async.cpp:242-258, simple.cpp:17-35)."""

    def __init__(self, initstate: int = 0, initseq: int = 1):
        self.seed(initstate, initseq)

    def seed(self, initstate: int, initseq: int = 1) -> None:
        self.state = 0
        self.inc = ((initseq << 1) | 1) & _MASK64
        self.next_uint()
        self.state = (self.state + initstate) & _MASK64
        self.next_uint()

    def next_uint(self, bound: int | None = None) -> int:
        if bound is not None:
            # unbiased: reject outputs below 2^32 mod bound
            threshold = ((1 << 32) - bound) % bound
            while True:
                r = self.next_uint()
                if r >= threshold:
                    return r % bound
        old = self.state
        self.state = (old * _MULT + self.inc) & _MASK64
        xorshifted = (((old >> 18) ^ old) >> 27) & 0xFFFFFFFF
        rot = old >> 59
        return ((xorshifted >> rot) | (xorshifted << ((-rot) & 31))) & 0xFFFFFFFF


def permutation(rng: Pcg32, n: int) -> list[int]:
    """Fisher-Yates over 0..n-1 with rng.next_uint(i + 1), i from n-1 down."""
    p = list(range(n))
    for i in range(n - 1, 0, -1):
        j = rng.next_uint(i + 1)
        p[i], p[j] = p[j], p[i]
    return p


# ---------------------------------------------------------------- dataset

@dataclass
class ImageDataset:
    """Host images with their cameras (the reference's DatasetBase with
    PngFolderDataset's in-memory image store, dataset/png_folder.cpp).

    images: uint8 arrays, either [C][padded tiled plane] (layout
    TGS_IMAGE_TILED_CHW, C = 3 or 4) or [H][W][C] rows as a decoder returns
    them (TGS_IMAGE_HWC, C = 3 or 4).  cameras: dicts with fx, fy, cx, cy,
    w2c (width/height/near/far are set by the loader)."""
    images: list[np.ndarray]
    cameras: list[dict]
    width: int
    height: int
    layout: int = _abi.TGS_IMAGE_TILED_CHW
    channels: int = 3

    def __len__(self) -> int:
        return len(self.images)

    def __post_init__(self):
        if len(self.images) != len(self.cameras):
            raise ValueError("one camera per image")
        for im in self.images:
            if im.dtype != np.uint8:
                raise ValueError("images are 8-bit")
            if im.nbytes != self.source_bytes():
                raise ValueError(f"image of {im.nbytes} bytes, expected {self.source_bytes()}")

    def padded_plane(self) -> int:
        return ((self.width + 7) // 8 * 8) * ((self.height + 7) // 8 * 8)

    def source_bytes(self) -> int:
        if self.layout == _abi.TGS_IMAGE_TILED_CHW:
            return self.channels * self.padded_plane()
        return self.width * self.height * self.channels


@dataclass
class Batch:
    """GPUBatchInputOutput (dataloader.hpp:8-27): the view's camera and its
    target image (device, tiled layout)."""
    camera: dict
    image: torch.Tensor
    index: int = -1
    slot: int = -1
    ready: torch.cuda.Event | None = field(default=None, repr=False)


def _torch_dtype(dtype: int) -> torch.dtype:
    return {_abi.TGS_FLOAT32: torch.float32, _abi.TGS_FLOAT16: torch.float16}[dtype]


class _Converter:
    """DataLoaderBase::transfer_gpu (dataloader.cu:218-339) on the device:
    pinned host bytes -> device scratch -> converted (and, when the output
    shape differs from the dataset's, resized) target."""

    def __init__(self, dataset: ImageDataset, dtype: int, out_w: int, out_h: int, device: torch.device,
                 blur_state: torch.Tensor | None):
        self.ds, self.dtype, self.out_w, self.out_h = dataset, dtype, out_w, out_h
        self.lib = load_library()
        self.host = torch.empty(dataset.source_bytes(), dtype=torch.uint8).pin_memory()
        self.raw = torch.empty(dataset.source_bytes(), dtype=torch.uint8, device=device)
        self.resize = (out_w, out_h) != (dataset.width, dataset.height)
        self.tiled_u8 = None
        if self.resize and dataset.layout == _abi.TGS_IMAGE_HWC:
            self.tiled_u8 = torch.empty(3 * dataset.padded_plane(), dtype=torch.uint8, device=device)
        self.blur_state = blur_state

    def out_channels(self) -> int:
        return 3 if self.ds.layout == _abi.TGS_IMAGE_HWC else self.ds.channels

    def issue(self, image: np.ndarray, out: torch.Tensor, stream: torch.cuda.Stream) -> None:
        self.host.numpy()[:] = image.reshape(-1)
        h = _stream_handle(stream)
        with torch.cuda.stream(stream):
            self.raw.copy_(self.host, non_blocking=True)
        ds = self.ds
        if not self.resize:
            check(self.lib.tgs_image_from_u8(self.raw.data_ptr(), ds.layout, ds.channels, ds.width, ds.height,
                                             out.data_ptr(), self.dtype, h), "tgs_image_from_u8")
            return
        src = self.raw
        if self.tiled_u8 is not None:
            check(self.lib.tgs_image_from_u8(self.raw.data_ptr(), ds.layout, ds.channels, ds.width, ds.height,
                                             self.tiled_u8.data_ptr(), _abi.TGS_UINT8, h), "tgs_image_from_u8")
            src = self.tiled_u8
        check(self.lib.tgs_image_resize_u8(src.data_ptr(), ds.width, ds.height, self.out_channels(), out.data_ptr(),
                                           self.dtype, self.out_w, self.out_h, self.blur_state.data_ptr(), h),
              "tgs_image_resize_u8")


def blur_state(n: int, seed: int = 0, device="cuda", stream=None) -> torch.Tensor:
    """The resize's per-element PCG32 states (DataLoaderBase::reset,
    dataloader.cu:361-378): tgs_image_blur_state_init."""
    st = torch.empty(max(n, 1), dtype=torch.int64, device=device)
    check(load_library().tgs_image_blur_state_init(st.data_ptr(), n, seed, _stream_handle(stream)),
          "tgs_image_blur_state_init")
    return st


class DataLoaderBase:
    """tinygs::DataLoaderBase (dataloader.hpp:29-96)."""

    NEAR, FAR = 0.1, 100.0  # GPUBatchInput defaults of the reference loaders

    def __init__(self, dataset: ImageDataset, data_type: int = _abi.TGS_FLOAT32, seed: int = 0,
                 device: str | torch.device = "cuda"):
        self.dataset = dataset
        self.data_type = data_type
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.out_w, self.out_h = dataset.width, dataset.height
        self.rng = Pcg32(seed, 1)
        self._blur: torch.Tensor | None = None
        # both reference loaders draw a permutation in their constructor
        self._shuffle()

    def _shuffle(self) -> None:
        self.perm = permutation(self.rng, len(self.dataset))
        self.cursor = 0

    def set_output_shape(self, width: int, height: int) -> None:
        """DataLoaderBase::set_output_shape (dataloader.cu:200-212): the
        targets are resized to width x height from now on."""
        self.out_w, self.out_h = int(width), int(height)
        self.reset()

    def reset(self) -> None:
        raise NotImplementedError

    def _next_index(self) -> int:
        if self.cursor >= len(self.perm):
            self.perm = permutation(self.rng, len(self.dataset))
            self.cursor = 0
        i = self.perm[self.cursor]
        self.cursor += 1
        return i

    def _camera(self, i: int) -> dict:
        c = dict(self.dataset.cameras[i])
        c.update(width=self.out_w, height=self.out_h, near=self.NEAR, far=self.FAR)
        return c

    def _blur_state(self) -> torch.Tensor:
        # sized for the dataset's image (the largest the loader produces),
        # initialised once as the reference does
        if self._blur is None:
            self._blur = blur_state(4 * max(self.dataset.padded_plane(),
                                            ((self.out_w + 7) // 8 * 8) * ((self.out_h + 7) // 8 * 8)),
                                    device=self.device)
        return self._blur

    def _out_numel(self) -> int:
        c = 3 if self.dataset.layout == _abi.TGS_IMAGE_HWC else self.dataset.channels
        return c * ((self.out_w + 7) // 8 * 8) * ((self.out_h + 7) // 8 * 8)


class SimpleDataLoader(DataLoaderBase):
    """tinygs::SimpleDataLoader (simple.cpp): one output buffer; ``next``
    issues the copy and conversion on the caller's stream."""

    def __init__(self, dataset: ImageDataset, data_type: int = _abi.TGS_FLOAT32, seed: int = 0,
                 device: str | torch.device = "cuda"):
        super().__init__(dataset, data_type, seed, device)
        self._alloc()

    def reset(self) -> None:
        """SimpleDataLoader::reset (simple.cpp:97-101): a new permutation."""
        self._shuffle()
        self._alloc()

    def _alloc(self) -> None:
        self.out = torch.empty(self._out_numel(), dtype=_torch_dtype(self.data_type), device=self.device)
        resize = (self.out_w, self.out_h) != (self.dataset.width, self.dataset.height)
        self.conv = _Converter(self.dataset, self.data_type, self.out_w, self.out_h, self.device,
                               self._blur_state() if resize else None)

    def next(self, stream=None) -> Batch:
        i = self._next_index()
        st = stream if isinstance(stream, torch.cuda.Stream) else torch.cuda.current_stream(self.device)
        self.conv.issue(self.dataset.images[i], self.out, st)
        return Batch(self._camera(i), self.out, index=i)


class AsyncDataLoader(DataLoaderBase):
    """tinygs::AsyncDataLoader (async.cpp): a prefetch thread keeps up to
    ``prefetch_factor`` converted targets ready in a device ring.

    ``next(stream)`` hands out the next ready batch and makes `stream` wait
    (on the device) for its conversion; the slot handed out by the previous
    call goes back to the prefetch thread, which reuses it only after the
    work queued on the consumer stream before this call has finished (an
    event, waited for on the prefetch stream)."""

    def __init__(self, dataset: ImageDataset, data_type: int = _abi.TGS_FLOAT32, seed: int = 0,
                 prefetch_factor: int = 4, device: str | torch.device = "cuda"):
        super().__init__(dataset, data_type, seed, device)
        self.prefetch_factor = int(prefetch_factor)
        self._thread: threading.Thread | None = None
        self._lock = threading.Lock()
        self.reset()

    def reset(self) -> None:
        """AsyncDataLoader::reset (async.cpp:331-351): stop the prefetch
        thread, draw a new permutation, restart.  The reference's first
        ``next()`` resets an unstarted loader; the constructor does it here,
        so the first epoch is the second permutation drawn, as there."""
        self.shutdown()
        with self._lock:
            self._shuffle()
        resize = (self.out_w, self.out_h) != (self.dataset.width, self.dataset.height)
        blur = self._blur_state() if resize else None
        dt = _torch_dtype(self.data_type)
        self.slots = [torch.empty(self._out_numel(), dtype=dt, device=self.device)
                      for _ in range(self.prefetch_factor)]
        self.convs = [_Converter(self.dataset, self.data_type, self.out_w, self.out_h, self.device, blur)
                      for _ in range(self.prefetch_factor)]
        self.ready_ev = [torch.cuda.Event() for _ in range(self.prefetch_factor)]
        self.free_ev: list[torch.cuda.Event | None] = [None] * self.prefetch_factor
        self.stream = torch.cuda.Stream(self.device)
        self.free: queue.Queue = queue.Queue()
        self.ready: queue.Queue = queue.Queue()
        for k in range(self.prefetch_factor):
            self.free.put(k)
        self.last_slot = -1
        self._stop = threading.Event()
        self._error: BaseException | None = None
        self._thread = threading.Thread(target=self._prefetch, name="tgs-prefetch", daemon=True)
        self._thread.start()

    def _prefetch(self) -> None:
        try:
            torch.cuda.set_device(self.device)
            while not self._stop.is_set():
                try:
                    k = self.free.get(timeout=0.05)
                except queue.Empty:
                    continue
                if k is None:
                    break
                with self._lock:
                    i = self._next_index()
                if self.free_ev[k] is not None:
                    self.stream.wait_event(self.free_ev[k])  # the consumer is done with the slot
                # the pinned staging buffer is rewritten only after its last copy left
                self.ready_ev[k].synchronize()
                self.convs[k].issue(self.dataset.images[i], self.slots[k], self.stream)
                self.ready_ev[k].record(self.stream)
                self.ready.put((i, k))
        except BaseException as e:  # reported to the consumer by next()
            self._error = e
            self.ready.put(None)

    def next(self, stream=None) -> Batch:
        if self._error is not None:
            raise RuntimeError(f"prefetch thread failed: {self._error}") from self._error
        st = stream if isinstance(stream, torch.cuda.Stream) else torch.cuda.current_stream(self.device)
        if self.last_slot >= 0:
            ev = torch.cuda.Event()
            ev.record(st)
            self.free_ev[self.last_slot] = ev
            self.free.put(self.last_slot)
        item = self.ready.get()
        if item is None:
            raise RuntimeError(f"prefetch thread failed: {self._error}") from self._error
        i, k = item
        st.wait_event(self.ready_ev[k])
        self.last_slot = k
        return Batch(self._camera(i), self.slots[k], index=i, slot=k, ready=self.ready_ev[k])

    def shutdown(self) -> None:
        if self._thread is not None:
            self._stop.set()
            self.free.put(None)
            self._thread.join()
            self._thread = None
            torch.cuda.synchronize(self.device)

    def close(self) -> None:
        self.shutdown()


def create_dataloader(kind: str, dataset: ImageDataset, **kw) -> DataLoaderBase:
    """create_dataloader (dataloader.cu:386-397): "simple" or "async"."""
    k = kind.lower()
    if k == "simple":
        return SimpleDataLoader(dataset, **kw)
    if k == "async":
        return AsyncDataLoader(dataset, **kw)
    raise ValueError(f"Unknown dataloader type: {kind}")
