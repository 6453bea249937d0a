"""Data-parallel training over several GPUs: one process per GPU, each rank
renders its own view of the replicated model per step, the gradient arenas
are summed with one all-reduce, and every rank applies the same Adam step.

This is the reference's gradient accumulation over several views
(Orchestrator::train_step with accumulate_grad_steps = N,
tinygs/src/orchestrator.cu:343-403: N backward passes add into one gradient
arena, then one optimizer step with gradient scale 1/(grad_scaler * N)),
with the N views of one optimizer step rendered on N GPUs at once.  Any
torch.distributed backend works (NCCL on GPUs, gloo in the CPU tests).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


def _as_torch_stream(stream) -> torch.cuda.Stream:
    """`stream` as a torch stream object (None: the current stream; a raw
    cudaStream_t handle is wrapped as an external stream)."""
    if stream is None:
        return torch.cuda.current_stream()
    if isinstance(stream, torch.cuda.Stream):
        return stream
    return torch.cuda.ExternalStream(int(stream))


@dataclass
class DataParallel:
    world: int = 1
    rank: int = 0
    group: object = None

    @classmethod
    def from_env(cls, group=None) -> "DataParallel":
        if dist.is_available() and dist.is_initialized():
            return cls(dist.get_world_size(group), dist.get_rank(group), group)
        return cls()

    def view_index(self, step: int, n_views: int) -> int:
        """View rendered by this rank at `step`: the N ranks of one step take
        N consecutive views of the orbit, so one step covers the same views
        the reference's accumulation loop would take in N iterations."""
        return (step * self.world + self.rank) % n_views

    def gradient_scale(self, grad_scaler: float) -> float:
        """Adam's gradient scale after the sum over ranks."""
        return 1.0 / (grad_scaler * self.world)

    def reduce_gradients(self, grads: torch.Tensor) -> torch.Tensor:
        """Sum the gradient arena over the ranks in place (one collective)."""
        if self.world > 1:
            dist.all_reduce(grads, op=dist.ReduceOp.SUM, group=self.group)
        return grads

    def max_over_ranks(self, value: float, device) -> float:
        """Largest value over the ranks (timings are reported as the max)."""
        if self.world == 1:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return float(t.item())


# ------------------------------------------------------------------------
# Accumulation + Adam as one kernel over NVLink peer memory (the product path
# for several GPUs; `reduce_gradients` + a local Adam is the NCCL baseline).

import ctypes  # noqa: E402

from . import runtime as rt  # noqa: E402
from ._abi import TgsGaussians, TgsIpcHandle, check, load_library  # noqa: E402


def shared_gaussian_set(n: int, sh_degree: int, capacity: int | None = None) -> "rt.GaussianSet":
    """A GaussianSet whose storage other processes can map (CUDA IPC).  The
    allocation is released when the set is garbage collected."""
    lib = load_library()
    cap = max(int(n), int(capacity) if capacity is not None else int(n))
    npad = (cap + 3) // 4 * 4
    nbytes = 4 * rt.FLOATS_PER_GAUSSIAN * npad
    ptr, handle = ctypes.c_void_p(), TgsIpcHandle()
    check(lib.tgs_shared_alloc(nbytes, ctypes.byref(ptr), ctypes.byref(handle)), "tgs_shared_alloc")
    view = rt._DeviceView(ptr.value, rt.FLOATS_PER_GAUSSIAN * npad, "<f4")
    storage = torch.as_tensor(view, device="cuda")
    g = rt.GaussianSet(n, sh_degree, storage=storage, capacity=cap)
    g.ipc_handle = handle.raw()
    g._shared = _SharedBlock(lib, ptr.value)
    return g


class _SharedBlock:
    def __init__(self, lib, ptr: int):
        self.lib, self.ptr = lib, ptr

    def __del__(self):
        try:
            self.lib.tgs_shared_free(ctypes.c_void_p(self.ptr))
        except Exception:
            pass


class PeerAdam:
    """Data-parallel optimizer step over peer memory (tgs_dp_reduce_adam).

    Every rank holds the parameters and its gradient arena in shared memory;
    the arenas of all ranks are mapped into every process once.  step()
    orders itself after every rank's backward and before every rank's next
    forward with a one-element all-reduce on the stream, then rank r sums
    the gradients of its slice of the Gaussians over the ranks, applies
    Adam with its moments, and writes the new parameters into every rank's
    arena."""

    def __init__(self, dp: DataParallel, params: "rt.GaussianSet", grads: "rt.GaussianSet",
                 cfg: "rt.AdamParams | None" = None):
        self.lib = load_library()
        self.dp, self.params, self.grads = dp, params, grads
        self.cfg = cfg or rt.AdamParams()
        self.exp_avg = params.zeros_like()
        self.exp_avg_sq = params.zeros_like()
        self.global_steps = 0
        self.flag = torch.zeros(1, dtype=torch.float32, device="cuda")
        handles = [None] * dp.world
        mine = (params.ipc_handle, grads.ipc_handle)
        if dp.world > 1:
            dist.all_gather_object(handles, mine, group=dp.group)
        else:
            handles = [mine]
        self.opened: list[int] = []
        base_p, base_g = [], []
        for r, (hp, hg) in enumerate(handles):
            if r == dp.rank:
                base_p.append(params.storage.data_ptr())
                base_g.append(grads.storage.data_ptr())
                continue
            ptrs = []
            for h in (hp, hg):
                ih = TgsIpcHandle.from_raw(h)
                p = ctypes.c_void_p()
                check(self.lib.tgs_shared_open(ctypes.byref(ih), ctypes.byref(p)), "tgs_shared_open")
                self.opened.append(p.value)
                ptrs.append(p.value)
            base_p.append(ptrs[0])
            base_g.append(ptrs[1])
        self.base_p, self.base_g = base_p, base_g

    def _sets(self, bases: list[int], like: "rt.GaussianSet"):
        arr = (TgsGaussians * self.dp.world)()
        offs, off = {}, 0
        for name in rt.SEGMENTS:
            offs[name] = off
            off += rt.WIDTHS[name] * like.npad
        for r, b in enumerate(bases):
            for name in rt.SEGMENTS:
                setattr(arr[r], name, b + 4 * offs[name])
            arr[r].n = like.n
            arr[r].sh_degree = like.sh_degree
        return arr

    def barrier(self, stream=None) -> None:
        """A one-element all-reduce ordered on `stream` (torch's current
        stream if None): the exchange kernel launched on that stream runs
        after every rank's earlier work on its own stream."""
        if self.dp.world > 1:
            with torch.cuda.stream(_as_torch_stream(stream)):
                dist.all_reduce(self.flag, group=self.dp.group)

    def step(self, gradient_scale: float, stream=None, events=None) -> None:
        """`events`: optional pair of CUDA events recorded around the kernel
        (between the two barriers)."""
        if stream is None:
            stream = torch.cuda.current_stream()
        self.global_steps += 1
        P = self._sets(self.base_p, self.params)
        G = self._sets(self.base_g, self.grads)
        m, v = self.exp_avg.abi(), self.exp_avg_sq.abi()
        cfg = self.cfg.abi()
        self.barrier(stream)  # every rank's gradients are written
        if events is not None:
            events[0].record(stream)
        check(self.lib.tgs_dp_reduce_adam(P, G, self.dp.world, self.dp.rank, ctypes.byref(m), ctypes.byref(v),
                                          ctypes.byref(cfg), self.global_steps, float(gradient_scale),
                                          rt._stream_handle(stream)), "tgs_dp_reduce_adam")
        if events is not None:
            events[1].record(stream)
        self.barrier(stream)  # every rank's parameters are updated

    def close(self) -> None:
        for p in self.opened:
            self.lib.tgs_shared_close(ctypes.c_void_p(p))
        self.opened = []


# ------------------------------------------------------------------------
# The same exchange through NVLink SHARP (multimem loads that reduce in the
# switch and multimem stores that reach every GPU), over arenas allocated in
# torch's symmetric memory, which binds them to a multicast object.

def symmetric_gaussian_set(dp: DataParallel, n: int, sh_degree: int) -> "rt.GaussianSet":
    """A GaussianSet in symmetric memory (collective: every rank calls it
    with the same n); `.symm` is the rendezvous handle."""
    import torch.distributed._symmetric_memory as symm_mem

    npad = (int(n) + 3) // 4 * 4
    t = symm_mem.empty(rt.FLOATS_PER_GAUSSIAN * npad, dtype=torch.float32, device="cuda")
    t.zero_()
    h = symm_mem.rendezvous(t, dp.group if dp.group is not None else dist.group.WORLD)
    g = rt.GaussianSet(n, sh_degree, storage=t)
    g.symm = h
    return g


class MulticastAdam:
    """PeerAdam through the switch: rank r reads its slice's gradient sum with
    one reducing load per 16 bytes and writes the new parameters to every
    rank with one multicast store (tgs_dp_reduce_adam_multicast).  Raises
    RuntimeError when the arenas have no multicast address."""

    def __init__(self, dp: DataParallel, params: "rt.GaussianSet", grads: "rt.GaussianSet",
                 cfg: "rt.AdamParams | None" = None):
        self.lib = load_library()
        self.dp, self.params, self.grads = dp, params, grads
        self.cfg = cfg or rt.AdamParams()
        self.exp_avg = params.zeros_like()
        self.exp_avg_sq = params.zeros_like()
        self.global_steps = 0
        self.flag = torch.zeros(1, dtype=torch.float32, device="cuda")
        self.mc = []
        for s in (params, grads):
            mc = int(s.symm.multicast_ptr)
            if mc == 0:
                raise RuntimeError("no multicast address for the symmetric arenas (NVLink SHARP unavailable)")
            self.mc.append(mc)

    def _mc_set(self, mc_base: int, like: "rt.GaussianSet") -> TgsGaussians:
        local = like.abi()
        base = like.storage.data_ptr()
        out = TgsGaussians()
        for name in rt.SEGMENTS:
            setattr(out, name, mc_base + (getattr(local, name) - base))
        out.n, out.sh_degree = like.n, like.sh_degree
        return out

    def barrier(self, stream=None) -> None:
        """A one-element all-reduce ordered on `stream` (torch's current
        stream if None): the exchange kernel launched on that stream runs
        after every rank's earlier work on its own stream."""
        if self.dp.world > 1:
            with torch.cuda.stream(_as_torch_stream(stream)):
                dist.all_reduce(self.flag, group=self.dp.group)

    def step(self, gradient_scale: float, stream=None, events=None) -> None:
        if stream is None:
            stream = torch.cuda.current_stream()
        self.global_steps += 1
        pm, gm = self._mc_set(self.mc[0], self.params), self._mc_set(self.mc[1], self.grads)
        p, m, v = self.params.abi(), self.exp_avg.abi(), self.exp_avg_sq.abi()
        cfg = self.cfg.abi()
        self.barrier(stream)
        if events is not None:
            events[0].record(stream)
        check(self.lib.tgs_dp_reduce_adam_multicast(ctypes.byref(pm), ctypes.byref(gm), ctypes.byref(p),
                                                    self.dp.world, self.dp.rank, ctypes.byref(m), ctypes.byref(v),
                                                    ctypes.byref(cfg), self.global_steps, float(gradient_scale),
                                                    rt._stream_handle(stream)), "tgs_dp_reduce_adam_multicast")
        if events is not None:
            events[1].record(stream)
        self.barrier(stream)

    def close(self) -> None:
        pass


# ------------------------------------------------------------------------
# Gradient routing: the backward stores each Gaussian's gradients straight
# into the gradient inbox of the rank that owns it, so the gradient transfer
# overlaps the backward; the exchange kernel then sums the local inbox slots
# and only broadcasts the new parameters.

def dp_slice_begin(n: int, world: int, r: int) -> int:
    """First Gaussian of rank r's slice (as the C library cuts them)."""
    return n if r >= world else (n * r // world) // 4 * 4


class InboxAdam:
    """Routed data-parallel step.  Usage per training step:
    `rast.backward_routed(ctx, *opt.route())` after the forward and loss, then
    `opt.step(scale)` (barrier, tgs_dp_inbox_adam, barrier)."""

    def __init__(self, dp: DataParallel, params: "rt.GaussianSet", cfg: "rt.AdamParams | None" = None):
        self.lib = load_library()
        self.dp, self.params = dp, params
        self.cfg = cfg or rt.AdamParams()
        self.exp_avg = params.zeros_like()
        self.exp_avg_sq = params.zeros_like()
        self.global_steps = 0
        self.flag = torch.zeros(1, dtype=torch.float32, device="cuda")
        n, w = params.n, dp.world
        widest = max(dp_slice_begin(n, w, r + 1) - dp_slice_begin(n, w, r) for r in range(w))
        self.slice_pad = (widest + 3) // 4 * 4
        nbytes = 4 * rt.FLOATS_PER_GAUSSIAN * self.slice_pad * w
        ptr, handle = ctypes.c_void_p(), TgsIpcHandle()
        check(self.lib.tgs_shared_alloc(max(nbytes, 256), ctypes.byref(ptr), ctypes.byref(handle)),
              "tgs_shared_alloc")
        self.inbox = ptr.value
        self._inbox_block = _SharedBlock(self.lib, ptr.value)
        handles = [None] * w
        mine = (params.ipc_handle, handle.raw())
        if w > 1:
            dist.all_gather_object(handles, mine, group=dp.group)
        else:
            handles = [mine]
        self.opened: list[int] = []
        self.base_p, self.inboxes = [], []
        for r, (hp, hi) in enumerate(handles):
            if r == dp.rank:
                self.base_p.append(params.storage.data_ptr())
                self.inboxes.append(self.inbox)
                continue
            ptrs = []
            for h in (hp, hi):
                p = ctypes.c_void_p()
                check(self.lib.tgs_shared_open(ctypes.byref(TgsIpcHandle.from_raw(h)), ctypes.byref(p)),
                      "tgs_shared_open")
                self.opened.append(p.value)
                ptrs.append(p.value)
            self.base_p.append(ptrs[0])
            self.inboxes.append(ptrs[1])

    def route(self):
        """Arguments of FastGSB200Rasterizer.backward_routed after ctx."""
        return self.inboxes, self.slice_pad, self.dp.world, self.dp.rank

    def barrier(self, stream=None) -> None:
        """A one-element all-reduce ordered on `stream` (torch's current
        stream if None): the exchange kernel launched on that stream runs
        after every rank's earlier work on its own stream."""
        if self.dp.world > 1:
            with torch.cuda.stream(_as_torch_stream(stream)):
                dist.all_reduce(self.flag, group=self.dp.group)

    def step(self, gradient_scale: float, stream=None, events=None) -> None:
        if stream is None:
            stream = torch.cuda.current_stream()
        self.global_steps += 1
        arr = (TgsGaussians * self.dp.world)()
        offs, off = {}, 0
        for name in rt.SEGMENTS:
            offs[name] = off
            off += rt.WIDTHS[name] * self.params.npad
        for r, b in enumerate(self.base_p):
            for name in rt.SEGMENTS:
                setattr(arr[r], name, b + 4 * offs[name])
            arr[r].n, arr[r].sh_degree = self.params.n, self.params.sh_degree
        m, v = self.exp_avg.abi(), self.exp_avg_sq.abi()
        cfg = self.cfg.abi()
        self.barrier(stream)  # every rank's routed gradients have landed
        if events is not None:
            events[0].record(stream)
        check(self.lib.tgs_dp_inbox_adam(arr, ctypes.c_void_p(self.inbox), self.slice_pad, self.dp.world,
                                         self.dp.rank, ctypes.byref(m), ctypes.byref(v), ctypes.byref(cfg),
                                         self.global_steps, float(gradient_scale), rt._stream_handle(stream)),
              "tgs_dp_inbox_adam")
        if events is not None:
            events[1].record(stream)
        self.barrier(stream)  # every rank's parameters are updated

    def close(self) -> None:
        for p in self.opened:
            self.lib.tgs_shared_close(ctypes.c_void_p(p))
        self.opened = []


# ------------------------------------------------------------------------
# Owner-split step: every rank owns a slice of the Gaussians (parameters and
# Adam moments) and renders one view.  Only screen-space records (owner ->
# view) and screen-space gradients (view -> owner) cross NVLink; nothing is
# broadcast, and the per-Gaussian backward + Adam work is split N ways.

def owner_slice(n: int, world: int, r: int) -> tuple[int, int]:
    """Rank r's Gaussians [first, last): starts on multiples of 256 (one
    preprocess block has one owner)."""
    def begin(k):
        return n if k >= world else (n * k // world) // 256 * 256
    return begin(r), begin(r + 1)


class OwnerSplit:
    """Owner-split data-parallel training step over the ranks of `dp`
    (tgs_raster_preprocess_views / forward_gathered / backward_screen /
    backward_views_adam).  Per step:

        opt.forward(cams_of_all_ranks, image)        # records to the views, barrier, bin + blend
        (loss into grad_image)
        opt.backward_adam(cams_of_all_ranks, image, grad_image, scale)

    Every rank holds the full parameter arena, but only its slice's rows are
    read (preprocess, backward) and updated (Adam); the moments likewise."""

    def __init__(self, dp: DataParallel, rast: "rt.FastGSB200Rasterizer", params: "rt.GaussianSet",
                 cfg: "rt.AdamParams", dtype: int):
        self.dp, self.rast, self.params, self.cfg, self.dtype = dp, rast, params, cfg, dtype
        self.lib = load_library()
        self.first, self.last = owner_slice(params.n, dp.world, dp.rank)
        self.exp_avg, self.exp_avg_sq = params.zeros_like(), params.zeros_like()
        self.global_steps = 0
        self.flag = torch.zeros(1, device=params.storage.device)
        mine = rast.share()
        handles = [mine] * dp.world
        if dp.world > 1:
            handles = [None] * dp.world
            dist.all_gather_object(handles, mine, group=dp.group)
        self.opened: list[int] = []
        arenas = []
        for r, h in enumerate(handles):
            if r == dp.rank:
                arenas.append(rast.arena())
                continue
            p = ctypes.c_void_p()
            check(self.lib.tgs_shared_open(ctypes.byref(TgsIpcHandle.from_raw(h)), ctypes.byref(p)),
                  "tgs_shared_open")
            self.opened.append(p.value)
            arenas.append(p.value)
        rast.attach_views(arenas, dp.rank)

    def barrier(self, stream=None) -> None:
        if self.dp.world > 1:
            with torch.cuda.stream(_as_torch_stream(stream)):
                dist.all_reduce(self.flag, group=self.dp.group)

    def forward(self, cams: list[dict], image: torch.Tensor, dens: torch.Tensor | None = None, stream=None,
                events=None) -> None:
        """This rank's slice preprocessed for every view, then (after every
        owner's records have landed) this rank's view binned and blended."""
        self.rast.preprocess_views(self.params, cams, self.dtype, self.first, self.last, dens, stream)
        if events is not None:
            events[0].record(_as_torch_stream(stream))
        self.barrier(stream)
        if events is not None:
            events[1].record(_as_torch_stream(stream))
        self.rast.forward_gathered(self.params.n, cams[self.dp.rank], image, stream=stream)

    def backward_adam(self, cams: list[dict], image: torch.Tensor, grad_image: torch.Tensor,
                      gradient_scale: float, dens: torch.Tensor | None = None, stream=None, events=None) -> None:
        """Blend backward of this rank's view, then (after every view's
        screen-space gradients are in place) this rank's slice: per-Gaussian
        backward for every view, summed in view order, and Adam."""
        self.global_steps += 1
        self.rast.backward_screen(cams[self.dp.rank], image, grad_image, False, stream)
        if events is not None:
            events[0].record(_as_torch_stream(stream))
        self.barrier(stream)
        if events is not None:
            events[1].record(_as_torch_stream(stream))
        self.rast.backward_views_adam(self.params, cams, self.first, self.last, None, self.exp_avg,
                                      self.exp_avg_sq, self.cfg, self.global_steps, gradient_scale, dens, stream)

    def close(self) -> None:
        for p in self.opened:
            self.lib.tgs_shared_close(ctypes.c_void_p(p))
        self.opened = []
