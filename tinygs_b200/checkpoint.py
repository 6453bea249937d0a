"""Checkpoint and resume of a training run (tgs_checkpoint_save / _info /
_load): the live rows of the parameters, both Adam moments and the
densification statistics, with the step counters and the strategy's PCG32
state.  A run resumed from a checkpoint continues bit for bit where the
saved one stopped.

The reference leaves this to a user callback (Orchestrator::
set_checkpoint_callback, tinygs/src/orchestrator.cu:291-293, called every
checkpoint_interval steps at :433-435) that its example does not set.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

from ._abi import TgsTrainState, check, load_library
from .runtime import Densifier, GaussianSet, SimpleAdam, _stream_handle


@dataclass
class CheckpointInfo:
    n: int
    sh_degree: int
    has_moments: bool
    has_densification: bool
    step: int
    adam_step: int
    strategy_step: int
    rng_state: int
    rng_inc: int


def _path(p) -> bytes:
    return os.fsencode(os.fspath(p))


def save_checkpoint(path, params: GaussianSet, optimizer: SimpleAdam | None = None,
                    densifier: Densifier | None = None, step: int = 0, stream=None) -> None:
    """Write the training state to `path` (synchronises `stream`)."""
    st = TgsTrainState()
    st.step = int(step)
    if optimizer is not None:
        st.adam_step = optimizer.global_steps
    if densifier is not None:
        st.strategy_step = densifier.step_count
        st.rng.state, st.rng.inc = densifier.rng.state, densifier.rng.inc
    p = params.abi()
    m = optimizer.exp_avg.abi() if optimizer is not None else None
    v = optimizer.exp_avg_sq.abi() if optimizer is not None else None
    dens = densifier.dens_storage.data_ptr() if densifier is not None else None
    check(load_library().tgs_checkpoint_save(_path(path), ctypes.byref(p), ctypes.byref(m) if m else None,
                                             ctypes.byref(v) if v else None, dens, ctypes.byref(st),
                                             _stream_handle(stream)), "tgs_checkpoint_save")


def checkpoint_info(path) -> CheckpointInfo:
    n, sh, flags, st = ctypes.c_int64(), ctypes.c_int32(), ctypes.c_uint32(), TgsTrainState()
    check(load_library().tgs_checkpoint_info(_path(path), ctypes.byref(n), ctypes.byref(sh), ctypes.byref(flags),
                                             ctypes.byref(st)), "tgs_checkpoint_info")
    return CheckpointInfo(n.value, sh.value, bool(flags.value & 1), bool(flags.value & 2), st.step, st.adam_step,
                          st.strategy_step, st.rng.state, st.rng.inc)


def load_checkpoint(path, params: GaussianSet, optimizer: SimpleAdam | None = None,
                    densifier: Densifier | None = None, stream=None) -> int:
    """Restore the state saved in `path` into existing objects (arrays with
    room for the saved count; the live counts of the parameters, gradients
    and moments move to it).  Returns the saved training step."""
    p = params.abi()
    m = optimizer.exp_avg.abi() if optimizer is not None else None
    v = optimizer.exp_avg_sq.abi() if optimizer is not None else None
    dens = densifier.dens_storage.data_ptr() if densifier is not None else None
    st = TgsTrainState()
    check(load_library().tgs_checkpoint_load(_path(path), params.capacity, ctypes.byref(p),
                                             ctypes.byref(m) if m else None, ctypes.byref(v) if v else None, dens,
                                             ctypes.byref(st), _stream_handle(stream)), "tgs_checkpoint_load")
    params.sh_degree = p.sh_degree
    sets = [params]
    if optimizer is not None:
        optimizer.global_steps = int(st.adam_step)
        sets += [optimizer.exp_avg, optimizer.exp_avg_sq]
        if optimizer.grads is not None:
            sets.append(optimizer.grads)
    if densifier is not None:
        densifier.step_count = int(st.strategy_step)
        densifier.rng.state, densifier.rng.inc = st.rng.state, st.rng.inc
        if densifier.grads is not None:
            sets.append(densifier.grads)
    for s in sets:
        s.resize(p.n)
    return int(st.step)
