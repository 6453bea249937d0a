"""The owner's half of the multi-GPU exchange (tgs_dp_inbox_adam) on ONE GPU:
N simulated ranks, each with its own parameter arena, every owner's inbox
holding the N ranks' gradient rows of its slice in its N slots (local
memory).  After every owner has run, every rank's parameters must equal --
bit for bit -- one tgs_adam_step over the rank-order sum of the N gradient
sets: the reference's accumulate_grad_steps = N (orchestrator.cu:343-403),
whose N backward passes add into one arena in view order."""
import ctypes

import numpy as np
import pytest
import torch

from tinygs_b200 import dp as dpm
from tinygs_b200 import runtime as rt
from tinygs_b200 import scenes
from tinygs_b200._abi import TgsGaussians, check

pytestmark = pytest.mark.gpu

WIDTHS = {"means": 3, "opacities": 1, "rotations": 4, "scales": 3, "sh0": 3, "sh_rest": 45}


@pytest.mark.parametrize("world", [2, 4, 8])
def test_inbox_adam_equals_adam_over_summed_gradients(cuda_lib, world):
    n, sh = 10_001, 3
    params = scenes.gaussian_params(n, sh, "normal", 21)
    rng = np.random.default_rng(world)
    grads = [{k: rng.standard_normal(v.shape).astype(np.float32) for k, v in params.items()} for _ in range(world)]
    cfg = rt.AdamParams(max_grad_1=0.3)
    scale = 1.0 / (10.0 * world)
    # one GPU over the summed gradients, summed in rank order
    total = {k: grads[0][k].copy() for k in params}
    for r in range(1, world):
        for k in params:
            total[k] = (total[k] + grads[r][k]).astype(np.float32)
    ref = rt.GaussianSet.from_numpy(params, sh)
    opt = rt.SimpleAdam(ref, rt.GaussianSet.from_numpy(total, sh), cfg)
    opt.step(scale)
    # world ranks: parameter arenas and one inbox per owner
    arenas = [rt.GaussianSet.from_numpy(params, sh) for _ in range(world)]
    lo = [dpm.dp_slice_begin(n, world, r) for r in range(world + 1)]
    slice_pad = (max(lo[r + 1] - lo[r] for r in range(world)) + 3) // 4 * 4
    arr = (TgsGaussians * world)()
    for r, a in enumerate(arenas):
        arr[r] = a.abi()
    lib = rt.load_library()
    c = cfg.abi()
    for owner in range(world):
        inbox = torch.zeros(world * 59 * slice_pad, device="cuda")
        rows = lo[owner + 1] - lo[owner]
        for r in range(world):
            off = r * 59 * slice_pad
            for k, w in WIDTHS.items():
                seg = grads[r][k].reshape(n, w)[lo[owner]:lo[owner + 1]]
                inbox[off: off + w * slice_pad].view(slice_pad, w)[:rows].copy_(torch.from_numpy(seg))
                off += w * slice_pad
        m, v = rt.GaussianSet(n, sh), rt.GaussianSet(n, sh)
        ma, va = m.abi(), v.abi()
        check(lib.tgs_dp_inbox_adam(arr, ctypes.c_void_p(inbox.data_ptr()), slice_pad, world, owner,
                                    ctypes.byref(ma), ctypes.byref(va), ctypes.byref(c), 1, scale,
                                    torch.cuda.current_stream().cuda_stream), "tgs_dp_inbox_adam")
        torch.cuda.synchronize()
    want = ref.to_numpy()
    for r, a in enumerate(arenas):
        got = a.to_numpy()
        for k in want:
            np.testing.assert_array_equal(got[k], want[k], err_msg=f"rank {r} {k}")
