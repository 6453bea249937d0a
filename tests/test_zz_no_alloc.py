"""tgs_loss_l1_ssim_noalloc: the loss entry point for callers that cannot
allocate device memory (hosts whose own pool owns all device memory, or code
running where allocation is not allowed).  It keeps its scratch in a fixed
array inside the library, so its results must equal those of
tgs_loss_l1_ssim, which uses scratch allocated with the TgsLoss handle --
for two calls in a row, so that leftovers of one call cannot leak into the
next.  This file is collected last; it passes alone in a fresh process and
after the other tests."""
import ctypes

import numpy as np
import pytest
import torch

from tinygs_b200 import _abi, scenes
from tinygs_b200.runtime import FusedLoss

pytestmark = pytest.mark.gpu


def _inputs(w, h, seed, dt):
    pred = scenes.target_image(w, h, seed).reshape(-1) * 1.2 - 0.1
    tgt = scenes.target_image(w, h, seed + 1).reshape(-1)
    return (torch.from_numpy(pred.astype(dt)).cuda(), torch.from_numpy(tgt.astype(dt)).cuda())


@pytest.mark.parametrize("dt", [np.float32, np.float16], ids=["fp32", "fp16"])
def test_noalloc_loss_equals_allocating_loss_two_calls(dt):
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    lib = _abi.load_library()
    dtype = _abi.TGS_FLOAT16 if dt == np.float16 else _abi.TGS_FLOAT32
    stream = torch.cuda.current_stream().cuda_stream
    # a full-size call, then smaller ones that reuse the same fixed array:
    # 509 x 507 pads to exactly TGS_NOALLOC_MAX_PIXELS, 203 x 131 has ragged
    # edge tiles in both directions
    shapes = [(512, 512, 30), (200, 136, 40), (509, 507, 50), (203, 131, 60)]
    assert ((509 + 7) // 8 * 8) * ((507 + 7) // 8 * 8) == _abi.TGS_NOALLOC_MAX_PIXELS
    for call, (w, h, seed) in enumerate(shapes):
        pred, tgt = _inputs(w, h, seed, dt)
        ref_loss, ref_grad = torch.zeros_like(pred), torch.zeros_like(pred)
        ref_sum = torch.zeros(1, device="cuda")
        FusedLoss(w, h).evaluate(pred, tgt, ref_loss, ref_grad, w, h, grad_scaler=10.0, loss_sum=ref_sum)
        loss, grad = torch.zeros_like(pred), torch.zeros_like(pred)
        lsum = torch.zeros(1, device="cuda")
        st = lib.tgs_loss_l1_ssim_noalloc(dtype, w, h, pred.data_ptr(), tgt.data_ptr(), loss.data_ptr(),
                                          grad.data_ptr(), 8.0, 2.0, lsum.data_ptr(), stream)
        assert st == _abi.TGS_OK, lib.tgs_status_string(st)
        torch.cuda.synchronize()
        # same kernels on the same inputs: per-pixel results are identical
        np.testing.assert_allclose(loss.float().cpu().numpy(), ref_loss.float().cpu().numpy(), rtol=1e-6, atol=0)
        np.testing.assert_allclose(grad.float().cpu().numpy(), ref_grad.float().cpu().numpy(), rtol=1e-6, atol=0)
        # the scalar is a sum of block partials added atomically in any order
        assert abs(float(lsum.item()) - float(ref_sum.item())) <= 1e-5 * abs(float(ref_sum.item())), call


def test_noalloc_rejects_images_beyond_its_array():
    lib = _abi.load_library()
    w, h = 520, 512  # 520 x 512 > TGS_NOALLOC_MAX_PIXELS
    assert ((w + 7) // 8 * 8) * ((h + 7) // 8 * 8) > _abi.TGS_NOALLOC_MAX_PIXELS
    buf = ctypes.c_void_p(1)  # never dereferenced: the size check comes first
    st = lib.tgs_loss_l1_ssim_noalloc(_abi.TGS_FLOAT32, w, h, buf, buf, buf, buf, 1.0, 1.0, None, None)
    assert st == _abi.TGS_ERR_CAPACITY
    assert lib.tgs_status_string(st) == b"capacity exceeded"
