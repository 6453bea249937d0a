"""Device-side PSNR (tgs_metric_psnr) against a numpy restatement of
PsnrMetric::evaluate (tinygs/src/loss/psnr.cu:72-128): the prediction is
saturated to [0, 1], MSE = sum of squared differences over the physical
(padded, zero-filled) elements / (3 W H), PSNR = -10 log10(MSE), 100 for a
perfect match.  The reference sums in float with thrust (order unspecified);
both sides here agree to 1e-6 relative."""
import numpy as np
import pytest
import torch

from tinygs_b200 import runtime as rt
from tinygs_b200 import scenes

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", [np.float32, np.float16], ids=["fp32", "fp16"])
@pytest.mark.parametrize("wh", [(1920, 1080), (203, 131)])
def test_psnr_matches_numpy(cuda_lib, dt, wh):
    w, h = wh
    pred = (scenes.target_image(w, h, 3).reshape(-1) * 1.3 - 0.15).astype(dt)
    tgt = scenes.target_image(w, h, 4).reshape(-1).astype(dt)
    out = rt.psnr(torch.from_numpy(pred).cuda(), torch.from_numpy(tgt).cuda(), w, h).cpu().numpy()
    d = np.clip(pred.astype(np.float64), 0, 1) - tgt.astype(np.float64)
    mse = float((d * d).sum() / (3 * w * h))
    assert abs(out[0] - mse) <= 1e-6 * mse
    assert abs(out[1] - (-10 * np.log10(mse))) <= 1e-5
    same = rt.psnr(torch.from_numpy(tgt).cuda(), torch.from_numpy(tgt).cuda(), w, h).cpu().numpy()
    assert same[0] == 0.0 and same[1] == 100.0
