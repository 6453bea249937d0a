"""Generates the golden vectors of tests/golden/ from the reference's own
CUDA kernels (oracle/_ref/libtgs_ref.so: Adversarr/tinygs
fastgs_ours/, fastgs_ours_fp16/, loss/l1.cu, loss/fused_ssim.cu, built
unchanged by oracle/build_ref.py).  Needs a GPU; run from the repository root:

    python tests/golden/make_reference_golden.py [output_dir]

(output_dir defaults to tests/golden/).

Scene: 1,000 Gaussians, SH degree 1, BASELINE config 0's distributions
(means U[-1,1]^3, log-scales N(-4, 0.5), normalised N(0,1) quaternions,
opacity logits N(0,1), RGB U[0,1]) seen from distance 3 by a 96 x 96 pinhole
camera (fx = fy = 110), in both rasterizer precisions.  For each precision
the reference renders, evaluates 0.8 L1 + 0.2 (1 - SSIM) with grad_scaler 10
(L1Loss::evaluate(ctx, 8), FusedSSIMLoss::evaluate(ctx, 2) against a seeded
U[0,1] target) and runs its backward on that gradient image.

Written: reference_scene.npz (the inputs) and reference_fp32.npz /
reference_fp16.npz (outputs).  Instances are stored in (tile, depth, index)
order: the reference orders equal depths by atomic arrival, and the few such
ties are put in index order so the file does not depend on the run.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

N, SH, W, H, F = 1000, 1, 96, 96, 110.0
SCENE_SEED, TARGET_SEED = 2024, 2025
OUT = Path(__file__).resolve().parent


def scene():
    from tinygs_b200 import scenes

    params = scenes.gaussian_params(N, SH, "uniform", SCENE_SEED)
    cfg = scenes.CONFIGS["cfg0"]
    cam = scenes.camera_dict(cfg, scenes.look_at_w2c((0.0, 0.0, -cfg.cam_distance)))
    cam.update(width=W, height=H, fx=F, fy=F, cx=W / 2, cy=H / 2)
    target = scenes.target_image(W, H, TARGET_SEED).reshape(-1)
    return params, cam, target


def main(out_dir: Path = OUT) -> None:
    import torch

    from oracle import refpy
    from tinygs_b200 import runtime as rt

    params, cam, target = scene()
    out_dir.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(out_dir / "reference_scene.npz", w2c=np.asarray(cam["w2c"], np.float32),
                        intrinsics=np.array([W, H, F, F, W / 2, H / 2, cam.get("near", 0.01), cam.get("far", 100.0)],
                                            np.float32),
                        sh_degree=np.int32(SH), target=target.astype(np.float32),
                        **{f"param_{k}": v.astype(np.float32) for k, v in params.items()})
    g = rt.GaussianSet.from_numpy(params, SH)
    gw, gh = (W + 15) // 16, (H + 15) // 16
    T = gw * gh
    pl = rt.image_numel(W, H) // 3
    for fp16 in (False, True):
        dt = torch.float16 if fp16 else torch.float32
        ref = refpy.RefRasterizer()
        img = torch.zeros(3 * pl, dtype=dt, device="cuda")
        V, I, B = ref.forward(g, cam, img, fp16)
        n_touched = ref.copy(refpy.N_TOUCHED, np.uint32, N)
        keys = ref.copy(refpy.INST_KEYS, np.uint32 if fp16 else np.uint16, I).astype(np.int64)
        prims = ref.copy(refpy.INST_PRIMS, np.uint32, I).astype(np.int64)
        sp = ref.copy(refpy.SORTED_PRIMS, np.uint32, V).astype(np.int64)
        sk = ref.copy(refpy.SORTED_DEPTH_KEYS, np.uint32, V).astype(np.int64)
        depth_of = np.zeros(N, np.int64)
        depth_of[sp] = sk
        order = np.lexsort((prims, depth_of[prims], keys))
        res = {"counts": np.array([V, I, B], np.int64), "n_touched": n_touched,
               "inst_tile": keys[order].astype(np.uint32), "inst_prim": prims[order].astype(np.uint32),
               "depth_key": depth_of.astype(np.uint32),
               "ranges": ref.copy(refpy.TILE_RANGES, np.uint32, 2 * T).reshape(T, 2),
               "bucket_offsets": ref.copy(refpy.BUCKET_OFFSETS, np.uint32, T),
               "tile_max": ref.copy(refpy.TILE_MAX_CONTRIB, np.uint16 if fp16 else np.uint32, T),
               "n_contrib": ref.copy(refpy.N_CONTRIB, np.uint16 if fp16 else np.uint32, pl),
               "bounds": ref.copy(refpy.BOUNDS, np.uint16, 4 * N).reshape(N, 4),
               "mean2d": ref.copy(refpy.MEAN2D, np.float32, 2 * N).reshape(N, 2),
               "image": img.cpu().numpy(),
               "alpha": ref.copy(refpy.ALPHA, np.float16 if fp16 else np.float32, pl)}
        if fp16:
            res["prim_info"] = ref.copy(refpy.CONIC_OPACITY, np.uint8, 16 * N).reshape(N, 16)
        else:
            res["conic_opacity"] = ref.copy(refpy.CONIC_OPACITY, np.float32, 4 * N).reshape(N, 4)
            res["color"] = ref.copy(refpy.COLOR, np.float32, 3 * N).reshape(N, 3)
        tgt = torch.from_numpy(target).to(dt).cuda()
        loss_map, grad_img = torch.zeros_like(img), torch.zeros_like(img)
        refpy.l1(fp16, W, H, img, tgt, loss_map, grad_img, 8.0)
        ref.ssim(fp16, W, H, img, tgt, loss_map, grad_img, 2.0)
        grads = g.zeros_like()
        ref.backward(g, cam, img, grad_img, grads, fp16)
        torch.cuda.synchronize()
        res["loss_map"] = loss_map.cpu().numpy()
        res["grad_image"] = grad_img.cpu().numpy()
        for k, v in grads.to_numpy().items():
            res[f"grad_{k}"] = v
        if not fp16:
            res["screen_grad_mean2d"] = ref.copy(refpy.GRAD_MEAN2D, np.float32, 2 * N).reshape(N, 2)
            res["screen_grad_conic"] = ref.copy(refpy.GRAD_CONIC, np.float32, 3 * N).reshape(3, N).T.copy()
            res["screen_grad_color"] = ref.copy(refpy.GRAD_COLOR, np.float32, 3 * N).reshape(N, 3)
        np.savez_compressed(out_dir / f"reference_{'fp16' if fp16 else 'fp32'}.npz", **res)
        ref.close()
        print(f"fp16={fp16}: V={V} I={I} B={B}")


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else OUT)
