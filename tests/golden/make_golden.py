"""Generate the golden vectors in tests/golden/*.npz from the reference's own brute force.

Run in a container that has the reference checkout ($G2V_REFERENCE_ROOT, else a "reference" folder beside the repo):

    python tests/golden/make_golden.py

It executes the reference's ``test/test_reference.py`` on the CPU: the source is read as text,
``DEVICE = "cuda"`` becomes ``"cpu"``, and the ``CudaGaussianVoxelizer`` import is satisfied by a stub
(the brute force itself never calls the CUDA module).  The reference's ``generate_inputs`` makes the
inputs, and its ``reference_voxelize`` (test/test_reference.py:57-79, float64) produces density,
grid_feats and -- through autograd with float64 leaves -- the gradients of
``sum(density * gD) + sum(grid_feats * gF)`` for randn upstream gradients, as in
test/test_reference.py:103-124.

The reference test takes each Gaussian's voxel box from the CUDA forward (``voxel_boxes``,
test/test_reference.py:48-54).  There is no GPU here, so the boxes come from the oracle's restatement
of src/cuda_gaussian_voxelizer.cu:367-532 instead; they are stored in the fixture so that the check is
the same as the reference's: splat and gradient maths given the boxes.

The GPU box never runs this script; it only reads the committed .npz files.
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from oracle import oracle  # noqa: E402

REF_ROOT = os.environ.get("G2V_REFERENCE_ROOT") or os.path.join(os.path.dirname(REPO), "reference")


def load_reference_test():
    path = os.path.join(REF_ROOT, "test", "test_reference.py")
    with open(path) as fh:
        src = fh.read()
    assert 'DEVICE = "cuda"' in src
    src = src.replace('DEVICE = "cuda"', 'DEVICE = "cpu"')
    stub = types.ModuleType("CudaGaussianVoxelizer")
    stub.PyCudaGaussianVoxelizer = None
    stub._C = None
    sys.modules["CudaGaussianVoxelizer"] = stub
    ns = {"__name__": "reference_test_reference"}
    exec(compile(src, path, "exec"), ns)
    return ns


def set_grid(ns, voxel_size, voxel_range):
    """Point the reference module's grid globals at another grid (they are read at call time)."""
    ns["VOXEL_SIZE"] = list(voxel_size)
    ns["VOXEL_RANGE"] = list(voxel_range)
    ns["lo"] = torch.tensor(voxel_range[:3], dtype=torch.float64)
    ns["hi"] = torch.tensor(voxel_range[3:], dtype=torch.float64)
    ns["vs"] = torch.tensor(voxel_size, dtype=torch.float64)
    X, Y, Z = [int(round(v)) for v in ((ns["hi"] - ns["lo"]) / ns["vs"]).tolist()]
    ns["X"], ns["Y"], ns["Z"] = X, Y, Z
    dims, _ = oracle.grid_shape(voxel_size, voxel_range)
    assert dims == (X, Y, Z), (dims, (X, Y, Z))
    return X, Y, Z


def make_case(ns, name, voxel_size, voxel_range, n, c, n_out, seed, sample_voxels=None):
    X, Y, Z = set_grid(ns, voxel_size, voxel_range)
    means, opacity, cov, feats = ns["generate_inputs"](n, c, num_outside=n_out, seed=seed)
    means, opacity, cov, feats = [t.detach() for t in (means, opacity, cov, feats)]
    bx = oracle.boxes(means.numpy(), cov.numpy(), voxel_size, voxel_range)
    lb = torch.from_numpy(bx.lb).long()
    ub = torch.from_numpy(bx.ub).long()
    torch.manual_seed(seed + 1000)
    gD = torch.randn(X, Y, Z)
    gF = torch.randn(X, Y, Z, c)
    leaves = [t.double().clone().requires_grad_() for t in (means, opacity, cov, feats)]
    density, grid_feats = ns["reference_voxelize"](*leaves, lb, ub)
    ((density * gD.double()).sum() + (grid_feats * gF.double()).sum()).backward()
    out = dict(
        voxel_size=np.asarray(voxel_size, np.float64), voxel_range=np.asarray(voxel_range, np.float64),
        dims=np.asarray([X, Y, Z], np.int32),
        means=means.numpy(), opacity=opacity.numpy(), cov=cov.numpy(), features=feats.numpy(),
        lb=bx.lb, ub=bx.ub, num_voxels=bx.num_voxels, g2t_offsets=bx.g2t_offsets, g2t_tile_ids=bx.g2t_tile_ids,
        grad_density=gD.numpy(), grad_feats=gF.numpy(),
        density=density.detach().numpy(),
        grad_means=leaves[0].grad.numpy(), grad_opacity=leaves[1].grad.numpy(), grad_cov=leaves[2].grad.numpy(),
        grad_features=leaves[3].grad.numpy(),
    )
    gfe = grid_feats.detach().numpy().reshape(X * Y * Z, c)
    if sample_voxels is None:
        out["grid_feats"] = gfe.reshape(X, Y, Z, c)
    else:
        rng = np.random.default_rng(seed)
        idx = np.sort(rng.choice(X * Y * Z, size=sample_voxels, replace=False)).astype(np.int64)
        out["grid_feats_sample_idx"] = idx
        out["grid_feats_sample"] = gfe[idx]
        # size-independent summaries of the whole tensor
        out["grid_feats_sum"] = np.asarray(gfe.sum(), np.float64)
        out["grid_feats_sqsum"] = np.asarray((gfe * gfe).sum(), np.float64)
    # the upstream grad of grid_feats is large; keep it only where the fixture is small
    if sample_voxels is not None:
        del out["grad_feats"]
        out["grad_feats_seed"] = np.asarray(seed + 1000, np.int64)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(f"{name}: N={means.shape[0]} C={c} grid={X}x{Y}x{Z} M={bx.g2t_tile_ids.size}")


def main():
    ns = load_reference_test()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    # ragged grid (10x10x6 -> 3x3x2 tiles), Gaussians inside and beyond x_max
    make_case(ns, "tiny", [0.4, 0.4, 0.4], [-2.0, -2.0, -1.0, 2.0, 2.0, 1.4], 40, 6, 6, seed=3)
    # the reference's backward case, scaled to a 20x20x8 grid
    make_case(ns, "small", [0.4, 0.4, 0.4], [-4.0, -4.0, -1.0, 4.0, 4.0, 2.2], 120, 12, 10, seed=1)
    # density only (no feature channels)
    make_case(ns, "nofeat", [0.4, 0.4, 0.4], [-4.0, -4.0, -1.0, 4.0, 4.0, 2.2], 64, 0, 4, seed=5)
    # anisotropic voxels, ragged 23x8x9 grid
    make_case(ns, "aniso", [0.25, 0.5, 0.375], [-3.0, -2.0, -1.5, 2.75, 2.0, 1.875], 80, 8, 6, seed=7)
    # cfg1 of the benchmark (N=512, C=32, 40x40x16); grid_feats sampled at 400 voxels
    make_case(ns, "cfg1", [0.4, 0.4, 0.4], [-8.0, -8.0, -1.0, 8.0, 8.0, 5.4], 512, 32, 0, seed=0,
              sample_voxels=400)


if __name__ == "__main__":
    main()
