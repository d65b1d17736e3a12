"""Generate tests/golden/cov_scale_rot.npz from the reference's own GaussTR front end.

Run in a container that has the reference checkout ($G2V_REFERENCE_ROOT, else a "reference" folder beside the repo):

    python tests/golden/make_golden_cov.py

It imports the reference's ``test/gaussian_voxelizer.py`` (plain PyTorch) and runs its ``quat_to_rotmat``
and ``get_covariance`` (:14-37) in float64 on batched (1, N) inputs, as ``GaussianVoxelizer.forward``
(:176-177) calls them; the gradients of sum(Sigma * G) for a randn G come from autograd through those
functions.  The GPU box never runs this script; it only reads the committed .npz file.
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from oracle import oracle  # noqa: E402

REF_ROOT = os.environ.get("G2V_REFERENCE_ROOT") or os.path.join(os.path.dirname(REPO), "reference")


def load_front_end():
    path = os.path.join(REF_ROOT, "test", "gaussian_voxelizer.py")
    spec = importlib.util.spec_from_file_location("reference_gaussian_voxelizer", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    ref = load_front_end()
    s32, q32 = oracle.generate_scale_rot(257, seed=21)
    q32[:3] = torch.tensor([[1.0, 0, 0, 0], [0, 1.0, 0, 0], [0.5, 0.5, 0.5, 0.5]])  # exact rotations
    s = s32.double()[None].requires_grad_(True)
    q = q32.double()[None].requires_grad_(True)
    cov = ref.get_covariance(s, ref.quat_to_rotmat(q))
    G = torch.randn(cov.shape, generator=torch.Generator().manual_seed(22), dtype=torch.float64)
    (cov * G).sum().backward()
    out = os.path.join(HERE, "cov_scale_rot.npz")
    np.savez_compressed(out, scales=s32.numpy(), rotations=q32.numpy(), cov=cov.detach()[0].numpy(),
                        grad_cov=G[0].numpy(), grad_scales=s.grad[0].numpy(), grad_rotations=q.grad[0].numpy())
    print("wrote", out)


if __name__ == "__main__":
    main()
