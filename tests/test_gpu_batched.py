"""GPU checks of the batched multi-scene path (one prepare / splat / backward for B scenes).

Scenes are stacked along x inside the library (volumes (B, X, Y, Z[, C])); each scene's result must be
that of a single-scene call on its own Gaussians:
  * boxes, counts and the Gaussian->Tile CSR bit-identical after the stacking shift (x + b X, tile id
    + b T, offsets + the earlier scenes' pairs);
  * density, grid_feats and every gradient within 1e-6 relative of the single-scene calls (the forward's
    fp16 split takes one power-of-two scale per channel over the whole batch, so the last bits may
    differ) and within the parity bar of the float64 oracle;
  * ragged sizes including an empty scene, the (B, N, ...) form through the module, scale/rotation
    inputs, and the error for an X that is not a multiple of 4.
"""
import numpy as np
import pytest
import torch

from gpu_util import assert_close
from oracle import oracle

pytestmark = pytest.mark.gpu

SIZE, RNG = [0.4] * 3, [-8.0, -8.0, -1.0, 8.0, 8.0, 5.4]  # 40 x 40 x 16


def _scene(n, c, seed):
    m, o, cov, f = oracle.generate_inputs(n, c, RNG, seed=seed, expand=0.05)
    return [t.cuda() for t in (m, o, cov, f)]


def _close(name, a, b, rtol=1e-6):
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    assert a.shape == b.shape, (name, a.shape, b.shape)
    if b.numel():
        err = float((a - b).norm() / max(float(b.norm()), 1e-30))
        assert err < rtol, f"{name}: relative L2 {err:.2e}"


@pytest.mark.parametrize("sizes,c", [([500, 0, 700], 16), ([300, 300], 0), ([1], 8)])
def test_forward_matches_single_scene_calls(sizes, c):
    from CudaGaussianVoxelizer import _C
    scenes = [_scene(n, max(c, 1), seed=40 + i) for i, n in enumerate(sizes)]
    cat = [torch.cat([sc[k] for sc in scenes]) for k in range(4)]
    feats = cat[3][:, :c].contiguous() if c > 0 else None
    off, B = _C._scene_offsets(sizes, sum(sizes), cat[0].device)
    (out, mb) = _C._forward_impl(cat[0], cat[1], cat[2], SIZE, RNG, feats, False, scenes=(off, B))
    density, cov_inv, lb, ub, nvox, grid_feats, g2t_off, g2t_ids, _ = out
    (X, Y, Z), (Tx, Ty, Tz) = _C.grid_shape(SIZE, RNG)
    assert density.shape == (B, X, Y, Z) and grid_feats.shape == (B, X, Y, Z, c)
    g0, p0 = 0, 0
    for b, n in enumerate(sizes):
        f = scenes[b][3][:, :c].contiguous() if c > 0 else None
        (one, _) = _C._forward_impl(*scenes[b][:3], SIZE, RNG, f, False, plan=True)
        sl = slice(g0, g0 + n)
        shift = torch.tensor([b * X, 0, 0], dtype=torch.int32, device="cuda")
        live = one[4] > 0  # empty boxes stay (0, -1)
        assert torch.equal(lb[sl][live], (one[2] + shift)[live]) and torch.equal(ub[sl][live], (one[3] + shift)[live])
        assert torch.equal(nvox[sl], one[4]) and torch.equal(cov_inv[sl], one[1])
        m1 = int(one[6][-1])
        assert torch.equal(g2t_off[g0:g0 + n + 1] - p0, one[6])
        assert torch.equal(g2t_ids[p0:p0 + m1], one[7] + b * Tx * Ty * Tz)
        _close(f"density[{b}]", density[b], one[0])
        _close(f"grid_feats[{b}]", grid_feats[b], one[5])
        g0 += n
        p0 += m1


def test_module_batch_dimension_with_gradients():
    from CudaGaussianVoxelizer import PyCudaGaussianVoxelizer
    B, n, c = 3, 400, 12
    scenes = [_scene(n, c, seed=60 + b) for b in range(B)]
    vox = PyCudaGaussianVoxelizer(voxel_size=SIZE, voxel_range=RNG)
    leaves = [torch.stack([sc[k] for sc in scenes]).requires_grad_(True) for k in range(4)]
    density, grid_feats, stats = vox(leaves[0], leaves[1], leaves[2], leaves[3])
    gen = torch.Generator("cuda").manual_seed(5)
    gD = torch.randn(density.shape, device="cuda", generator=gen)
    gF = torch.randn(grid_feats.shape, device="cuda", generator=gen)
    torch.autograd.backward([density, grid_feats], [gD, gF])
    assert stats[0] > 0 and stats[1] > 0
    for b in range(B):
        ls = [t.clone().requires_grad_(True) for t in scenes[b]]
        d1, f1, _ = vox(*ls)
        torch.autograd.backward([d1, f1], [gD[b], gF[b]])
        _close("density", density[b], d1)
        _close("grid_feats", grid_feats[b], f1)
        for k, name in enumerate(["means", "opacity", "cov", "features"]):
            _close(f"grad_{name}[{b}]", leaves[k].grad[b], ls[k].grad, rtol=1e-5)
    # and against the float64 oracle for one scene (boxes from the GPU, as the reference test does)
    m, o, cov, f = (t.detach().cpu().numpy() for t in scenes[1])
    bx = oracle.boxes(m, cov, SIZE, RNG)
    dims = bx.dims
    d_ref, f_ref = oracle.forward(m, o, cov, f, bx.lb, bx.ub, SIZE, RNG, dims)
    assert_close("density[1] vs oracle", density[1].detach().cpu().numpy(), d_ref)
    assert_close("grid_feats[1] vs oracle", grid_feats[1].detach().cpu().numpy(), f_ref)


def test_ragged_scale_rot_batch():
    from CudaGaussianVoxelizer import PyCudaGaussianVoxelizer
    sizes, c = [250, 600], 8
    vox = PyCudaGaussianVoxelizer(voxel_size=SIZE, voxel_range=RNG)
    parts = []
    for b, n in enumerate(sizes):
        m, o, _, f = _scene(n, c, seed=80 + b)
        s, q = (t.cuda() for t in oracle.generate_scale_rot(n, seed=90 + b))
        parts.append((m, o, s, q, f))
    cat = [torch.cat([p[k] for p in parts]).requires_grad_(True) for k in range(5)]
    density, grid_feats, _ = vox(cat[0], cat[1], features=cat[4], scales=cat[2], rotations=cat[3],
                                 scene_sizes=sizes)
    (density.square().sum() + grid_feats.sum()).backward()
    g0 = 0
    for b, n in enumerate(sizes):
        ls = [t.clone().requires_grad_(True) for t in parts[b]]
        d1, f1, _ = vox(ls[0], ls[1], features=ls[4], scales=ls[2], rotations=ls[3])
        (d1.square().sum() + f1.sum()).backward()
        _close("density", density[b], d1)
        _close("grid_feats", grid_feats[b], f1)
        for k, name in enumerate(["means", "opacity", "scales", "rotations", "features"]):
            _close(f"grad_{name}[{b}]", cat[k].grad[g0:g0 + n], ls[k].grad, rtol=1e-5)
        g0 += n


def test_batch_needs_x_multiple_of_four_and_consistent_sizes():
    from CudaGaussianVoxelizer import PyCudaGaussianVoxelizer
    vox = PyCudaGaussianVoxelizer(voxel_size=[0.5] * 3, voxel_range=[-8.0, -8.0, -1.0, 8.5, 8.0, 5.0])  # X = 33
    m, o, cov, f = _scene(20, 4, seed=1)
    with pytest.raises(RuntimeError, match="multiple of 4"):
        vox(m, o, cov, f, scene_sizes=[10, 10])
    with pytest.raises(RuntimeError, match="scene_sizes"):
        vox(m, o, cov, f, scene_sizes=[10, 11])
