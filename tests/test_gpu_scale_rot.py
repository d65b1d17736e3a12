"""GPU parity of the covariance-from-(scale, rotation) front end and the fused voxelizer paths.

* The standalone kernels (g2v_covariance_from_scale_rot[_backward]) against the float64 oracle and the
  golden vectors of the reference's own front end (tests/golden/cov_scale_rot.npz).
* The fused forward (covariances formed in the preparation kernel) against the unfused pipeline fed
  with the standalone kernel's covariances: boxes, counts, CSR and inverse covariances bit-identical.
* The fused backward (chain rule inside the gradient reduction) against the unfused chain
  g2v_backward -> g2v_covariance_from_scale_rot_backward: bit-identical.
* PyCudaGaussianVoxelizer(scales=, rotations=) end to end against the float64 oracle composed with
  the oracle front end, within the parity bar of tests/gpu_util.py.
"""
import numpy as np
import pytest
import torch

from gpu_util import assert_close
from oracle import oracle

pytestmark = pytest.mark.gpu

SIZE, RNG = [0.4] * 3, [-8.0, -8.0, -1.0, 8.0, 8.0, 5.4]


def _inputs(n, c, seed):
    means, opacity, _, feats = oracle.generate_inputs(n, c, RNG, seed=seed)
    s, q = oracle.generate_scale_rot(n, seed=seed + 100)
    return means, opacity, s, q, feats


def test_standalone_kernels_match_golden(golden):
    from CudaGaussianVoxelizer import _C
    g = golden("cov_scale_rot")
    s = torch.from_numpy(g["scales"]).cuda()
    q = torch.from_numpy(g["rotations"]).cuda()
    cov = _C.covariance_from_scale_rot(s, q).cpu().numpy()
    assert_close("cov", cov, g["cov"])
    gs, gq = _C.covariance_from_scale_rot_backward(s, q, torch.from_numpy(g["grad_cov"]).float().cuda())
    assert_close("grad_scales", gs.cpu().numpy(), g["grad_scales"])
    assert_close("grad_rotations", gq.cpu().numpy(), g["grad_rotations"])


def test_autograd_function_and_batched_shapes():
    from CudaGaussianVoxelizer import covariance_from_scale_rot
    s, q = oracle.generate_scale_rot(2 * 50, seed=5)
    s = s.reshape(2, 50, 3).cuda().requires_grad_(True)
    q = q.reshape(2, 50, 4).cuda().requires_grad_(True)
    cov = covariance_from_scale_rot(s, q)
    assert cov.shape == (2, 50, 3, 3)
    G = torch.randn(cov.shape, device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    (cov * G).sum().backward()
    sh, qh, Gh = (t.detach().cpu().numpy() for t in (s, q, G))
    assert_close("cov", cov.detach().cpu().numpy(), oracle.covariance_from_scale_rot(sh, qh))
    gs, gq = oracle.covariance_from_scale_rot_backward(sh, qh, Gh)
    assert_close("grad_scales", s.grad.cpu().numpy(), gs)
    assert_close("grad_rotations", q.grad.cpu().numpy(), gq)


@pytest.mark.parametrize("n,c", [(600, 16), (300, 0), (0, 8)])
def test_fused_forward_is_bit_identical_to_unfused(n, c):
    from CudaGaussianVoxelizer import _C
    means, opacity, s, q, feats = _inputs(max(n, 1), max(c, 1), seed=7)
    means, opacity, s, q = means[:n], opacity[:n], s[:n], q[:n]
    feats = feats[:n, :c].contiguous() if c > 0 else None
    m, o, sc, qq = (t.cuda() for t in (means, opacity, s, q))
    f = feats.cuda() if feats is not None else None
    cov = _C.covariance_from_scale_rot(sc, qq).reshape(n, 9)
    (a, mb_a) = _C._forward_impl(m, o, cov, SIZE, RNG, f, False, plan=True)
    (b, mb_b) = _C._forward_impl(m, o, None, SIZE, RNG, f, False, scale_rot=(sc, qq))
    torch.cuda.synchronize()
    assert mb_a == mb_b
    for name, x, y in zip(["density", "cov_inv", "lb", "ub", "nvox", "grid_feats", "g2t_offsets", "g2t_tile_ids"],
                          a[:8], b[:8]):
        assert torch.equal(x, y), name


def test_fused_backward_is_bit_identical_to_unfused_chain():
    from CudaGaussianVoxelizer import _C
    n, c = 700, 24
    means, opacity, s, q, feats = _inputs(n, c, seed=9)
    m, o, sc, qq, f = (t.cuda() for t in (means, opacity, s, q, feats))
    out, mb = _C._forward_impl(m, o, None, SIZE, RNG, f, False, scale_rot=(sc, qq))
    density, cov_inv, lb, ub, nvox, grid_feats, g2t_off, g2t_ids, _ = out
    gen = torch.Generator("cuda").manual_seed(3)
    gD = torch.randn(density.shape, device="cuda", generator=gen)
    gF = torch.randn(grid_feats.shape, device="cuda", generator=gen)
    args = (gD, gF, m, o, cov_inv, SIZE, RNG, lb, ub, nvox, g2t_off, g2t_ids, density, grid_feats, f)
    gm1, gcov, go1, gf1, _ = _C.gaussian_voxelizer_backward(*args, timing=False, num_block_pairs=mb)
    gs1, gq1 = _C.covariance_from_scale_rot_backward(sc, qq, gcov)
    gm2, (gs2, gq2), go2, gf2, _ = _C.gaussian_voxelizer_backward(*args, timing=False, num_block_pairs=mb,
                                                                  scale_rot=(sc, qq))
    torch.cuda.synchronize()
    for name, x, y in (("means", gm1, gm2), ("opacity", go1, go2), ("features", gf1, gf2), ("scales", gs1, gs2),
                       ("rotations", gq1, gq2)):
        assert torch.equal(x, y), name


def test_module_end_to_end_vs_oracle():
    from CudaGaussianVoxelizer import PyCudaGaussianVoxelizer
    n, c = 400, 12
    means, opacity, s, q, feats = _inputs(n, c, seed=11)
    leaves = [t.cuda().requires_grad_(True) for t in (means, opacity, s, q, feats)]
    vox = PyCudaGaussianVoxelizer(voxel_size=SIZE, voxel_range=RNG)
    density, grid_feats, stats = vox(leaves[0], leaves[1], features=leaves[4], scales=leaves[2],
                                     rotations=leaves[3])
    gen = torch.Generator().manual_seed(4)
    gD = torch.randn(density.shape, generator=gen)
    gF = torch.randn(grid_feats.shape, generator=gen)
    torch.autograd.backward([density, grid_feats], [gD.cuda(), gF.cuda()])
    torch.cuda.synchronize()
    assert stats[0] > 0 and stats[1] > 0
    # float64 oracle on the oracle front end's covariances, with the GPU's boxes (as the reference test)
    cov64 = oracle.covariance_from_scale_rot(s.numpy(), q.numpy()).reshape(n, 9)
    from CudaGaussianVoxelizer import _C
    lbub = _C._forward_impl(*[t.detach() for t in leaves[:2]], None, SIZE, RNG, leaves[4].detach(), False,
                            scale_rot=(leaves[2].detach(), leaves[3].detach()))[0]
    lb, ub = lbub[2].cpu().numpy(), lbub[3].cpu().numpy()
    dims = tuple(int(d) for d in density.shape)
    d_ref, f_ref = oracle.forward(means.numpy(), opacity.numpy(), cov64, feats.numpy(), lb, ub, SIZE, RNG, dims)
    gm, gc, go, gf = oracle.backward(means.numpy(), opacity.numpy(), cov64, feats.numpy(), lb, ub, SIZE, RNG, dims,
                                     gD.numpy(), gF.numpy(), d_ref, f_ref)
    gs, gq = oracle.covariance_from_scale_rot_backward(s.numpy(), q.numpy(), gc.reshape(n, 3, 3))
    assert_close("density", density.detach().cpu().numpy(), d_ref)
    assert_close("grid_feats", grid_feats.detach().cpu().numpy(), f_ref)
    assert_close("grad_means", leaves[0].grad.cpu().numpy(), gm)
    assert_close("grad_opacity", leaves[1].grad.cpu().numpy(), go)
    assert_close("grad_scales", leaves[2].grad.cpu().numpy(), gs)
    assert_close("grad_rotations", leaves[3].grad.cpu().numpy(), gq)
    assert_close("grad_features", leaves[4].grad.cpu().numpy(), gf)


def test_module_argument_errors():
    from CudaGaussianVoxelizer import PyCudaGaussianVoxelizer
    vox = PyCudaGaussianVoxelizer(voxel_size=SIZE, voxel_range=RNG)
    m = torch.zeros(4, 3, device="cuda")
    o = torch.ones(4, device="cuda")
    with pytest.raises(RuntimeError):
        vox(m, o)
    with pytest.raises(RuntimeError):
        vox(m, o, torch.zeros(4, 9, device="cuda"), scales=torch.ones(4, 3, device="cuda"),
            rotations=torch.ones(4, 4, device="cuda"))
    with pytest.raises(RuntimeError):
        vox(m, o, scales=torch.ones(4, 3, device="cuda"), rotations=torch.ones(4, 3, device="cuda"))
