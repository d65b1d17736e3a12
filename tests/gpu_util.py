"""Helpers shared by the GPU parity tests (tolerances, runners over the drop-in API)."""
import numpy as np
import torch

from oracle import oracle

# Tolerances of the parity bar: the reference's own metric (relative L2 < 1e-4, test_reference.py:22)
# and an elementwise bound |a - b| <= ATOL * max(1, max|b|) + RTOL * |b| (abs 1e-5 on unit-scale data).
RTOL = 1e-4
ATOL = 1e-5


def assert_close(name, got, ref, rtol=RTOL, atol=ATOL):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (name, got.shape, ref.shape)
    if ref.size == 0:
        return
    err = oracle.rel_err(got, ref)
    assert err < rtol, f"{name}: relative L2 error {err:.3e} >= {rtol}"
    scale = max(1.0, float(np.abs(ref).max()))
    bad = np.abs(got - ref) > atol * scale + rtol * np.abs(ref)
    assert not bad.any(), (f"{name}: {int(bad.sum())} of {bad.size} elements outside the elementwise bound; "
                           f"max abs diff {float(np.abs(got - ref).max()):.3e} (scale {scale:.3g})")


def margin(got, ref, rtol=RTOL, atol=ATOL):
    """Precision margin against the parity bar: (max elementwise |a - b| / bound, relative L2 / rtol).
    Both must stay below 1 for assert_close to pass; 0.1 means a 10x margin."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    if ref.size == 0:
        return 0.0, 0.0
    scale = max(1.0, float(np.abs(ref).max()))
    elem = float((np.abs(got - ref) / (atol * scale + rtol * np.abs(ref))).max())
    return elem, oracle.rel_err(got, ref) / rtol


def dev(*arrs, requires_grad=False):
    out = []
    for a in arrs:
        if a is None:
            out.append(None)
            continue
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        if requires_grad:
            t.requires_grad_()
        out.append(t)
    return out


def run_fwd_bwd(means, opacity, cov, feats, size, rng, gD, gF, timing=True):
    """Forward + backward through PyCudaGaussianVoxelizer; returns numpy outputs and grads."""
    from CudaGaussianVoxelizer import PyCudaGaussianVoxelizer
    vox = PyCudaGaussianVoxelizer(voxel_size=list(size), voxel_range=list(rng), timing=timing)
    m, o, c = dev(means, opacity, cov, requires_grad=True)
    f = dev(feats, requires_grad=True)[0] if feats is not None else None
    density, grid_feats, stats = vox(m, o, c, f)
    loss = (density * torch.from_numpy(np.ascontiguousarray(gD)).cuda()).sum()
    if f is not None and f.shape[1] > 0:
        loss = loss + (grid_feats * torch.from_numpy(np.ascontiguousarray(gF)).cuda()).sum()
    loss.backward()
    torch.cuda.synchronize()
    res = dict(density=density.detach().cpu().numpy(), grid_feats=grid_feats.detach().cpu().numpy(),
               grad_means=m.grad.cpu().numpy(), grad_opacity=o.grad.cpu().numpy(), grad_cov=c.grad.cpu().numpy(),
               stats=stats.numpy().copy())
    if f is not None:
        res["grad_features"] = f.grad.cpu().numpy() if f.grad is not None else np.zeros(f.shape, np.float32)
    return res
