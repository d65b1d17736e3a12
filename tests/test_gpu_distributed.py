"""Single-scene split on the GPU: slab-local forward/backward (g2v_forward_splat_local, g2v_backward_local)
against the whole-grid call, and the SlabGaussianVoxelizer module (one rank here; two NCCL ranks when two
GPUs are visible)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from gpu_util import assert_close, dev
from oracle import oracle

pytestmark = pytest.mark.gpu


def _scene(n=3000, c=96, half=10.0, seed=21, var_max=2.5):
    size, rng = [0.4] * 3, [-half, -half, -1.0, half, half, 5.4]
    m, o, cv, f = oracle.generate_inputs(n, c, rng, seed=seed, num_outside=n // 20, var_max=var_max)
    return size, rng, m.numpy(), o.numpy(), cv.numpy(), f.numpy()


@pytest.mark.parametrize("world,c,balanced", [(2, 96, False), (3, 96, False), (4, 37, False), (3, 0, False),
                                              (3, 96, True), (5, 37, True)])
def test_slab_local_matches_whole_grid(world, c, balanced):
    from CudaGaussianVoxelizer import _C
    from CudaGaussianVoxelizer import distributed as D
    size, rng, m, o, cv, f = _scene(c=max(c, 1))
    feats = f[:, :c] if c > 0 else None
    mt, ot, ct = dev(m, o, cv)
    ft = dev(np.ascontiguousarray(feats))[0] if feats is not None else None
    st, rt = torch.tensor(size, device="cuda"), torch.tensor(rng, device="cuda")
    full = _C.gaussian_voxelizer_forward(mt, ot, ct, st, rt, ft, timing=False)
    density, cov_inv, lb, ub, nvox, grid_feats, off, ids, _ = full
    X, Y, Z = density.shape
    g = torch.Generator(device="cuda").manual_seed(5)
    gD = torch.randn((X, Y, Z), device="cuda", generator=g)
    gF = torch.randn((X, Y, Z, c), device="cuda", generator=g)
    ref = _C.gaussian_voxelizer_backward(gD, gF if c > 0 else torch.empty(0, device="cuda"), mt, ot, cov_inv, st, rt,
                                         lb, ub, nvox, off, ids, density, grid_feats, ft, timing=False)
    tiles_x = (X + 3) // 4
    if balanced:  # slabs split by the (Gaussian, tile) pairs per tile column
        cols = D.tile_pairs_per_column(mt, ct, st, rt)
        assert len(cols) == tiles_x and sum(cols) == int(off[-1])
        bounds = D.balanced_slab_bounds(cols, world)
    sums = None
    for r in range(world):
        tr = (bounds[r], bounds[r + 1]) if balanced else D.slab_tiles(tiles_x, r, world)
        x0, x1 = D.slab_voxel_rows(X, tr)
        d_s, f_s, state = D.slab_forward(mt, ot, ct, st, rt, ft, tr)
        torch.cuda.synchronize()
        # the slab's rows are the whole-grid call's rows, bit for bit
        assert torch.equal(d_s, density[x0:x1])
        if c > 0:
            assert torch.equal(f_s, grid_feats[x0:x1])
        assert torch.equal(state[5], ids) and torch.equal(state[4], off)
        part = D.slab_backward(gD[x0:x1].contiguous(), gF[x0:x1].contiguous() if c > 0 else None, mt, ot, ft, st, rt,
                               d_s, f_s, state, tr)
        sums = [p.clone() for p in part] if sums is None else [a + b for a, b in zip(sums, part)]
    torch.cuda.synchronize()
    for name, a, b in zip(("grad_means", "grad_cov", "grad_opacity", "grad_features"), sums, ref[:4]):
        assert_close(name, a.cpu().numpy(), b.cpu().numpy(), rtol=1e-5)


def test_slab_module_single_rank_matches_reference_api():
    from CudaGaussianVoxelizer import PyCudaGaussianVoxelizer
    from CudaGaussianVoxelizer.distributed import SlabGaussianVoxelizer
    size, rng, m, o, cv, f = _scene(n=1500, c=48, half=8.0, seed=4)
    ins = dev(m, o, cv, f, requires_grad=True)
    ins2 = dev(m, o, cv, f, requires_grad=True)
    d1, f1, _ = PyCudaGaussianVoxelizer(size, rng, timing=False)(*ins)
    d2, f2, rows = SlabGaussianVoxelizer(size, rng)(*ins2)
    assert rows == (0, d1.shape[0])
    assert torch.equal(d1, d2) and torch.equal(f1, f2)
    g = torch.Generator(device="cuda").manual_seed(1)
    gD, gF = torch.randn(d1.shape, device="cuda", generator=g), torch.randn(f1.shape, device="cuda", generator=g)
    a = torch.autograd.grad([d1, f1], ins, [gD, gF])
    b = torch.autograd.grad([d2, f2], ins2, [gD, gF])
    for x, y in zip(a, b):
        assert_close("grad", x.cpu().numpy(), y.cpu().numpy(), rtol=1e-6)


def test_slab_module_tile_bounds():
    from CudaGaussianVoxelizer import distributed as D
    size, rng = [0.4] * 3, [-10.0, -10.0, -1.0, 10.0, 10.0, 5.4]  # 50 x 50 x 16 voxels, 13 tile columns
    bounds = [0, 2, 9, 13]
    for r in range(3):
        vox = D.SlabGaussianVoxelizer(size, rng, rank=r, world=3, tile_bounds=bounds)
        assert vox.tile_range == (bounds[r], bounds[r + 1])
        assert vox.rows == D.slab_voxel_rows(50, vox.tile_range)
    for bad in ([0, 2, 9], [0, 9, 2, 13], [1, 2, 9, 13], [0, 2, 9, 12], [0, 2, 2, 13]):
        with pytest.raises(ValueError):
            D.SlabGaussianVoxelizer(size, rng, rank=0, world=3, tile_bounds=bad)


def _nccl_rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world,
                                         device_id=torch.device("cuda", rank))
    try:
        from CudaGaussianVoxelizer.distributed import SlabGaussianVoxelizer
        size, rng, m, o, cv, f = _scene(n=2500, c=64, half=10.0, seed=8)
        ins = [torch.from_numpy(a).cuda().requires_grad_() for a in (m, o, cv, f)]
        d, fe, (x0, x1) = SlabGaussianVoxelizer(size, rng)(*ins)
        X = int(round((rng[3] - rng[0]) / size[0]))
        g = torch.Generator(device="cuda").manual_seed(2)
        gD = torch.randn((X,) + tuple(d.shape[1:]), device="cuda", generator=g)
        gF = torch.randn((X,) + tuple(fe.shape[1:]), device="cuda", generator=g)
        grads = torch.autograd.grad([d, fe], ins, [gD[x0:x1], gF[x0:x1]])
        torch.cuda.synchronize()
        if rank == 0:
            np.savez(out, *[t.cpu().numpy() for t in grads])
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_slab_module_two_nccl_ranks(tmp_path):
    from CudaGaussianVoxelizer import PyCudaGaussianVoxelizer
    out = str(tmp_path / "g.npz")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_nccl_rank, args=(2, port, out), nprocs=2, start_method="spawn", join=True)
    size, rng, m, o, cv, f = _scene(n=2500, c=64, half=10.0, seed=8)
    ins = dev(m, o, cv, f, requires_grad=True)
    d, fe, _ = PyCudaGaussianVoxelizer(size, rng, timing=False)(*ins)
    g = torch.Generator(device="cuda").manual_seed(2)
    gD = torch.randn(d.shape, device="cuda", generator=g)
    gF = torch.randn(fe.shape, device="cuda", generator=g)
    ref = torch.autograd.grad([d, fe], ins, [gD, gF])
    with np.load(out) as z:
        for i, r in enumerate(ref):
            assert_close(f"grad {i}", z[f"arr_{i}"], r.cpu().numpy(), rtol=1e-5)
