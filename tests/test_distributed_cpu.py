"""Host logic of the single-scene split (CudaGaussianVoxelizer.distributed) on CPU: the slab partition,
the gradient packing, and -- with two gloo ranks -- that the slab-partial gradients combined by
allreduce_grads equal the whole-grid gradients (per-slab compute by the float64 oracle)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from CudaGaussianVoxelizer import distributed as D
from oracle import oracle


@pytest.mark.parametrize("tiles,world", [(50, 1), (50, 2), (50, 8), (100, 8), (7, 3), (3, 8)])
def test_slab_tiles_partition(tiles, world):
    ranges = [D.slab_tiles(tiles, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == tiles
    for (b0, e0), (b1, e1) in zip(ranges, ranges[1:]):
        assert e0 == b1 and b0 <= e0
    sizes = [e - b for b, e in ranges]
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("tiles,world,seed", [(50, 2, 0), (100, 4, 1), (100, 8, 2), (13, 5, 3), (7, 7, 4)])
def test_balanced_slab_bounds(tiles, world, seed):
    rs = np.random.default_rng(seed)
    work = rs.integers(0, 1000, size=tiles).tolist()
    b = D.balanced_slab_bounds(work, world)
    assert len(b) == world + 1 and b[0] == 0 and b[-1] == tiles
    assert all(e > s for s, e in zip(b, b[1:]))  # every slab keeps a column
    total = sum(work)
    per = [sum(work[s:e]) for s, e in zip(b, b[1:])]
    assert sum(per) == total
    if tiles >= 4 * world:  # room to balance: no slab exceeds its share by more than one column
        assert max(per) <= total / world + max(work)
    # the same counts give the same slabs (every rank computes them on its own)
    assert D.balanced_slab_bounds(list(work), world) == b


def test_balanced_slab_bounds_uniform_and_degenerate():
    for tiles, world in [(50, 2), (100, 8), (12, 3)]:
        b = D.balanced_slab_bounds([5] * tiles, world)  # equal work: slab sizes differ by at most one column
        sizes = [e - s for s, e in zip(b, b[1:])]
        assert max(sizes) - min(sizes) <= 1 and sum(sizes) == tiles
    assert D.balanced_slab_bounds([0] * 10, 3) == [D.slab_tiles(10, r, 3)[0] for r in range(3)] + [10]
    # work piled on one edge column: the other slabs still get a column each
    b = D.balanced_slab_bounds([1000] + [0] * 9, 4)
    assert b[0] == 0 and b[-1] == 10 and all(e > s for s, e in zip(b, b[1:]))
    with pytest.raises(ValueError):
        D.balanced_slab_bounds([1, 2], 3)


@pytest.mark.parametrize("world", [4, 8])
def test_balanced_slabs_even_out_an_edge_thinned_scene(world):
    """The purpose of the balanced split: on a scene whose Gaussians thin out towards its x edges (means
    uniform over the range, so the edge columns see Gaussians from one side only; large variances as in
    the single-scene config), the busiest balanced slab carries no more pairs than the busiest equal-width
    slab, and at most one column more than the mean share."""
    size, rng = [0.4] * 3, [-20.0, -20.0, -1.0, 20.0, 20.0, 5.4]  # 100 x 100 x 16 voxels, 25 tile columns
    m, _, cv, _ = oracle.generate_inputs(3000, 1, rng, seed=9, var_max=8.0)
    bx = oracle.boxes(m.numpy(), cv.numpy(), size, rng)
    tiles_x = (bx.dims[0] + 3) // 4
    cols = _pairs_per_column(bx, tiles_x)
    total = sum(cols)
    eq = [D.slab_tiles(tiles_x, r, world) for r in range(world)]
    b = D.balanced_slab_bounds(cols, world)
    eq_max = max(sum(cols[s:e]) for s, e in eq)
    bal_max = max(sum(cols[s:e]) for s, e in zip(b, b[1:]))
    assert bal_max <= eq_max
    assert bal_max <= total / world + max(cols)


def test_slab_voxel_rows_clip_the_last_tile():
    assert D.slab_voxel_rows(10, (0, 2)) == (0, 8)
    assert D.slab_voxel_rows(10, (2, 3)) == (8, 10)  # the last tile holds 2 voxel rows


def test_pack_unpack_roundtrip():
    g = torch.Generator().manual_seed(3)
    n, c = 17, 5
    parts = (torch.randn(n, 3, generator=g), torch.randn(n, 9, generator=g), torch.randn(n, generator=g),
             torch.randn(n, c, generator=g))
    buf = D.pack_grads(*parts)
    assert buf.shape == (n, 13 + c)
    for a, b in zip(D.unpack_grads(buf, c), parts):
        assert torch.equal(a, b)
    m, cv, o, f = D.unpack_grads(D.pack_grads(parts[0], parts[1], parts[2], None), 0)
    assert f.shape == (n, 0) and torch.equal(o, parts[2])


def _scene():
    size, rng = [0.4] * 3, [-4.0, -4.0, -1.0, 4.0, 4.0, 2.2]
    m, o, cv, f = oracle.generate_inputs(120, 6, rng, seed=5, num_outside=6)
    m, o, cv, f = m.numpy(), o.numpy(), cv.numpy(), f.numpy()
    bx = oracle.boxes(m, cv, size, rng)
    dims = bx.dims
    g = torch.Generator().manual_seed(11)
    gD = torch.randn(*dims, generator=g).numpy()
    gF = torch.randn(*dims, f.shape[1], generator=g).numpy()
    dref, fref = oracle.forward(m, o, cv, f, bx.lb, bx.ub, size, rng, dims)
    return size, rng, m, o, cv, f, bx, dims, gD, gF, dref, fref


def _pairs_per_column(bx, tiles_x):
    """(Gaussian, tile) pairs per tile x column of the oracle's boxes (what tile_pairs_per_column reads
    from the library's boxes on the GPU)."""
    live = (bx.ub >= bx.lb).all(axis=1)
    tlo, thi = bx.lb[live] // 4, bx.ub[live] // 4
    per = (thi[:, 1] - tlo[:, 1] + 1) * (thi[:, 2] - tlo[:, 2] + 1)
    cols = np.zeros(tiles_x + 1, np.int64)
    np.add.at(cols, tlo[:, 0], per)
    np.add.at(cols, thi[:, 0] + 1, -per)
    return np.cumsum(cols)[:tiles_x].tolist()


def _rank_main(rank, world, port, out_path, balanced=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        size, rng, m, o, cv, f, bx, dims, gD, gF, dref, fref = _scene()
        tiles_x = (dims[0] + 3) // 4
        if balanced:  # every rank derives the same bounds from the same boxes
            b = D.balanced_slab_bounds(_pairs_per_column(bx, tiles_x), world)
            tr = (b[rank], b[rank + 1])
        else:
            tr = D.slab_tiles(tiles_x, rank, world)
        xr = D.slab_voxel_rows(dims[0], tr)
        gm, gc, go, gf = oracle.backward(m, o, cv, f, bx.lb, bx.ub, size, rng, dims, gD, gF, dref, fref, x_range=xr)
        tm, tcv, to, tf = D.allreduce_grads(*(torch.from_numpy(np.ascontiguousarray(a)) for a in (gm, gc, go, gf)))
        if rank == 0:
            np.savez(out_path, m=tm.numpy(), c=tcv.numpy(), o=to.numpy(), f=tf.numpy())
    finally:
        torch.distributed.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,balanced", [(2, False), (3, False), (3, True)])
def test_gloo_slab_gradients_sum_to_whole_grid(tmp_path, world, balanced):
    out = str(tmp_path / "grads.npz")
    mp.start_processes(_rank_main, args=(world, _free_port(), out, balanced), nprocs=world, start_method="spawn",
                       join=True)
    size, rng, m, o, cv, f, bx, dims, gD, gF, dref, fref = _scene()
    if balanced:  # the pairs per column sum to the scene's (Gaussian, tile) pairs
        tiles_x = (dims[0] + 3) // 4
        live = (bx.ub >= bx.lb).all(axis=1)
        t = (bx.ub[live] // 4 - bx.lb[live] // 4 + 1).prod(axis=1).sum()
        assert sum(_pairs_per_column(bx, tiles_x)) == t
    rm, rc, ro, rf = oracle.backward(m, o, cv, f, bx.lb, bx.ub, size, rng, dims, gD, gF, dref, fref)
    with np.load(out) as z:
        for key, ref in (("m", rm), ("c", rc), ("o", ro), ("f", rf)):
            np.testing.assert_allclose(z[key], ref, rtol=1e-9, atol=1e-12)
