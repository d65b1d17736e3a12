"""GPU parity of libg2v.so against the oracle and the golden vectors of the reference's brute force.

Bar: CSR maps bit-exact; density, grid_feats and every gradient within relative L2 1e-4 (the
reference's RTOL, test/test_reference.py:22) and the elementwise bound of tests/gpu_util.py.
The float64 values, like the reference's test, are computed with the boxes the GPU returned
(test/test_reference.py:48-54); the boxes themselves are compared with the oracle separately.
"""
import numpy as np
import pytest
import torch

from gpu_util import assert_close, dev, margin, run_fwd_bwd
from oracle import oracle

pytestmark = pytest.mark.gpu

CASES = ["tiny", "small", "nofeat", "aniso", "cfg1"]


def _gf_upstream(g):
    if "grad_feats" in g:
        return g["grad_feats"]
    X, Y, Z = (int(v) for v in g["dims"])
    c = g["features"].shape[1]
    torch.manual_seed(int(g["grad_feats_seed"]))
    torch.randn(X, Y, Z)
    return torch.randn(X, Y, Z, c).numpy()


def _maps(means, opacity, cov, feats, size, rng):
    from CudaGaussianVoxelizer import _C
    m, o, c, f = dev(means, opacity, cov, feats)
    out, (toff, t2g) = _C.t2g_maps(m, o, c, size, rng, f)
    torch.cuda.synchronize()
    return [t.cpu().numpy() if isinstance(t, torch.Tensor) else t for t in out], toff.cpu().numpy(), t2g.cpu().numpy()


@pytest.mark.parametrize("name", CASES)
def test_csr_bit_exact_vs_oracle(golden, name):
    g = golden(name)
    feats = g["features"] if g["features"].shape[1] > 0 else None
    out, toff, t2g = _maps(g["means"], g["opacity"], g["cov"], feats, g["voxel_size"], g["voxel_range"])
    density, cov_inv, lb, ub, nvox, gf, off, ids, _ = out
    np.testing.assert_array_equal(lb, g["lb"])
    np.testing.assert_array_equal(ub, g["ub"])
    np.testing.assert_array_equal(nvox, g["num_voxels"])
    np.testing.assert_array_equal(off.astype(np.int64), g["g2t_offsets"])
    np.testing.assert_array_equal(ids, g["g2t_tile_ids"])
    _, _, otoff, ot2g = oracle.csr_from_boxes(lb, ub, tuple(int(v) for v in g["dims"]))
    np.testing.assert_array_equal(toff.astype(np.int64), otoff)
    np.testing.assert_array_equal(t2g, ot2g)
    bx = oracle.boxes(g["means"], g["cov"], g["voxel_size"], g["voxel_range"])
    np.testing.assert_allclose(cov_inv, bx.cov_inv, rtol=2e-5, atol=1e-6)


@pytest.mark.parametrize("n", [40000, 100000])
def test_csr_bit_exact_both_scan_paths(n):
    """g2t offsets of 40k Gaussians come from the one-block scan (5 chunks of 8192), of 100k from the
    three-kernel scan; both bit-exact against the oracle's CSR of the same boxes."""
    rng = [-20.0, -20.0, -1.0, 20.0, 20.0, 5.4]
    m, o, cv, _ = oracle.generate_inputs(n, 0, rng, seed=5, num_outside=n // 20)
    out, toff, t2g = _maps(m.numpy(), o.numpy(), cv.numpy(), None, [0.4] * 3, rng)
    density, cov_inv, lb, ub, nvox, gf, off, ids, _ = out
    dims = tuple(int(v) for v in density.shape)
    goff, gids, otoff, ot2g = oracle.csr_from_boxes(lb, ub, dims)
    np.testing.assert_array_equal(off.astype(np.int64), goff)
    np.testing.assert_array_equal(ids, gids)
    np.testing.assert_array_equal(toff.astype(np.int64), otoff)
    np.testing.assert_array_equal(t2g, ot2g)


@pytest.mark.parametrize("name", CASES)
def test_forward_backward_vs_reference_golden(golden, name):
    g = golden(name)
    c = g["features"].shape[1]
    feats = g["features"] if c > 0 else None
    gF = _gf_upstream(g) if c > 0 else None
    r = run_fwd_bwd(g["means"], g["opacity"], g["cov"], feats, g["voxel_size"], g["voxel_range"], g["grad_density"],
                    gF)
    assert_close("density", r["density"], g["density"])
    if c > 0:
        if "grid_feats" in g:
            assert_close("grid_feats", r["grid_feats"], g["grid_feats"])
        else:
            flat = r["grid_feats"].reshape(-1, c)
            assert_close("grid_feats(sample)", flat[g["grid_feats_sample_idx"]], g["grid_feats_sample"])
            assert abs(flat.astype(np.float64).sum() - g["grid_feats_sum"]) < 1e-4 * np.sqrt(g["grid_feats_sqsum"])
    assert_close("grad_means", r["grad_means"], g["grad_means"])
    assert_close("grad_opacity", r["grad_opacity"], g["grad_opacity"])
    assert_close("grad_cov", r["grad_cov"], g["grad_cov"])
    if c > 0:
        assert_close("grad_features", r["grad_features"], g["grad_features"])
    assert r["stats"][0] > 0 and r["stats"][1] > 0


def _random_case(n, c, size, rng, seed, n_out=0, var_max=2.5, expand=0.0):
    m, o, cv, f = oracle.generate_inputs(n, c, rng, num_outside=n_out, seed=seed, var_max=var_max, expand=expand)
    return m.numpy(), o.numpy(), cv.numpy(), (f.numpy() if f is not None else None)


def _slab_upstream(dims, c, x_rows, seed):
    """randn upstream gradients on the voxel rows x_rows, zeros elsewhere (the slab backward reads only its
    own rows, so the rest need not be drawn)."""
    X, Y, Z = dims
    x0, x1 = x_rows
    g = torch.Generator().manual_seed(seed + 7)
    gD = np.zeros((X, Y, Z), np.float32)
    gD[x0:x1] = torch.randn(x1 - x0, Y, Z, generator=g).numpy()
    gF = None
    if c > 0:
        gF = np.zeros((X, Y, Z, c), np.float32)
        gF[x0:x1] = torch.randn(x1 - x0, Y, Z, c, generator=g).numpy()
    return gD, gF


def _oracle_check(means, opacity, cov, feats, size, rng, seed, x_tiles=None, check_boxes=True, slab_upstream=False,
                  margins=None):
    """Full forward+backward on the GPU vs the float64 oracle (given the GPU's boxes).  `margins` (a dict)
    receives each output's precision margin (gpu_util.margin)."""
    from CudaGaussianVoxelizer import _C
    dims, tiles = oracle.grid_shape(size, rng)
    X, Y, Z = dims
    c = 0 if feats is None else feats.shape[1]
    if slab_upstream:
        gD, gF = _slab_upstream(dims, c, (x_tiles[0] * 4, min(x_tiles[1] * 4, X)), seed)
    else:
        g = torch.Generator().manual_seed(seed + 7)
        gD = torch.randn(X, Y, Z, generator=g).numpy()
        gF = torch.randn(X, Y, Z, c, generator=g).numpy() if c > 0 else None
    mt, ot, ct, ft = dev(means, opacity, cov, feats)
    out = _C.gaussian_voxelizer_forward(mt, ot, ct, list(size), list(rng), ft)
    density, cov_inv, lb, ub, nvox, grid_feats, off, ids, _ = out
    lb_h, ub_h = lb.cpu().numpy(), ub.cpu().numpy()
    if check_boxes:
        bx = oracle.boxes(means, cov, size, rng)
        flips = int((bx.lb != lb_h).any(axis=1).sum() + (bx.ub != ub_h).any(axis=1).sum())
        # fast-math sqrt/division flips at exact voxel boundaries are allowed only very rarely
        assert flips <= max(1, means.shape[0] // 5000), f"{flips} boxes differ from the IEEE restatement"
    xr = None
    tr = None
    if x_tiles is not None:
        tr = x_tiles
        xr = (x_tiles[0] * 4, min(x_tiles[1] * 4, X))
    dref, fref = oracle.forward(means, opacity, cov, feats, lb_h, ub_h, size, rng, dims, x_range=xr)
    sl = slice(None) if xr is None else slice(xr[0], xr[1])
    checks = [("density", density[sl].cpu().numpy(), dref[sl])]
    if c > 0:
        checks.append(("grid_feats", grid_feats[sl].cpu().numpy(), fref[sl]))
    for name, a, b in checks:
        if margins is not None:
            margins[name] = margin(a, b)
        assert_close(name, a, b)
    gDt = torch.from_numpy(gD).cuda()
    gFt = torch.from_numpy(gF).cuda() if c > 0 else torch.empty(0, device="cuda")
    gm, gc, go, gfe, _ = _C.gaussian_voxelizer_backward(gDt, gFt, mt, ot, cov_inv, list(size), list(rng), lb, ub,
                                                        nvox, off, ids, density, grid_feats, ft, tile_x_range=tr)
    rm, rc, ro, rf = oracle.backward(means, opacity, cov, feats, lb_h, ub_h, size, rng, dims, gD, gF, dref, fref,
                                     x_range=xr)
    checks = [("grad_means", gm.cpu().numpy(), rm), ("grad_cov", gc.cpu().numpy(), rc),
              ("grad_opacity", go.cpu().numpy(), ro)]
    if c > 0:
        checks.append(("grad_features", gfe.cpu().numpy(), rf))
    for name, a, b in checks:
        if margins is not None:
            margins[name] = margin(a, b)
        assert_close(name, a, b)
    return out


def _print_margins(label, margins):
    print(f"\nprecision margin {label} (max |err| / elementwise bound, rel L2 / 1e-4):")
    for k, (e, r) in margins.items():
        print(f"  {k:14s} {e:.3e}  {r:.3e}")


def test_reference_backward_case():
    """test/test_reference.py:103-124: 500 Gaussians + 50 beyond x_max, 40-D, 200x200x16 grid."""
    size, rng = [0.4] * 3, [-40.0, -40.0, -1.0, 40.0, 40.0, 5.4]
    args = _random_case(500, 40, size, rng, seed=1, n_out=50)
    _oracle_check(*args, size, rng, seed=1)


@pytest.mark.parametrize("c", [1, 5, 37, 300])
def test_odd_channel_counts(c):
    size, rng = [0.4] * 3, [-6.0, -6.0, -1.0, 6.0, 6.0, 3.0]
    args = _random_case(200, c, size, rng, seed=c, n_out=10)
    _oracle_check(*args, size, rng, seed=c)


def test_density_only_path():
    size, rng = [0.4] * 3, [-8.0, -8.0, -1.0, 8.0, 8.0, 5.4]
    m, o, cv, _ = _random_case(512, 4, size, rng, seed=11)
    _oracle_check(m, o, cv, None, size, rng, seed=11)


def test_anisotropic_large_gaussians():
    """Large anisotropic Gaussians (cfg5-like variance), long tile lists (bitmap sort path)."""
    size, rng = [0.2] * 3, [-6.0, -6.0, -1.0, 6.0, 6.0, 2.2]
    args = _random_case(3000, 16, size, rng, seed=5, var_max=8.0)
    _oracle_check(*args, size, rng, seed=5)


def test_cfg3_shape_slab_against_oracle():
    """Headline shape (N=18000, C=1024, 200x200x16): forward + backward checked on an x-slab of tiles
    against the oracle restricted to the same voxels (size-independent property: the slab's values)."""
    size, rng = [0.4] * 3, [-40.0, -40.0, -1.0, 40.0, 40.0, 5.4]
    args = _random_case(18000, 1024, size, rng, seed=0)
    margins = {}
    _oracle_check(*args, size, rng, seed=0, x_tiles=(10, 12), margins=margins)
    _print_margins("cfg3 slab", margins)


def test_cfg5_shape_slab_against_oracle():
    """Single-scene config (N=100000, C=256, 0.2 m voxels -> 400x400x32, covariance eigenvalues U(0.5, 8)):
    ~2400 Gaussians per tile, so nearly every unit runs several slot passes and its e_v from grid_feats.
    Forward + backward on a 2-tile x-slab against the oracle restricted to the same voxels."""
    size, rng = [0.2] * 3, [-40.0, -40.0, -1.0, 40.0, 40.0, 5.4]
    args = _random_case(100000, 256, size, rng, seed=0, var_max=8.0)
    margins = {}
    _oracle_check(*args, size, rng, seed=0, x_tiles=(50, 52), slab_upstream=True, margins=margins)
    _print_margins("cfg5 slab", margins)


def test_features_with_zero_channels_zero_density():
    """features (N,0): the reference's density sum sits inside its channel loop, so density stays 0."""
    from CudaGaussianVoxelizer import _C
    size, rng = [0.4] * 3, [-4.0, -4.0, -1.0, 4.0, 4.0, 2.2]
    m, o, cv, _ = _random_case(50, 1, size, rng, seed=3)
    mt, ot, ct = dev(m, o, cv)
    out = _C.gaussian_voxelizer_forward(mt, ot, ct, size, rng, torch.zeros(50, 0, device="cuda"))
    assert out[0].abs().max().item() == 0.0
    assert tuple(out[5].shape) == (20, 20, 8, 0)
    out2 = _C.gaussian_voxelizer_forward(mt, ot, ct, size, rng, None)
    assert out2[0].abs().max().item() > 0.0


def test_empty_and_outside_inputs():
    from CudaGaussianVoxelizer import PyCudaGaussianVoxelizer
    size, rng = [0.4] * 3, [-4.0, -4.0, -1.0, 4.0, 4.0, 2.2]
    vox = PyCudaGaussianVoxelizer(size, rng)
    # no Gaussians
    m = torch.zeros(0, 3, device="cuda", requires_grad=True)
    o = torch.zeros(0, device="cuda", requires_grad=True)
    c = torch.zeros(0, 9, device="cuda", requires_grad=True)
    f = torch.zeros(0, 8, device="cuda", requires_grad=True)
    d, gf, st = vox(m, o, c, f)
    assert d.shape == (20, 20, 8) and gf.shape == (20, 20, 8, 8)
    assert d.abs().sum().item() == 0 and gf.abs().sum().item() == 0
    (d.sum() + gf.sum()).backward()
    assert m.grad.shape == (0, 3) and f.grad.shape == (0, 8)
    # all Gaussians far outside the range: empty boxes, zero outputs, zero gradients
    mm = torch.full((30, 3), 100.0, device="cuda") + torch.rand(30, 3, device="cuda")
    mm.requires_grad_()
    oo = torch.rand(30, device="cuda", requires_grad=True)
    cc = torch.eye(3, device="cuda").reshape(1, 9).repeat(30, 1).requires_grad_()
    ff = torch.randn(30, 8, device="cuda", requires_grad=True)
    d, gf, st = vox(mm, oo, cc, ff)
    assert d.abs().sum().item() == 0 and gf.abs().sum().item() == 0
    (d.sum() + gf.sum()).backward()
    for t in (mm, oo, cc, ff):
        assert t.grad.abs().sum().item() == 0


def test_determinism():
    size, rng = [0.4] * 3, [-10.0, -10.0, -1.0, 10.0, 10.0, 5.4]
    m, o, cv, f = _random_case(2000, 64, size, rng, seed=21)
    X, Y, Z = oracle.grid_shape(size, rng)[0]
    g = torch.Generator().manual_seed(4)
    gD = torch.randn(X, Y, Z, generator=g).numpy()
    gF = torch.randn(X, Y, Z, 64, generator=g).numpy()
    a = run_fwd_bwd(m, o, cv, f, size, rng, gD, gF)
    b = run_fwd_bwd(m, o, cv, f, size, rng, gD, gF)
    for k in ("density", "grid_feats", "grad_means", "grad_cov", "grad_opacity", "grad_features"):
        np.testing.assert_array_equal(a[k], b[k], err_msg=k)


def test_slab_decomposition_matches_full_grid():
    """x-slabs of tiles (the sharded path): slab forwards tile the full forward bit for bit and the
    slab backward partials sum to the full gradient."""
    from CudaGaussianVoxelizer import _C, _lib
    import ctypes
    size, rng = [0.4] * 3, [-10.0, -10.0, -1.0, 10.0, 10.0, 5.4]
    m, o, cv, f = _random_case(1500, 32, size, rng, seed=8)
    mt, ot, ct, ft = dev(m, o, cv, f)
    full = _C.gaussian_voxelizer_forward(mt, ot, ct, size, rng, ft)
    density, cov_inv, lb, ub, nvox, grid_feats, off, ids, _ = full
    (X, Y, Z), (TX, TY, TZ) = oracle.grid_shape(size, rng)
    lib = _lib.load()
    cuts = [0, 4, 5, 9, TX]
    d2 = torch.full_like(density, -1.0)
    f2 = torch.full_like(grid_feats, -1.0)
    ids2 = torch.empty_like(ids)
    nb = ctypes.c_size_t()
    lib.g2v_forward_splat_workspace_size(1500, ids.numel(), _lib.i3((X, Y, Z)), 32, ctypes.byref(nb))
    ws = torch.empty(nb.value, dtype=torch.uint8, device="cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    for a, b in zip(cuts[:-1], cuts[1:]):
        _lib.check(lib.g2v_forward_splat(P(mt), P(ot), P(ft), 1500, 32, _lib.f3(size), _lib.f6(rng), P(cov_inv), P(lb),
                                         P(ub), P(off), ids.numel(), P(ids2), P(d2), P(f2), a, b, P(ws), ws.numel(), s),
                   "splat")
    torch.cuda.synchronize()
    assert torch.equal(d2, density) and torch.equal(f2, grid_feats) and torch.equal(ids2, ids)
    gD = torch.randn(X, Y, Z, device="cuda")
    gF = torch.randn(X, Y, Z, 32, device="cuda")
    ref = _C.gaussian_voxelizer_backward(gD, gF, mt, ot, cov_inv, size, rng, lb, ub, nvox, off, ids, density,
                                         grid_feats, ft)
    acc = None
    for a, b in zip(cuts[:-1], cuts[1:]):
        part = _C.gaussian_voxelizer_backward(gD, gF, mt, ot, cov_inv, size, rng, lb, ub, nvox, off, ids, density,
                                              grid_feats, ft, tile_x_range=(a, b))
        acc = list(part[:4]) if acc is None else [x + y for x, y in zip(acc, part[:4])]
    for name, x, y in zip(("means", "cov", "opacity", "features"), acc, ref[:4]):
        assert_close(f"slab-sum grad_{name}", x.cpu().numpy(), y.cpu().numpy(), rtol=1e-5)


def test_noncontiguous_and_errors():
    from CudaGaussianVoxelizer import _C
    size, rng = [0.4] * 3, [-4.0, -4.0, -1.0, 4.0, 4.0, 2.2]
    m, o, cv, f = _random_case(64, 8, size, rng, seed=2)
    mt, ot, ct, ft = dev(m, o, cv, f)
    ref = _C.gaussian_voxelizer_forward(mt, ot, ct, size, rng, ft)
    wide = torch.zeros(64, 6, device="cuda")
    wide[:, ::2] = mt
    alt = _C.gaussian_voxelizer_forward(wide[:, ::2], ot, ct, size, rng, ft)
    assert torch.equal(alt[0], ref[0]) and torch.equal(alt[5], ref[5])
    with pytest.raises(RuntimeError):
        _C.gaussian_voxelizer_forward(mt, ot.double(), ct, size, rng, ft)
    with pytest.raises(RuntimeError):
        _C.gaussian_voxelizer_forward(mt, ot, ct[:, :8], size, rng, ft)
    with pytest.raises(RuntimeError):  # backward insists on contiguous inputs like the reference
        _C.gaussian_voxelizer_backward(torch.zeros(20, 20, 8, device="cuda").transpose(0, 1), None, mt, ot, ref[1], size, rng,
                                       ref[2], ref[3], ref[4], ref[6], ref[7], ref[0], ref[5], None)
