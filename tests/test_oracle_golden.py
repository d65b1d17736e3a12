"""Pin the CPU oracle against the golden vectors made from the reference's own brute force.

The fixtures come from test/test_reference.py:57-79 of the reference (float64, autograd gradients),
see tests/golden/make_golden.py.  The oracle must reproduce them to float64 rounding.
"""
import numpy as np
import pytest

from oracle import oracle

CASES = ["tiny", "small", "nofeat", "aniso", "cfg1"]
TOL = 1e-10


def _grad_feats(g):
    if "grad_feats" in g:
        return g["grad_feats"]
    import torch
    X, Y, Z = (int(v) for v in g["dims"])
    c = g["features"].shape[1]
    torch.manual_seed(int(g["grad_feats_seed"]))
    torch.randn(X, Y, Z)
    return torch.randn(X, Y, Z, c).numpy()


@pytest.mark.parametrize("name", CASES)
def test_boxes_match_fixture(golden, name):
    g = golden(name)
    bx = oracle.boxes(g["means"], g["cov"], g["voxel_size"], g["voxel_range"])
    assert tuple(bx.dims) == tuple(int(v) for v in g["dims"])
    np.testing.assert_array_equal(bx.lb, g["lb"])
    np.testing.assert_array_equal(bx.ub, g["ub"])
    np.testing.assert_array_equal(bx.num_voxels, g["num_voxels"])
    np.testing.assert_array_equal(bx.g2t_offsets, g["g2t_offsets"])
    np.testing.assert_array_equal(bx.g2t_tile_ids, g["g2t_tile_ids"])


@pytest.mark.parametrize("name", CASES)
def test_forward_matches_reference_bruteforce(golden, name):
    g = golden(name)
    dims = tuple(int(v) for v in g["dims"])
    c = g["features"].shape[1]
    feats = g["features"] if c > 0 else None
    dens, gf = oracle.forward(g["means"], g["opacity"], g["cov"], feats, g["lb"], g["ub"], g["voxel_size"],
                              g["voxel_range"], dims)
    assert oracle.rel_err(dens, g["density"]) < TOL
    np.testing.assert_allclose(dens, g["density"], rtol=1e-12, atol=1e-14)
    if "grid_feats" in g:
        if c > 0:
            assert oracle.rel_err(gf, g["grid_feats"]) < TOL
    else:
        flat = gf.reshape(-1, c)
        np.testing.assert_allclose(flat[g["grid_feats_sample_idx"]], g["grid_feats_sample"], rtol=1e-10, atol=1e-12)
        assert abs(flat.sum() - g["grid_feats_sum"]) < 1e-8 * max(1.0, abs(float(g["grid_feats_sum"])))
        assert abs((flat * flat).sum() - g["grid_feats_sqsum"]) < 1e-9 * float(g["grid_feats_sqsum"])


@pytest.mark.parametrize("name", CASES)
def test_backward_matches_reference_autograd(golden, name):
    g = golden(name)
    dims = tuple(int(v) for v in g["dims"])
    c = g["features"].shape[1]
    feats = g["features"] if c > 0 else None
    dens, gf = oracle.forward(g["means"], g["opacity"], g["cov"], feats, g["lb"], g["ub"], g["voxel_size"],
                              g["voxel_range"], dims)
    gm, gc, go, gfe = oracle.backward(g["means"], g["opacity"], g["cov"], feats, g["lb"], g["ub"],
                                      g["voxel_size"], g["voxel_range"], dims, g["grad_density"], _grad_feats(g),
                                      dens, gf)
    assert oracle.rel_err(gm, g["grad_means"]) < TOL
    assert oracle.rel_err(gc, g["grad_cov"]) < TOL
    assert oracle.rel_err(go, g["grad_opacity"]) < TOL
    if c > 0:
        assert oracle.rel_err(gfe, g["grad_features"]) < TOL
