"""CPU checks of the covariance-from-(scale, rotation) oracle.

oracle.covariance_from_scale_rot / _backward restate the reference's GaussTR front end
(test/gaussian_voxelizer.py:14-37) in float64.  They are pinned to tests/golden/cov_scale_rot.npz, which
tests/golden/make_golden_cov.py made by running the reference's own quat_to_rotmat / get_covariance and
autograd through them; and to properties of the map: invariance under q -> c q (so dL/dq is orthogonal
to q), q and -q give the same rotation, Sigma is symmetric positive definite with eigenvalues s^2.
"""
import numpy as np
import pytest

from oracle import oracle


def test_forward_matches_reference_front_end(golden):
    g = golden("cov_scale_rot")
    cov = oracle.covariance_from_scale_rot(g["scales"], g["rotations"])
    np.testing.assert_allclose(cov, g["cov"], rtol=1e-12, atol=1e-14)


def test_gradients_match_autograd_through_reference(golden):
    g = golden("cov_scale_rot")
    gs, gq = oracle.covariance_from_scale_rot_backward(g["scales"], g["rotations"], g["grad_cov"])
    np.testing.assert_allclose(gs, g["grad_scales"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(gq, g["grad_rotations"], rtol=1e-10, atol=1e-12)


def test_properties():
    s, q = (t.numpy().astype(np.float64) for t in oracle.generate_scale_rot(64, seed=3))
    cov = oracle.covariance_from_scale_rot(s, q)
    np.testing.assert_allclose(cov, np.swapaxes(cov, -1, -2), atol=1e-12)
    eig = np.sort(np.linalg.eigvalsh(cov), axis=-1)
    np.testing.assert_allclose(eig, np.sort(s ** 2, axis=-1), rtol=1e-10)
    np.testing.assert_allclose(oracle.covariance_from_scale_rot(s, -2.5 * q), cov, rtol=1e-12, atol=1e-12)
    G = np.random.default_rng(0).standard_normal(cov.shape)
    _, gq = oracle.covariance_from_scale_rot_backward(s, q, G)
    assert np.abs((gq * q).sum(-1)).max() < 1e-10 * np.abs(gq).max()


@pytest.mark.parametrize("eps", [1e-6])
def test_gradient_finite_difference(eps):
    s, q = (t.numpy().astype(np.float64) for t in oracle.generate_scale_rot(8, seed=4))
    G = np.random.default_rng(1).standard_normal((8, 3, 3))
    gs, gq = oracle.covariance_from_scale_rot_backward(s, q, G)
    f = lambda s_, q_: (oracle.covariance_from_scale_rot(s_, q_) * G).sum()  # noqa: E731
    for k in range(3):
        d = np.zeros_like(s)
        d[:, k] = eps
        num = np.array([(f(s + d, q) - f(s - d, q)) / (2 * eps)])
        assert abs(num - gs[:, k].sum()) < 1e-6 * max(1.0, abs(num))
    for k in range(4):
        d = np.zeros_like(q)
        d[:, k] = eps
        num = (f(s, q + d) - f(s, q - d)) / (2 * eps)
        assert abs(num - gq[:, k].sum()) < 1e-6 * max(1.0, abs(num))
