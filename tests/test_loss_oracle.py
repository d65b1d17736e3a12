"""CPU checks of the feature cosine-loss oracle (oracle.cosine_loss_forward / _backward).

The oracle restates src/cuda_feats_loss.cu in float64.  It is pinned here by
  * closed forms of the reference's own test cases (test/test_feats_loss_backward.py:151-180):
    target = prediction gives loss_v = eps / (|p|^2 + eps) and gradient -s eps p / (|p|^2 + eps)^2,
    target = -prediction gives loss_v = 1 + |p|^2 / (|p|^2 + eps);
  * the PyTorch comparator those tests use (masked rows, fp16, F.normalize(eps=1e-6), mean of
    1 - cos, autograd), within the tests' own tolerances (forward 5e-5 abs / 5e-4 rel, gradient
    1e-3 abs, :151-152 and :145-148);
  * float64 autograd of the forward formula, which must equal the reference's analytic gradient;
  * the edge cases: no valid voxel (loss 0, count 0, zero gradient), zero prediction rows (the
    |p|^2 > eps branch), channel counts that are not multiples of 4.
The same oracle is compared with the reference's CUDA build and with libg2v.so in tests/test_gpu_loss.py.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle

EPS = oracle.LOSS_EPS
DIMS = (12, 10, 8)


def _np(*ts):
    return [t.numpy() for t in ts]


def _valid(label, mask):
    return (mask.reshape(-1).astype(bool)) & (label.reshape(-1) > 0)


@pytest.mark.parametrize("C", [64, 7])
def test_same_target_closed_form(C):
    label, mask, p, g = _np(*oracle.generate_loss_inputs(DIMS, C, "same", seed=1))
    loss, count = oracle.cosine_loss_forward(label, mask, p, g)
    v = _valid(label, mask)
    assert count == int(v.sum()) > 0
    pp = (p.reshape(-1, C)[v].astype(np.float64) ** 2).sum(1)
    assert loss == pytest.approx(float((EPS / (pp + EPS)).mean()), rel=1e-9)
    grad = oracle.cosine_loss_backward(1.0, count, label, mask, p, g).reshape(-1, C)
    want = -(1.0 / count) * EPS * p.reshape(-1, C)[v] / ((pp + EPS) ** 2)[:, None]
    np.testing.assert_allclose(grad[v], want, rtol=1e-6, atol=1e-30)
    assert not grad[~v].any()


def test_negated_target_closed_form():
    label, mask, p, g = _np(*oracle.generate_loss_inputs(DIMS, 64, "neg", seed=2))
    loss, count = oracle.cosine_loss_forward(label, mask, p, g)
    v = _valid(label, mask)
    pp = (p.reshape(-1, 64)[v].astype(np.float64) ** 2).sum(1)
    assert loss == pytest.approx(float((1.0 + pp / (pp + EPS)).mean()), rel=1e-12)


def _reference_test_comparator(label, mask, p, g):
    """The PyTorch loss the reference's tests compare against (feat_loss, test_feats_loss_backward.py:6-27)."""
    pt = torch.from_numpy(p).clone().requires_grad_(True)
    keep = torch.from_numpy(_valid(label, mask))
    C = p.shape[-1]
    pr = pt.reshape(-1, C)[keep].to(torch.float16)
    gr = torch.from_numpy(g).reshape(-1, C)[keep].to(torch.float16)
    cos = (F.normalize(pr, dim=-1, eps=1e-6) * F.normalize(gr, dim=-1, eps=1e-6)).sum(-1)
    loss = torch.mean(1 - cos)
    loss.backward()
    return float(loss.detach()), pt.grad.numpy()


@pytest.mark.parametrize("case", ["same", "neg", "noise"])
def test_matches_reference_test_comparator(case):
    label, mask, p, g = _np(*oracle.generate_loss_inputs((20, 20, 16), 64, case, seed=3))
    loss, count = oracle.cosine_loss_forward(label, mask, p, g)
    grad = oracle.cosine_loss_backward(1.0, count, label, mask, p, g)
    ref_loss, ref_grad = _reference_test_comparator(label, mask, p, g)
    f_diff = abs(loss - ref_loss)
    assert f_diff <= 5e-5 or f_diff <= 5e-4 * abs(ref_loss), (loss, ref_loss)
    assert np.abs(grad - ref_grad).max() <= 1e-3


def test_gradient_is_autograd_of_the_forward():
    label, mask, p, g = _np(*oracle.generate_loss_inputs(DIMS, 20, "noise", noise=0.7, seed=4))
    p = p.copy()
    p.reshape(-1, 20)[:5] = 0.0  # |p|^2 <= eps rows: the clamp's branch
    v = torch.from_numpy(_valid(label, mask))
    pt = torch.from_numpy(p.astype(np.float64)).reshape(-1, 20).requires_grad_(True)
    gt = torch.from_numpy(g.astype(np.float64)).reshape(-1, 20)
    pv, gv = pt[v], gt[v]
    a = torch.sqrt(torch.clamp((pv * pv).sum(1), min=EPS))
    b = torch.sqrt(torch.clamp((gv * gv).sum(1), min=EPS))
    loss = (1 - (pv * gv).sum(1) / (a * b + EPS)).sum() / int(v.sum())
    loss.backward()
    got_loss, count = oracle.cosine_loss_forward(label, mask, p, g)
    assert got_loss == pytest.approx(float(loss.detach()), rel=1e-12)
    grad = oracle.cosine_loss_backward(2.5, count, label, mask, p, g).reshape(-1, 20)
    np.testing.assert_allclose(grad, 2.5 * pt.grad.numpy(), rtol=1e-10, atol=1e-18)


def test_no_valid_voxel():
    label, mask, p, g = _np(*oracle.generate_loss_inputs(DIMS, 16, "noise", seed=5))
    label[:] = 0.0
    assert oracle.cosine_loss_forward(label, mask, p, g) == (0.0, 0)
    assert not oracle.cosine_loss_backward(1.0, 0, label, mask, p, g).any()


def test_terms_bound_the_gradient():
    label, mask, p, g = _np(*oracle.generate_loss_inputs(DIMS, 9, "noise", seed=6))
    _, count = oracle.cosine_loss_forward(label, mask, p, g)
    grad, terms = oracle.cosine_loss_backward(1.0, count, label, mask, p, g, return_terms=True)
    assert (np.abs(grad) <= terms * (1 + 1e-12)).all()


def test_zero_channels_and_empty_grid():
    # C = 0: every valid voxel has loss 1 - 0 / (sqrt(eps) sqrt(eps) + eps) = 1
    label, mask, p, g = _np(*oracle.generate_loss_inputs((6, 5, 4), 0, "noise", seed=8))
    loss, count = oracle.cosine_loss_forward(label, mask, p, g)
    assert count > 0 and loss == 1.0
    assert oracle.cosine_loss_backward(1.0, count, label, mask, p, g).shape == (6, 5, 4, 0)
    label, mask, p, g = _np(*oracle.generate_loss_inputs((0, 4, 4), 8, "noise", seed=7))
    assert oracle.cosine_loss_forward(label, mask, p, g) == (0.0, 0)
    assert oracle.cosine_loss_backward(1.0, 0, label, mask, p, g).shape == (0, 4, 4, 8)
