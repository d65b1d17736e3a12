"""GPU parity of the feature cosine loss (libg2v.so through the drop-in API) with the float64 oracle
and with the reference's own CUDA build (oracle/_ref, src/cuda_feats_loss.cu compiled with its flags).

Tolerances: the valid count is exact; the loss within |d| <= 1e-5 + 1e-4 |loss|; the gradient
elementwise within 1e-4 of the size of its two terms (|g/D| + |c2 p|, scaled), which is where float32
rounding lives when they cancel (target = +-prediction: the exact gradient is O(eps) there), plus
relative L2 < 1e-4 where they do not.
Cases follow the reference's tests (test/test_feats_loss_backward.py:151-180: 200x200x16 voxels, C=64,
target = prediction / its negation / prediction + 0.1 noise) and the edges: channel counts that are
not multiples of 4 or exceed the register-resident rows, unaligned rows, no valid voxel, empty grids,
C = 0, an upstream gradient other than 1, the count as a host int or a device tensor.
"""

import numpy as np
import pytest
import torch

from gpu_util import assert_close
from oracle import build_ref, oracle

pytestmark = pytest.mark.gpu

REF = build_ref.load()
needs_ref = pytest.mark.skipif(REF is None, reason="oracle/_ref has no reference build")

REF_DIMS = (200, 200, 16)


def _cuda(*ts):
    return [t.cuda() for t in ts]


def _host(*ts):
    return [t.detach().cpu().numpy() for t in ts]


def _check_loss(loss, count, inputs):
    want, want_count = oracle.cosine_loss_forward(*inputs)
    assert count == want_count
    assert abs(float(loss) - want) <= 1e-5 + 1e-4 * abs(want), (float(loss), want)


def _check_grad(grad, gout, count, inputs, l2=True):
    want, terms = oracle.cosine_loss_backward(gout, count, *inputs, return_terms=True)
    grad = np.asarray(grad, np.float64)
    assert grad.shape == want.shape
    err = np.abs(grad - want)
    bad = err > 1e-4 * terms
    assert not bad.any(), f"{int(bad.sum())} elements off; max err {err.max():.3e}"
    if l2 and np.abs(want).max() > 0:
        assert_close("grad", grad, want)


def _run(label, mask, p, g, gout=1.0):
    from CudaGaussianVoxelizer import _C
    loss, count, _ = _C.CudaFeatsCosinelossForward(label, mask, p, g)
    grad, _ = _C.CudaFeatsCosinelossBackward(torch.tensor(gout, device="cuda"), label, mask, p, g, count)
    torch.cuda.synchronize()
    return loss, count, grad


@pytest.mark.parametrize("case", ["same", "neg", "noise"])
def test_reference_cases_full_grid(case):
    host = oracle.generate_loss_inputs(REF_DIMS, 64, case, seed=11)
    loss, count, grad = _run(*_cuda(*host))
    inputs = [t.numpy() for t in host]
    _check_loss(loss, count, inputs)
    _check_grad(grad.cpu().numpy(), 1.0, count, inputs, l2=(case == "noise"))


@pytest.mark.parametrize("C", [1, 3, 4, 12, 64, 100, 128, 256, 384, 768, 1030])
def test_channel_counts(C):
    host = oracle.generate_loss_inputs((9, 7, 5), C, "noise", noise=0.5, seed=C)
    loss, count, grad = _run(*_cuda(*host), gout=0.37)
    inputs = [t.numpy() for t in host]
    _check_loss(loss, count, inputs)
    _check_grad(grad.cpu().numpy(), 0.37, count, inputs)


def test_unaligned_rows_use_the_scalar_path():
    label, mask, p, g = oracle.generate_loss_inputs((16, 12, 8), 64, "noise", seed=5)
    n = p.numel()
    bp = torch.empty(n + 1, device="cuda")
    bg = torch.empty(n + 3, device="cuda")
    pu = bp[1:].view(p.shape)
    gu = bg[3:].view(g.shape)
    pu.copy_(p)
    gu.copy_(g)
    assert pu.data_ptr() % 16 and gu.data_ptr() % 16
    loss, count, grad = _run(label.cuda(), mask.cuda(), pu, gu)
    inputs = [t.numpy() for t in (label, mask, p, g)]
    _check_loss(loss, count, inputs)
    _check_grad(grad.cpu().numpy(), 1.0, count, inputs)


def test_no_valid_voxel_gives_zero_loss_and_gradient():
    label, mask, p, g = oracle.generate_loss_inputs((10, 10, 8), 32, "noise", seed=6)
    label.zero_()
    label_c, mask_c, p_c, g_c = _cuda(label, mask, p, g)
    from CudaGaussianVoxelizer import _C
    loss, count, _ = _C.CudaFeatsCosinelossForward(label_c, mask_c, p_c, g_c)
    assert count == 0 and float(loss) == 0.0
    grad, _ = _C.CudaFeatsCosinelossBackward(torch.ones((), device="cuda"), label_c, mask_c, p_c, g_c, 0)
    assert grad.shape == p.shape and not grad.any()


def test_empty_grid_and_zero_channels():
    from CudaGaussianVoxelizer import _C
    label, mask, p, g = _cuda(*oracle.generate_loss_inputs((0, 4, 4), 8, "noise", seed=7))
    loss, count, _ = _C.CudaFeatsCosinelossForward(label, mask, p, g)
    assert count == 0 and float(loss) == 0.0
    grad, _ = _C.CudaFeatsCosinelossBackward(torch.ones((), device="cuda"), label, mask, p, g, count)
    assert grad.shape == (0, 4, 4, 8)
    # C = 0: every valid voxel has loss 1 - 0 / (sqrt(eps) sqrt(eps) + eps) = 1
    host = oracle.generate_loss_inputs((6, 5, 4), 0, "noise", seed=8)
    loss, count, _ = _C.CudaFeatsCosinelossForward(*_cuda(*host))
    want, want_count = oracle.cosine_loss_forward(*[t.numpy() for t in host])
    assert count == want_count > 0 and want == 1.0 and float(loss) == 1.0


def test_zero_prediction_rows_take_the_clamped_branch():
    label, mask, p, g = oracle.generate_loss_inputs((8, 8, 8), 48, "noise", seed=9)
    p.view(-1, 48)[::3] = 0.0
    label.fill_(1.0)
    mask.fill_(True)
    loss, count, grad = _run(*_cuda(label, mask, p, g))
    inputs = [t.numpy() for t in (label, mask, p, g)]
    _check_loss(loss, count, inputs)
    _check_grad(grad.cpu().numpy(), 1.0, count, inputs)


def test_count_as_int_or_device_tensor_is_bit_identical():
    from CudaGaussianVoxelizer import _C
    label, mask, p, g = _cuda(*oracle.generate_loss_inputs((20, 20, 8), 64, "noise", seed=10))
    gout = torch.tensor(1.7, device="cuda")
    loss, count, _ = _C.CudaFeatsCosinelossForward(label, mask, p, g)
    loss2, count_dev, _ = _C._cosine_loss_forward_impl(label, mask, p, g, False)
    assert torch.equal(loss, loss2) and int(count_dev.item()) == count  # deterministic sum
    g1, _ = _C.CudaFeatsCosinelossBackward(gout, label, mask, p, g, count)
    g2, _ = _C.CudaFeatsCosinelossBackward(gout, label, mask, p, g, count_dev)
    g3, _ = _C.CudaFeatsCosinelossBackward(1.7, label, mask, p, g, count)
    assert torch.equal(g1, g2) and torch.equal(g1, g3)


@pytest.mark.parametrize("timing", [True, False])
def test_module_autograd_like_reference_test(timing):
    """The reference test's flow (test_feats_loss_backward.py:89-111): module call -> (loss, stats) -> backward."""
    from CudaGaussianVoxelizer import PyCudaFeatsCosineLoss
    label, mask, p, g = oracle.generate_loss_inputs(REF_DIMS, 64, "noise", seed=12)
    crit = PyCudaFeatsCosineLoss(voxel_size=[0.4] * 3, voxel_range=[-40, -40, -1, 40, 40, 5.4], timing=timing)
    pc = p.cuda().requires_grad_(True)
    loss, stats = crit(label.cuda(), mask.cuda(), pc, g.cuda())
    assert loss.dim() == 0 and loss.dtype == torch.float32 and stats.shape == (2,)
    (3.0 * loss).backward()
    torch.cuda.synchronize()
    inputs = [t.numpy() for t in (label, mask, p, g)]
    want, count = oracle.cosine_loss_forward(*inputs)
    assert abs(float(loss) - want) <= 1e-5 + 1e-4 * abs(want)
    _check_grad(pc.grad.cpu().numpy(), 3.0, count, inputs)
    if timing:
        assert stats[0] > 0 and stats[1] > 0
    else:
        assert stats[0] == 0 and stats[1] == 0


@needs_ref
@pytest.mark.parametrize("case,C", [("same", 64), ("neg", 64), ("noise", 64), ("noise", 100), ("noise", 384)])
def test_matches_reference_build(case, C):
    dims = REF_DIMS if C == 64 else (40, 40, 16)
    host = oracle.generate_loss_inputs(dims, C, case, seed=13)
    label, mask, p, g = _cuda(*host)
    loss, count, grad = _run(label, mask, p, g, gout=1.0)
    r_loss, r_count, _ = REF.CudaFeatsCosinelossForward(label, mask, p, g)
    r_grad, _ = REF.CudaFeatsCosinelossBackward(torch.ones((), device="cuda"), label, mask, p, g, r_count)
    torch.cuda.synchronize()
    assert count == r_count
    assert abs(float(loss) - float(r_loss)) <= 1e-5 + 1e-4 * abs(float(r_loss))
    inputs = [t.numpy() for t in host]
    _, terms = oracle.cosine_loss_backward(1.0, count, *inputs, return_terms=True)
    err = np.abs(grad.cpu().numpy().astype(np.float64) - r_grad.cpu().numpy())
    assert (err <= 1e-4 * terms).all(), float(err.max())
    # and the reference build itself sits inside the same bound around the oracle
    _check_loss(r_loss, r_count, inputs)
    _check_grad(r_grad.cpu().numpy(), 1.0, r_count, inputs, l2=(case == "noise"))
