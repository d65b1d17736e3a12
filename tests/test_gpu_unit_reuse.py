"""The backward's tile pass on the unit lists the forward splat built (g2v_forward_splat_unit_lists +
g2v_backward_units, the default autograd path) gives bit-identical gradients to g2v_backward, which
rebuilds the same lists."""
import numpy as np
import pytest
import torch

from gpu_util import dev
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,c,seed,half,var_max", [(2000, 300, 5, 8.0, 2.5), (3000, 40, 6, 6.0, 8.0)])
def test_backward_on_forward_unit_lists_is_bit_identical(n, c, seed, half, var_max):
    from CudaGaussianVoxelizer import _C
    size, rng = [0.4] * 3, [-half, -half, -1.0, half, half, 5.4]
    m, o, cv, f = oracle.generate_inputs(n, c, rng, seed=seed, num_outside=n // 20, var_max=var_max)
    mt, ot, ct, ft = dev(m.numpy(), o.numpy(), cv.numpy(), f.numpy())
    out, mb, units = _C._forward_impl(mt, ot, ct, size, rng, ft, False, plan=True, keep_units=True)
    assert units is not None
    uoff, ulist = units
    uo = uoff.cpu().numpy()
    assert uo[0] == 0 and np.all(np.diff(uo) >= 0) and uo[-1] <= ulist.numel()
    density, cov_inv, lb, ub, nvox, grid_feats, off, ids, _ = out
    dims = tuple(density.shape)
    g = torch.Generator().manual_seed(seed + 11)
    gD, gF = torch.randn(*dims, generator=g).cuda(), torch.randn(*dims, c, generator=g).cuda()
    args = (gD, gF, mt, ot, cov_inv, size, rng, lb, ub, nvox, off, ids, density, grid_feats, ft)
    ref = _C.gaussian_voxelizer_backward(*args, num_block_pairs=mb)
    got = _C.gaussian_voxelizer_backward(*args, num_block_pairs=mb, units=units)
    torch.cuda.synchronize()
    for name, a, b in zip(("grad_means", "grad_cov", "grad_opacity", "grad_features"), got[:4], ref[:4]):
        np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy(), err_msg=name)
