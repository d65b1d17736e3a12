"""Both splat variants (tcgen05 split-f16 and FP32-FMA) against the oracle and against each other."""
import os

import numpy as np
import pytest
import torch

from gpu_util import assert_close, dev
from oracle import oracle

pytestmark = pytest.mark.gpu


def _forward(variant, means, opacity, cov, feats, size, rng):
    from CudaGaussianVoxelizer import _C
    old = os.environ.get("G2V_VARIANT")
    os.environ["G2V_VARIANT"] = variant
    try:
        out = _C.gaussian_voxelizer_forward(*dev(means, opacity, cov), size, rng, dev(feats)[0])
        torch.cuda.synchronize()
    finally:
        if old is None:
            del os.environ["G2V_VARIANT"]
        else:
            os.environ["G2V_VARIANT"] = old
    return [t.cpu().numpy() if isinstance(t, torch.Tensor) else t for t in out]


@pytest.mark.parametrize("n,c,seed,size,half", [(300, 24, 1, 0.4, 6.0), (2000, 512, 2, 0.4, 10.0),
                                                (1500, 1000, 3, 0.4, 10.0), (4000, 1100, 4, 0.4, 12.0)])
def test_tensor_core_splat_matches_oracle_and_fp32_variant(n, c, seed, size, half):
    rng = [-half, -half, -1.0, half, half, 5.4]
    m, o, cv, f = oracle.generate_inputs(n, c, rng, seed=seed, num_outside=n // 20)
    m, o, cv, f = m.numpy(), o.numpy(), cv.numpy(), f.numpy()
    tc = _forward("tc", m, o, cv, f, [size] * 3, rng)
    fp = _forward("simt", m, o, cv, f, [size] * 3, rng)
    for i in (1, 2, 3, 4, 6, 7):  # maps and inverse are variant-independent
        np.testing.assert_array_equal(tc[i], fp[i])
    assert_close("density tc vs simt", tc[0], fp[0], rtol=1e-6)
    assert_close("grid_feats tc vs simt", tc[5], fp[5])
    dims = oracle.grid_shape([size] * 3, rng)[0]
    dref, fref = oracle.forward(m, o, cv, f, tc[2], tc[3], [size] * 3, rng, dims)
    assert_close("density", tc[0], dref)
    assert_close("grid_feats", tc[5], fref)


def test_tensor_core_splat_handles_feature_scales():
    """Channels spanning 1e-30 .. 1e30 and opacities up to 50: the power-of-two scaling keeps the split exact."""
    rng = [-6.0, -6.0, -1.0, 6.0, 6.0, 5.4]
    m, o, cv, f = oracle.generate_inputs(400, 40, rng, seed=9)
    scales = np.logspace(-30, 30, 40).astype(np.float32)
    f = (f.numpy() * scales[None, :]).astype(np.float32)
    o = (o.numpy() * 50.0).astype(np.float32)
    m, cv = m.numpy(), cv.numpy()
    tc = _forward("tc", m, o, cv, f, [0.4] * 3, rng)
    dims = oracle.grid_shape([0.4] * 3, rng)[0]
    dref, fref = oracle.forward(m, o, cv, f, tc[2], tc[3], [0.4] * 3, rng, dims)
    assert_close("density", tc[0], dref)
    for ch in (0, 13, 39):  # per channel, relative to that channel's own scale
        assert_close(f"grid_feats[..., {ch}]", tc[5][..., ch], fref[..., ch])


def test_device_error_word_is_clear():
    import ctypes
    from CudaGaussianVoxelizer import _lib
    w = ctypes.c_int(-1)
    _lib.check(_lib.load().g2v_device_error(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(w)),
               "g2v_device_error")
    assert w.value == 0


def _with_env(env, fn):
    old = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        out = fn()
        torch.cuda.synchronize()
    finally:
        for k, v in old.items():
            if v is None:
                del os.environ[k]
            else:
                os.environ[k] = v
    return out


def _with_variant(variant, fn):
    return _with_env({"G2V_VARIANT": variant}, fn)


@pytest.mark.parametrize("n,c,seed,half,var_max,xt", [
    (300, 24, 1, 6.0, 2.5, None),      # one slot pass, one channel group
    (2000, 37, 2, 8.0, 2.5, None),     # C not a multiple of 4 (scalar gradient loads)
    (3000, 300, 3, 6.0, 8.0, None),    # > 256 Gaussians per block (several slot passes), 2 channel groups
    (4000, 520, 4, 10.0, 2.5, (3, 9)),  # x-slab of tiles (partial rows of blocks cut by the slab)
])
def test_tensor_core_backward_matches_oracle_and_fp32_variant(n, c, seed, half, var_max, xt):
    from CudaGaussianVoxelizer import _C
    size, rng = [0.4] * 3, [-half, -half, -1.0, half, half, 5.4]
    m, o, cv, f = oracle.generate_inputs(n, c, rng, seed=seed, num_outside=n // 20, var_max=var_max)
    m, o, cv, f = m.numpy(), o.numpy(), cv.numpy(), f.numpy()
    dims = oracle.grid_shape(size, rng)[0]
    g = torch.Generator().manual_seed(seed + 3)
    gD = torch.randn(*dims, generator=g)
    gF = torch.randn(*dims, c, generator=g)
    mt, ot, ct, ft = dev(m, o, cv, f)
    out = _C.gaussian_voxelizer_forward(mt, ot, ct, size, rng, ft)
    density, cov_inv, lb, ub, nvox, grid_feats, off, ids, _ = out
    gDt, gFt = gD.cuda(), gF.cuda()

    def bwd():
        return [t.cpu().numpy() for t in _C.gaussian_voxelizer_backward(
            gDt, gFt, mt, ot, cov_inv, size, rng, lb, ub, nvox, off, ids, density, grid_feats, ft,
            tile_x_range=xt)[:4]]

    tc = _with_variant("tc", bwd)
    fp = _with_variant("simt", bwd)
    names = ("grad_means", "grad_cov", "grad_opacity", "grad_features")
    for name, a, b in zip(names, tc, fp):
        assert_close(f"{name} tc vs simt", a, b)

    xr = None if xt is None else (xt[0] * 4, min(xt[1] * 4, dims[0]))
    lb_h, ub_h = lb.cpu().numpy(), ub.cpu().numpy()
    dref, fref = oracle.forward(m, o, cv, f, lb_h, ub_h, size, rng, dims, x_range=xr)
    ref = oracle.backward(m, o, cv, f, lb_h, ub_h, size, rng, dims, gD.numpy(), gF.numpy(), dref, fref, x_range=xr)
    for name, a, b in zip(names, tc, ref):
        assert_close(name, a, b)


@pytest.mark.parametrize("n,c,seed,half,var_max", [
    (300, 24, 1, 6.0, 2.5),      # one slot pass, a single channel group with most channels beyond C
    (3000, 300, 3, 6.0, 8.0),    # blocks of > 256 and > 512 Gaussians (several slot passes)
    (2000, 37, 2, 8.0, 2.5),     # C not a multiple of 4 (converters load the gradient rows themselves)
])
def test_feature_gradient_pass_against_oracle(n, c, seed, half, var_max):
    """The tensor-core backward on block lists of one, two and several slot passes: every gradient,
    the feature gradient included, within the parity bar of the float64 oracle."""
    from CudaGaussianVoxelizer import _C
    size, rng = [0.4] * 3, [-half, -half, -1.0, half, half, 5.4]
    m, o, cv, f = oracle.generate_inputs(n, c, rng, seed=seed, num_outside=n // 20, var_max=var_max)
    dims = oracle.grid_shape(size, rng)[0]
    g = torch.Generator().manual_seed(seed + 7)
    gD, gF = torch.randn(*dims, generator=g).cuda(), torch.randn(*dims, c, generator=g).cuda()
    mt, ot, ct, ft = dev(m.numpy(), o.numpy(), cv.numpy(), f.numpy())
    density, cov_inv, lb, ub, nvox, grid_feats, off, ids, _ = _C.gaussian_voxelizer_forward(mt, ot, ct, size, rng, ft)
    got = [t.cpu().numpy() for t in _C.gaussian_voxelizer_backward(
        gD, gF, mt, ot, cov_inv, size, rng, lb, ub, nvox, off, ids, density, grid_feats, ft)[:4]]
    lb_h, ub_h = lb.cpu().numpy(), ub.cpu().numpy()
    m, o, cv, f = m.numpy(), o.numpy(), cv.numpy(), f.numpy()
    dref, fref = oracle.forward(m, o, cv, f, lb_h, ub_h, size, rng, dims)
    ref = oracle.backward(m, o, cv, f, lb_h, ub_h, size, rng, dims, gD.cpu().numpy(), gF.cpu().numpy(), dref, fref)
    for name, a, b in zip(("grad_means", "grad_cov", "grad_opacity", "grad_features"), got, ref):
        assert_close(name, a, b)


@pytest.mark.parametrize("env,c", [({"G2V_SPLAT_WW": "8"}, 600), ({"G2V_SPLAT_WCACHE": "0"}, 600),
                                   ({"G2V_SPLAT_WW": "8", "G2V_SPLAT_WCACHE": "0"}, 600),
                                   ({"G2V_SPLAT_WW": "4"}, 200), ({"G2V_SPLAT_WCACHE": "0"}, 200)])
def test_splat_weight_variants_match_default(env, c):
    """The weight cache changes where the weights come from, not their values: bit-identical.  Four and eight
    weight warps (the default is eight for one channel group, four for several) sum the density over a
    different grouping of the Gaussians: within the parity bar."""
    rng = [-10.0, -10.0, -1.0, 10.0, 10.0, 5.4]
    m, o, cv, f = oracle.generate_inputs(3000, c, rng, seed=11, num_outside=150)
    args = (m.numpy(), o.numpy(), cv.numpy(), f.numpy(), [0.4] * 3, rng)
    ref = _forward("tc", *args)
    got = _with_env(env, lambda: _forward("tc", *args))
    if "G2V_SPLAT_WW" in env:
        assert_close("density", got[0], ref[0], rtol=1e-6)
        assert_close("grid_feats", got[5], ref[5])
        same_ww = _with_env({"G2V_SPLAT_WW": env["G2V_SPLAT_WW"]}, lambda: _forward("tc", *args))
        ref = same_ww
    np.testing.assert_array_equal(got[0], ref[0])
    np.testing.assert_array_equal(got[5], ref[5])


@pytest.mark.parametrize("shape", ["2,2,4", "1,1,4", "2,1,2", "4,4,2"])
def test_feature_gradient_block_shapes_match_default(shape):
    """The feature-gradient blocks (G2V_FPASS_BLOCK) change which Gaussians share a block, how many slot
    passes a block takes and how many partial rows a Gaussian sums, not the gradient: every shape agrees
    with the default blocks and with the float64 oracle within the parity bar."""
    from CudaGaussianVoxelizer import _C
    size, rng = [0.4] * 3, [-8.0, -8.0, -1.0, 8.0, 8.0, 5.4]
    n, c = 3000, 300
    m, o, cv, f = oracle.generate_inputs(n, c, rng, seed=21, num_outside=n // 20, var_max=8.0)
    dims = oracle.grid_shape(size, rng)[0]
    g = torch.Generator().manual_seed(22)
    gD, gF = torch.randn(*dims, generator=g).cuda(), torch.randn(*dims, c, generator=g).cuda()
    mt, ot, ct, ft = dev(m.numpy(), o.numpy(), cv.numpy(), f.numpy())
    density, cov_inv, lb, ub, nvox, grid_feats, off, ids, _ = _C.gaussian_voxelizer_forward(mt, ot, ct, size, rng, ft)

    def bwd():
        return [t.cpu().numpy() for t in _C.gaussian_voxelizer_backward(
            gD, gF, mt, ot, cov_inv, size, rng, lb, ub, nvox, off, ids, density, grid_feats, ft)[:4]]

    ref = bwd()
    got = _with_env({"G2V_FPASS_BLOCK": shape}, bwd)
    names = ("grad_means", "grad_cov", "grad_opacity", "grad_features")
    for name, a, b in zip(names, got, ref):
        assert_close(f"{name} ({shape} vs default blocks)", a, b)
    lb_h, ub_h = lb.cpu().numpy(), ub.cpu().numpy()
    m, o, cv, f = m.numpy(), o.numpy(), cv.numpy(), f.numpy()
    dref, fref = oracle.forward(m, o, cv, f, lb_h, ub_h, size, rng, dims)
    oref = oracle.backward(m, o, cv, f, lb_h, ub_h, size, rng, dims, gD.cpu().numpy(), gF.cpu().numpy(), dref, fref)
    for name, a, b in zip(names, got, oref):
        assert_close(f"{name} ({shape} blocks vs oracle)", a, b)
