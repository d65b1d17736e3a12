"""CPU oracle for the G2V path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py`` import this module, and
only as the checker (or as the timed CPU baseline).  The product library never calls it.

It wraps ``g2v_oracle.c`` (built into ``oracle/_build/libg2v_oracle.so`` by :func:`build`) with numpy
arrays.  The C file lists, per function, which part of the reference it restates:
``src/cuda_gaussian_voxelizer.cu`` for the grid shape, the boxes and the CSR maps, and
``test/test_reference.py:57-79`` (float64 brute force) for the values and, by analytic differentiation,
the gradients.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(HERE, "_build")
LIB_PATH = os.path.join(BUILD_DIR, "libg2v_oracle.so")
SRC = os.path.join(HERE, "g2v_oracle.c")

_lib = None


def build(force: bool = False) -> str:
    """Compile the oracle with gcc (no fp contraction, OpenMP) into oracle/_build/."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    if not force and os.path.exists(LIB_PATH) and os.path.getmtime(LIB_PATH) >= os.path.getmtime(SRC):
        return LIB_PATH
    tmp = LIB_PATH + f".tmp{os.getpid()}"
    subprocess.check_call(["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
                           "-fno-fast-math", SRC, "-o", tmp, "-lm"])
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(SRC):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        i64, i32 = ctypes.c_int64, ctypes.c_int
        L.g2v_oracle_grid_shape.argtypes = [P, P, P, P]
        L.g2v_oracle_grid_shape.restype = i32
        L.g2v_oracle_boxes.argtypes = [i64, P, P, P, P, P, P, P, P, P, P, P, P, P]
        L.g2v_oracle_boxes.restype = None
        L.g2v_oracle_g2t_offsets.argtypes = [i64, P, P]
        L.g2v_oracle_g2t_offsets.restype = i64
        L.g2v_oracle_g2t_fill.argtypes = [i64, P, P, P, P, P]
        L.g2v_oracle_g2t_fill.restype = None
        L.g2v_oracle_t2g.argtypes = [i64, i64, P, P, P, P]
        L.g2v_oracle_t2g.restype = None
        L.g2v_oracle_forward.argtypes = [i64, i32, P, P, P, P, P, P, P, P, P, i32, i32, P, P, i32]
        L.g2v_oracle_forward.restype = None
        L.g2v_oracle_backward.argtypes = [i64, i32, P, P, P, P, P, P, P, P, P, i32, i32, P, P, P, P, P, P, P,
                                          P, i32]
        L.g2v_oracle_backward.restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def grid_shape(voxel_size, voxel_range):
    """(dims, tiles) with the reference's float32 arithmetic; raises ValueError on an invalid grid."""
    size, rng = _f32(voxel_size), _f32(voxel_range)
    dims = np.zeros(3, np.int32)
    tiles = np.zeros(3, np.int32)
    if lib().g2v_oracle_grid_shape(_p(size), _p(rng), _p(dims), _p(tiles)) != 0:
        raise ValueError(f"invalid voxel grid: size={voxel_size} range={voxel_range}")
    return tuple(int(v) for v in dims), tuple(int(v) for v in tiles)


@dataclass
class Boxes:
    dims: tuple
    tiles: tuple
    lb: np.ndarray
    ub: np.ndarray
    num_voxels: np.ndarray
    tile_lo: np.ndarray
    tile_hi: np.ndarray
    num_tiles: np.ndarray
    cov_inv: np.ndarray
    g2t_offsets: np.ndarray      # int64 (N+1)
    g2t_tile_ids: np.ndarray     # int32 (M)
    tile_offsets: np.ndarray     # int64 (num_tiles_total+1)
    t2g_gaussians: np.ndarray    # int32 (M)


def boxes(means, cov, voxel_size, voxel_range) -> Boxes:
    """Boxes, G2T and T2G maps of the reference (float32 box arithmetic, IEEE sqrt/div)."""
    means, cov = _f32(means).reshape(-1, 3), _f32(cov).reshape(-1, 9)
    size, rng = _f32(voxel_size), _f32(voxel_range)
    dims, tiles = grid_shape(size, rng)
    n = means.shape[0]
    d = np.asarray(dims, np.int32)
    t = np.asarray(tiles, np.int32)
    lb = np.zeros((n, 3), np.int32)
    ub = np.zeros((n, 3), np.int32)
    nv = np.zeros(n, np.int32)
    tlo = np.zeros((n, 3), np.int32)
    thi = np.zeros((n, 3), np.int32)
    nt = np.zeros(n, np.int32)
    ci = np.zeros((n, 9), np.float32)
    L = lib()
    L.g2v_oracle_boxes(n, _p(means), _p(cov), _p(size), _p(rng), _p(d), _p(t), _p(lb), _p(ub), _p(nv), _p(tlo),
                       _p(thi), _p(nt), _p(ci))
    off = np.zeros(n + 1, np.int64)
    m = L.g2v_oracle_g2t_offsets(n, _p(nt), _p(off))
    ids = np.zeros(max(m, 1), np.int32)
    L.g2v_oracle_g2t_fill(n, _p(tlo), _p(thi), _p(off), _p(t), _p(ids))
    ntt = int(t[0]) * int(t[1]) * int(t[2])
    toff = np.zeros(ntt + 1, np.int64)
    t2g = np.zeros(max(m, 1), np.int32)
    L.g2v_oracle_t2g(n, ntt, _p(off), _p(ids), _p(toff), _p(t2g))
    return Boxes(dims, tiles, lb, ub, nv, tlo, thi, nt, ci, off, ids[:m], toff, t2g[:m])


def csr_from_boxes(lb, ub, dims):
    """G2T / T2G maps of given voxel boxes (tile box = voxel box / 4, empty when ub < lb)."""
    lb, ub = _i32(lb).reshape(-1, 3), _i32(ub).reshape(-1, 3)
    n = lb.shape[0]
    tiles = np.asarray([(d + 3) // 4 for d in dims], np.int32)
    empty = (ub < lb).any(axis=1)
    tlo = np.where(empty[:, None], 0, lb // 4).astype(np.int32)
    thi = np.where(empty[:, None], -1, ub // 4).astype(np.int32)
    nt = np.where(empty, 0, np.prod(thi - tlo + 1, axis=1)).astype(np.int32)
    L = lib()
    off = np.zeros(n + 1, np.int64)
    m = L.g2v_oracle_g2t_offsets(n, _p(nt), _p(off))
    ids = np.zeros(max(m, 1), np.int32)
    L.g2v_oracle_g2t_fill(n, _p(np.ascontiguousarray(tlo)), _p(np.ascontiguousarray(thi)), _p(off), _p(tiles),
                          _p(ids))
    ntt = int(tiles.prod())
    toff = np.zeros(ntt + 1, np.int64)
    t2g = np.zeros(max(m, 1), np.int32)
    L.g2v_oracle_t2g(n, ntt, _p(off), _p(ids), _p(toff), _p(t2g))
    return off, ids[:m], toff, t2g[:m]


def forward(means, opacity, cov, features, lb, ub, voxel_size, voxel_range, dims, x_range=None, nthreads=0):
    """float64 brute-force density (X,Y,Z) and grid_feats (X,Y,Z,C) given the boxes lb/ub.

    ``voxel_size``/``voxel_range`` are taken as float64 (the reference test builds them from Python
    floats).  With ``x_range=(x0, x1)`` only that voxel slab is computed (the rest stays zero).
    """
    means, opacity, cov = _f32(means).reshape(-1, 3), _f32(opacity).reshape(-1), _f32(cov).reshape(-1, 9)
    n = means.shape[0]
    feats = None if features is None else _f32(features).reshape(n, -1)
    c = 0 if feats is None else feats.shape[1]
    X, Y, Z = dims
    vlo = np.asarray(voxel_range[:3], np.float64)
    vs = np.asarray(voxel_size, np.float64)
    dm = np.asarray(dims, np.int32)
    x0, x1 = (0, X) if x_range is None else x_range
    dens = np.zeros((X, Y, Z), np.float64)
    gf = np.zeros((X, Y, Z, c), np.float64) if c > 0 else None
    lib().g2v_oracle_forward(n, c, _p(means), _p(opacity), _p(cov), _p(feats), _p(_i32(lb)), _p(_i32(ub)),
                             _p(vlo), _p(vs), _p(dm), x0, x1, _p(dens), _p(gf), nthreads)
    if gf is None:
        gf = np.zeros((X, Y, Z, 0), np.float64)
    return dens, gf


def backward(means, opacity, cov, features, lb, ub, voxel_size, voxel_range, dims, grad_density, grad_feats,
             density, grid_feats, x_range=None, nthreads=0):
    """float64 analytic gradients (means (N,3), cov (N,9), opacity (N,), features (N,C))."""
    means, opacity, cov = _f32(means).reshape(-1, 3), _f32(opacity).reshape(-1), _f32(cov).reshape(-1, 9)
    n = means.shape[0]
    feats = None if features is None else _f32(features).reshape(n, -1)
    c = 0 if feats is None else feats.shape[1]
    X, Y, Z = dims
    vlo = np.asarray(voxel_range[:3], np.float64)
    vs = np.asarray(voxel_size, np.float64)
    dm = np.asarray(dims, np.int32)
    x0, x1 = (0, X) if x_range is None else x_range
    gD = _f32(grad_density).reshape(-1)
    gF = _f32(grad_feats).reshape(-1) if c > 0 else None
    D = np.ascontiguousarray(np.asarray(density, np.float64)).reshape(-1)
    F = np.ascontiguousarray(np.asarray(grid_feats, np.float64)).reshape(-1) if c > 0 else None
    g_means = np.zeros((n, 3), np.float64)
    g_cov = np.zeros((n, 9), np.float64)
    g_op = np.zeros(n, np.float64)
    g_feat = np.zeros((n, c), np.float64)
    lib().g2v_oracle_backward(n, c, _p(means), _p(opacity), _p(cov), _p(feats), _p(_i32(lb)), _p(_i32(ub)),
                              _p(vlo), _p(vs), _p(dm), x0, x1, _p(gD), _p(gF), _p(D), _p(F), _p(g_means),
                              _p(g_cov), _p(g_op), _p(g_feat), nthreads)
    return g_means, g_cov, g_op, g_feat


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def rel_err(a, b) -> float:
    """Relative L2 error, as test/test_reference.py:82-83 defines it."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), 1e-30))


def generate_inputs(num_gaussians, feat_dim, voxel_range, num_outside=0, seed=0, var_max=2.5, expand=0.0):
    """Seeded CPU inputs with the reference's distributions (test/test_reference.py:30-45).

    means ~ U(range) (optionally widened by ``expand`` x extent on each side), opacity ~ U(0,1),
    cov = R diag(U(0.5, var_max)) R^T with R from QR of randn(3,3), features ~ randn.  ``num_outside``
    extra Gaussians are centred beyond x_max by U(0, 1.5).  Uses torch's CPU generator so that the
    same seed gives the same inputs everywhere.
    """
    import torch
    g = torch.Generator().manual_seed(seed)
    lo = torch.tensor(voxel_range[:3], dtype=torch.float32)
    hi = torch.tensor(voxel_range[3:], dtype=torch.float32)
    if expand:
        ext = hi - lo
        lo, hi = lo - expand * ext, hi + expand * ext
    means = torch.rand(num_gaussians, 3, generator=g) * (hi - lo) + lo
    if num_outside:
        lo0 = torch.tensor(voxel_range[:3], dtype=torch.float32)
        hi0 = torch.tensor(voxel_range[3:], dtype=torch.float32)
        out = torch.rand(num_outside, 3, generator=g) * (hi0 - lo0) + lo0
        out[:, 0] = hi0[0] + torch.rand(num_outside, generator=g) * 1.5
        means = torch.cat([means, out])
    n = means.shape[0]
    opacity = torch.rand(n, generator=g)
    R, _ = torch.linalg.qr(torch.randn(n, 3, 3, generator=g))
    var = torch.rand(n, 3, generator=g) * (var_max - 0.5) + 0.5
    cov = (R @ torch.diag_embed(var) @ R.mT).reshape(n, 9)
    feats = torch.randn(n, feat_dim, generator=g) if feat_dim is not None else None
    return means.contiguous(), opacity.contiguous(), cov.contiguous(), (
        feats.contiguous() if feats is not None else None)


# ---------------------------------------------------------------------------------------------------
# Feature cosine loss (src/cuda_feats_loss.cu), float64 numpy restatement.

LOSS_EPS = 1e-6  # include/utils.cuh:80 (`eps`), shared by the norm clamps and the denominator


def _loss_rows(voxel_label, occ_mask, grid_feats, gt_feats):
    """(valid mask [V], prediction rows, target rows) -- the rows of the valid voxels only, in float64."""
    c = np.shape(grid_feats)[-1]
    label = np.asarray(voxel_label, np.float32).reshape(-1)
    mask = np.asarray(occ_mask).reshape(-1).astype(bool)
    valid = mask & (label > 0)  # cuda_feats_loss.cu:70-71 (and :138, :251)
    pv = np.asarray(grid_feats).reshape(label.size, c)[valid].astype(np.float64)
    gv = np.asarray(gt_feats).reshape(label.size, c)[valid].astype(np.float64)
    return valid, pv, gv


def _row_sums(pv, gv):
    return (np.einsum("ij,ij->i", pv, gv), np.einsum("ij,ij->i", pv, pv), np.einsum("ij,ij->i", gv, gv))


def cosine_loss_forward(voxel_label, occ_mask, grid_feats, gt_feats):
    """(mean loss, valid count) of CudaFeatsCosinelossForward (cuda_feats_loss.cu:146-225).

    Per valid voxel (VoxelCosineLossKernel, :80-99): dot, |p|^2, |g|^2 over the channels, then
    1 - dot / (sqrt(max(|p|^2, eps)) sqrt(max(|g|^2, eps)) + eps); invalid voxels contribute 0.
    The sum and the count (ReduceLossAndCountKernel, :104-143) give mean = sum / count, or 0 when
    count is 0 (:196-198).
    """
    valid, pv, gv = _loss_rows(voxel_label, occ_mask, grid_feats, gt_feats)
    dot, pp, gg = _row_sums(pv, gv)
    pn = np.sqrt(np.maximum(pp, LOSS_EPS))
    gn = np.sqrt(np.maximum(gg, LOSS_EPS))
    loss_v = 1.0 - dot / (pn * gn + LOSS_EPS)
    count = int(valid.sum())
    return (float(loss_v.sum()) / count if count > 0 else 0.0), count


def cosine_loss_backward(grad_output, num_valid_voxel, voxel_label, occ_mask, grid_feats, gt_feats,
                         return_terms=False):
    """d loss / d grid_feats of CudaFeatsCosinelossBackward (cuda_feats_loss.cu:311-366).

    inv_count = 1/count or 0 (:319); per valid voxel (CosineLossBackwardKernel, :262-287) with
    a = sqrt(max(|p|^2, eps)), b = sqrt(max(|g|^2, eps)), D = a b + eps:
    grad = grad_out inv_count (-g / D + [|p|^2 > eps] dot b / (a D^2) p); invalid voxels get 0.
    ``return_terms`` also returns |grad_out inv_count| (|g / D| + |c2 p|) per element: the size of the
    two terms whose difference is the gradient, the scale of float32 rounding when they cancel.
    """
    valid, pv, gv = _loss_rows(voxel_label, occ_mask, grid_feats, gt_feats)
    inv_count = 1.0 / num_valid_voxel if num_valid_voxel > 0 else 0.0
    dot, pp, gg = _row_sums(pv, gv)
    a = np.sqrt(np.maximum(pp, LOSS_EPS))
    b = np.sqrt(np.maximum(gg, LOSS_EPS))
    D = a * b + LOSS_EPS
    c1 = -1.0 / D
    c2 = np.where(pp > LOSS_EPS, dot * b / (a * D * D), 0.0)
    scale = float(grad_output) * inv_count
    grad = np.zeros((valid.size, pv.shape[1]), np.float64)
    grad[valid] = scale * (c1[:, None] * gv + c2[:, None] * pv)
    if not return_terms:
        return grad.reshape(np.shape(grid_feats))
    terms = np.zeros_like(grad)
    terms[valid] = abs(scale) * (np.abs(c1[:, None] * gv) + np.abs(c2[:, None] * pv))
    return grad.reshape(np.shape(grid_feats)), terms.reshape(np.shape(grid_feats))


def generate_loss_inputs(dims, channels, case="noise", p_label=0.25, p_mask=0.7, noise=0.1, seed=0):
    """Seeded inputs shaped like the reference's loss tests (test/test_feats_loss_backward.py:58-64,
    :151-180): label = (U < p_label) as float, mask = U < p_mask, grid_feats ~ randn(X,Y,Z,C) and a
    target that is the prediction ("same"), its negation ("neg") or the prediction plus
    ``noise`` x randn ("noise")."""
    import torch
    gen = torch.Generator().manual_seed(seed)
    X, Y, Z = dims
    feats = torch.randn(X, Y, Z, channels, generator=gen)
    label = (torch.rand(X, Y, Z, generator=gen) < p_label).float()
    mask = torch.rand(X, Y, Z, generator=gen) < p_mask
    if case == "same":
        gt = feats.clone()
    elif case == "neg":
        gt = -feats
    elif case == "noise":
        gt = feats + noise * torch.randn(X, Y, Z, channels, generator=gen)
    else:
        raise ValueError(case)
    return label.contiguous(), mask.contiguous(), feats.contiguous(), gt.contiguous()


# ---------------------------------------------------------------------------------------------------
# Covariance from (scale, rotation quaternion): the GaussTR front end of the voxelizer
# (test/gaussian_voxelizer.py:14-37, quat_to_rotmat and get_covariance), float64 numpy restatement.

def _rotmat(q):
    """Rotation matrices (..., 3, 3) of quaternions (..., 4) = (r, x, y, z) after normalisation (:14-29)."""
    q = q / np.sqrt((q ** 2).sum(axis=-1, keepdims=True))
    r, x, y, z = q[..., 0], q[..., 1], q[..., 2], q[..., 3]
    R = np.empty(q.shape[:-1] + (3, 3))
    R[..., 0, 0] = 1 - 2 * (y * y + z * z)
    R[..., 0, 1] = 2 * (x * y - r * z)
    R[..., 0, 2] = 2 * (x * z + r * y)
    R[..., 1, 0] = 2 * (x * y + r * z)
    R[..., 1, 1] = 1 - 2 * (x * x + z * z)
    R[..., 1, 2] = 2 * (y * z - r * x)
    R[..., 2, 0] = 2 * (x * z - r * y)
    R[..., 2, 1] = 2 * (y * z + r * x)
    R[..., 2, 2] = 1 - 2 * (x * x + y * y)
    return q, R


def covariance_from_scale_rot(scales, rotations):
    """Sigma = (R diag(s)) (R diag(s))^T, (..., 3, 3), of get_covariance(s, quat_to_rotmat(q)) (:31-37)."""
    s = np.asarray(scales, np.float64)
    _, R = _rotmat(np.asarray(rotations, np.float64))
    M = R * s[..., None, :]
    return M @ np.swapaxes(M, -1, -2)


def covariance_from_scale_rot_backward(scales, rotations, grad_cov):
    """(dL/ds (..., 3), dL/dq (..., 4)) from dL/dSigma (..., 3, 3) with independent entries, by the chain
    rule through Sigma = M M^T, M = R diag(s), R = R(q / |q|) -- what autograd through the reference
    front end computes."""
    s = np.asarray(scales, np.float64)
    q0 = np.asarray(rotations, np.float64)
    G = np.asarray(grad_cov, np.float64).reshape(s.shape[:-1] + (3, 3))
    q, R = _rotmat(q0)
    M = R * s[..., None, :]
    gM = (G + np.swapaxes(G, -1, -2)) @ M
    gs = (gM * R).sum(axis=-2)
    gR = gM * s[..., None, :]
    r, x, y, z = q[..., 0], q[..., 1], q[..., 2], q[..., 3]
    g = [gR[..., i, j] for i in range(3) for j in range(3)]
    gr = 2 * (-z * g[1] + y * g[2] + z * g[3] - x * g[5] - y * g[6] + x * g[7])
    gx = 2 * (y * g[1] + z * g[2] + y * g[3] - 2 * x * g[4] - r * g[5] + z * g[6] + r * g[7] - 2 * x * g[8])
    gy = 2 * (-2 * y * g[0] + x * g[1] + r * g[2] + x * g[3] + z * g[5] - r * g[6] + z * g[7] - 2 * y * g[8])
    gz = 2 * (-2 * z * g[0] - r * g[1] + x * g[2] + r * g[3] - 2 * z * g[4] + y * g[5] + x * g[6] + y * g[7])
    gqh = np.stack([gr, gx, gy, gz], axis=-1)
    norm = np.sqrt((q0 ** 2).sum(axis=-1, keepdims=True))
    gq = (gqh - q * (q * gqh).sum(axis=-1, keepdims=True)) / norm
    return gs, gq


def generate_scale_rot(n, seed=0, var_max=2.5):
    """Seeded scales and quaternions with cfg-like spreads: s = sqrt(U(0.5, var_max)) per axis (the
    variances of generate_inputs), q = randn(4) scaled by U(0.5, 2) (unnormalised, as networks emit)."""
    import torch
    g = torch.Generator().manual_seed(seed)
    s = torch.sqrt(torch.rand(n, 3, generator=g) * (var_max - 0.5) + 0.5)
    q = torch.randn(n, 4, generator=g) * (torch.rand(n, 1, generator=g) * 1.5 + 0.5)
    return s.contiguous(), q.contiguous()
