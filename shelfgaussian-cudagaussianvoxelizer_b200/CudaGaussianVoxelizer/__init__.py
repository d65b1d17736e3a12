"""B200 Gaussian-to-voxel splatting, drop-in for the reference ``CudaGaussianVoxelizer`` package.

    from CudaGaussianVoxelizer import PyCudaGaussianVoxelizer, PyCudaFeatsCosineLoss
    voxelizer = PyCudaGaussianVoxelizer(voxel_size=[0.4] * 3, voxel_range=[-40, -40, -1, 40, 40, 5.4])
    density, grid_feats, stats = voxelizer(means3D, opacity, covariances, features)
    loss, loss_stats = PyCudaFeatsCosineLoss()(voxel_label, occ_mask, grid_feats, target_feats)

Same modules, autograd functions, argument meaning, outputs and ``stats`` semantics as the reference's
``CudaGaussianVoxelizer/__init__.py:10-95``; the compute runs in libg2v.so (hand-written sm_100a
kernels behind a C ABI, include/g2v.h).
"""
from __future__ import annotations

import os

import torch
import torch.nn as nn

from . import _C, _lib
from ._C import (CudaFeatsCosinelossBackward, CudaFeatsCosinelossForward, _cosine_loss_forward_impl, _forward_impl,
                 gaussian_voxelizer_backward, gaussian_voxelizer_forward)

_lib.load()  # fail loudly at import when the native library is missing

# G2V_REUSE_UNITS=0: the backward rebuilds the tile pass's unit lists instead of taking the forward's
_REUSE_UNITS = os.environ.get("G2V_REUSE_UNITS", "1") != "0"

from .graphs import GraphedGaussianVoxelizer  # noqa: E402

__all__ = ["PyCudaGaussianVoxelizer", "GraphedGaussianVoxelizer", "_CudaGaussianVoxelizeFunction",
           "_CudaGaussianVoxelizeSRFunction",
           "covariance_from_scale_rot", "gaussian_voxelizer_forward",
           "gaussian_voxelizer_backward", "PyCudaFeatsCosineLoss", "_CudaFeatsCosinelossFunction",
           "CudaFeatsCosinelossForward", "CudaFeatsCosinelossBackward", "_C"]


class _CudaGaussianVoxelizeFunction(torch.autograd.Function):
    """Autograd function of the splat (reference CudaGaussianVoxelizer/__init__.py:10-47)."""

    @staticmethod
    def forward(ctx, means3D, opacity, covariances, voxel_size, voxel_range, features, timing=True, scenes=None,
                caps=None):
        # the forward also counts the backward's (Gaussian, block) pairs in its one synchronisation (or, with
        # capacities, synchronises not at all)
        # the splat's unit lists are kept for the backward's tile pass (it would rebuild the same ones)
        ((density, cov_inv, lb, ub, nvox, grid_feats, g2t_offsets, g2t_tile_ids, fwd_sec),
         num_block_pairs, units) = _forward_impl(means3D, opacity, covariances, voxel_size, voxel_range, features,
                                                 timing, plan=True, scenes=scenes, caps=caps,
                                                 keep_units=_REUSE_UNITS)
        ctx.units = units
        ctx.num_scenes = 1 if scenes is None else scenes[1]
        stats = torch.zeros(2, dtype=torch.float32, device="cpu")
        stats[0] = fwd_sec
        ctx.save_for_backward(means3D, opacity, voxel_size, voxel_range, cov_inv, lb, ub, nvox, g2t_offsets,
                              g2t_tile_ids, density, grid_feats, features, stats)
        ctx.timing = timing
        ctx.num_block_pairs = num_block_pairs
        ctx.mark_non_differentiable(stats)
        return density, grid_feats, stats

    @staticmethod
    def backward(ctx, grad_density_output, grad_feats_output, grad_stats):
        (means3D, opacity, voxel_size, voxel_range, cov_inv, lb, ub, nvox, g2t_offsets, g2t_tile_ids, density,
         grid_feats, features, stats) = ctx.saved_tensors
        gout = grad_density_output.to(torch.float32).contiguous()
        if features is not None and features.shape[1] > 0:
            gfeat = grad_feats_output.to(torch.float32).contiguous()
        else:
            gfeat = grad_feats_output
        grad_means, grad_cov, grad_op, grad_feats, bwd_sec = gaussian_voxelizer_backward(
            gout, gfeat, means3D, opacity, cov_inv, voxel_size, voxel_range, lb, ub, nvox, g2t_offsets,
            g2t_tile_ids, density, grid_feats, features, timing=ctx.timing, num_block_pairs=ctx.num_block_pairs,
            num_scenes=ctx.num_scenes, units=ctx.units)
        ctx.units = None
        stats[1] = bwd_sec
        return (grad_means, grad_op, grad_cov, None, None, grad_feats if features is not None else None, None, None,
                None)


class _CudaGaussianVoxelizeSRFunction(torch.autograd.Function):
    """The splat for Gaussians given by scales (N,3) and rotation quaternions (N,4) instead of covariances:
    the covariances are formed inside the preparation kernel and the gradient reduction applies the chain
    rule, so neither Sigma nor dL/dSigma is materialised.  Same outputs as _CudaGaussianVoxelizeFunction;
    gradients flow to means3D, opacity, scales, rotations and features (the composition of the reference
    voxelizer with GaussTR's get_covariance / quat_to_rotmat, test/gaussian_voxelizer.py:14-37)."""

    @staticmethod
    def forward(ctx, means3D, opacity, scales, rotations, voxel_size, voxel_range, features, timing=True,
                scenes=None):
        ((density, cov_inv, lb, ub, nvox, grid_feats, g2t_offsets, g2t_tile_ids, fwd_sec),
         num_block_pairs) = _forward_impl(means3D, opacity, None, voxel_size, voxel_range, features, timing,
                                          scale_rot=(scales, rotations), scenes=scenes)
        ctx.num_scenes = 1 if scenes is None else scenes[1]
        stats = torch.zeros(2, dtype=torch.float32, device="cpu")
        stats[0] = fwd_sec
        ctx.save_for_backward(means3D, opacity, scales, rotations, voxel_size, voxel_range, cov_inv, lb, ub, nvox,
                              g2t_offsets, g2t_tile_ids, density, grid_feats, features, stats)
        ctx.timing = timing
        ctx.num_block_pairs = num_block_pairs
        ctx.mark_non_differentiable(stats)
        return density, grid_feats, stats

    @staticmethod
    def backward(ctx, grad_density_output, grad_feats_output, grad_stats):
        (means3D, opacity, scales, rotations, voxel_size, voxel_range, cov_inv, lb, ub, nvox, g2t_offsets,
         g2t_tile_ids, density, grid_feats, features, stats) = ctx.saved_tensors
        gout = grad_density_output.to(torch.float32).contiguous()
        if features is not None and features.shape[1] > 0:
            gfeat = grad_feats_output.to(torch.float32).contiguous()
        else:
            gfeat = grad_feats_output
        grad_means, (grad_scales, grad_rot), grad_op, grad_feats, bwd_sec = gaussian_voxelizer_backward(
            gout, gfeat, means3D, opacity, cov_inv, voxel_size, voxel_range, lb, ub, nvox, g2t_offsets,
            g2t_tile_ids, density, grid_feats, features, timing=ctx.timing, num_block_pairs=ctx.num_block_pairs,
            scale_rot=(scales, rotations), num_scenes=ctx.num_scenes)
        stats[1] = bwd_sec
        return (grad_means, grad_op, grad_scales, grad_rot, None, None,
                grad_feats if features is not None else None, None, None)


class _CovarianceFromScaleRot(torch.autograd.Function):
    @staticmethod
    def forward(ctx, scales, rotations):
        ctx.save_for_backward(scales, rotations)
        return _C.covariance_from_scale_rot(scales, rotations)

    @staticmethod
    def backward(ctx, grad_cov):
        scales, rotations = ctx.saved_tensors
        gs, gq = _C.covariance_from_scale_rot_backward(scales, rotations, grad_cov.to(torch.float32))
        return gs, gq


def covariance_from_scale_rot(scales, rotations):
    """Differentiable covariances (..., 3, 3) = R(q/|q|) diag(s)^2 R(q/|q|)^T from (..., 3) scales and
    (..., 4) (r, x, y, z) quaternions: get_covariance(scales, quat_to_rotmat(rotations)) of the reference's
    GaussTR front end (test/gaussian_voxelizer.py:14-37), one sm_100a kernel each way."""
    return _CovarianceFromScaleRot.apply(scales, rotations)


class PyCudaGaussianVoxelizer(nn.Module):
    """Splat 3D Gaussians (and optional per-Gaussian features) into a dense voxel grid.

    forward(means3D (N,3), opacity (N,), covariances (N,9), features (N,C) or None)
        -> (density (X,Y,Z), grid_feats (X,Y,Z,C), stats (2,) CPU float32)
    or forward(means3D, opacity, features=..., scales=(N,3), rotations=(N,4)) for Gaussians given by
    scale and rotation quaternion (the covariance is formed and differentiated inside the kernels).
    ``stats[0]`` is the forward device time in seconds, ``stats[1]`` the backward's (filled by
    ``.backward()``).  ``timing=False`` skips the two end-of-call synchronisations that fill them
    (stats stay 0).  ``max_pairs`` (and ``max_block_pairs`` with features), with ``timing=False``: the
    pair buffers are sized by these capacities instead of the forward's one synchronisation, so a whole
    training step through this module can be captured in a CUDA graph (overflow is flagged in the device
    error word; see ``GraphedGaussianVoxelizer.check``).  Reference: CudaGaussianVoxelizer/__init__.py:69-82.
    """

    def __init__(self, voxel_size=[0.4, 0.4, 0.4], voxel_range=[-40, -40, -1, 40, 40, 5.4], timing: bool = True,
                 max_pairs: int | None = None, max_block_pairs: int | None = None):
        super().__init__()
        self.voxel_size = torch.tensor(voxel_size, dtype=torch.float32, device="cuda")
        self.voxel_range = torch.tensor(voxel_range, dtype=torch.float32, device="cuda")
        self.timing = timing
        # capacities: forward and backward without any host synchronisation (capturable in a CUDA graph)
        self.caps = None if max_pairs is None else (int(max_pairs), int(max_block_pairs or 0))
        if self.caps is not None and timing:
            raise RuntimeError("PyCudaGaussianVoxelizer: max_pairs needs timing=False (no synchronisation)")
        # host copies: the C ABI takes the geometry by value, so no device read-back is needed
        _C._host_values(self.voxel_size, 3, "voxel_size")
        _C._host_values(self.voxel_range, 6, "voxel_range")

    def forward(self, means3D, opacity, covariances=None, features=None, *, scales=None, rotations=None,
                scene_sizes=None):
        """``covariances`` (N,9) as in the reference, or -- in its place -- ``scales`` (N,3) and
        ``rotations`` (N,4) quaternions (r, x, y, z), as GaussTR's voxelizer accepts them
        (test/gaussian_voxelizer.py:168-177); gradients then flow to scales and rotations.

        Batches of scenes splat in one call: either a leading batch dimension on every per-Gaussian input
        (means3D (B,N,3), opacity (B,N), covariances (B,N,9) or (B,N,3,3), features (B,N,C), scales (B,N,3),
        rotations (B,N,4)), or the scenes' Gaussians concatenated along N with ``scene_sizes`` (B counts,
        ragged).  The outputs are then (B,X,Y,Z) and (B,X,Y,Z,C); each scene's result is that of a
        single-scene call.  X must be a multiple of 4 for B > 1."""
        scenes = None
        if means3D.dim() == 3:  # (B, N, ...) equal-size batch
            b, n = means3D.shape[:2]
            flat = lambda t, k: None if t is None else t.reshape(b * n, *k)  # noqa: E731
            means3D, opacity = flat(means3D, (3,)), flat(opacity, ())
            covariances, scales, rotations = flat(covariances, (9,)), flat(scales, (3,)), flat(rotations, (4,))
            features = None if features is None else features.reshape(b * n, features.shape[-1])
            scene_sizes = [n] * b
        if scene_sizes is not None:
            scenes = _C._scene_offsets(scene_sizes, means3D.shape[0], means3D.device)
        if covariances is None:
            if scales is None or rotations is None:
                raise RuntimeError("PyCudaGaussianVoxelizer: pass covariances, or scales and rotations")
            return _CudaGaussianVoxelizeSRFunction.apply(means3D, opacity, scales, rotations, self.voxel_size,
                                                         self.voxel_range, features, self.timing, scenes)
        if scales is not None or rotations is not None:
            raise RuntimeError("PyCudaGaussianVoxelizer: pass covariances or scales/rotations, not both")
        return _CudaGaussianVoxelizeFunction.apply(means3D, opacity, covariances, self.voxel_size, self.voxel_range,
                                                   features, self.timing, scenes, self.caps)


class _CudaFeatsCosinelossFunction(torch.autograd.Function):
    """Autograd function of the feature cosine loss (reference CudaGaussianVoxelizer/__init__.py:49-70).

    Unlike the reference, the valid-voxel count stays on the device between forward and backward and
    the upstream gradient is read on the device, so with ``timing=False`` neither pass synchronises.
    """

    @staticmethod
    def forward(ctx, voxel_label, occ_gt_mask_camera, d_grid_feats, pseudo_dino_gt, timing=True):
        loss, count, fwd_sec = _cosine_loss_forward_impl(voxel_label, occ_gt_mask_camera, d_grid_feats,
                                                         pseudo_dino_gt, timing)
        stats = torch.zeros(2, dtype=torch.float32, device="cpu")
        stats[0] = fwd_sec
        ctx.save_for_backward(voxel_label, occ_gt_mask_camera, d_grid_feats, pseudo_dino_gt, count, stats)
        ctx.timing = timing
        ctx.mark_non_differentiable(stats)
        return loss, stats

    @staticmethod
    def backward(ctx, grad_output, grad_stats):
        voxel_label, occ_gt_mask_camera, d_grid_feats, pseudo_dino_gt, count, stats = ctx.saved_tensors
        grad_p, bwd_sec = CudaFeatsCosinelossBackward(grad_output, voxel_label, occ_gt_mask_camera, d_grid_feats,
                                                      pseudo_dino_gt, count, timing=ctx.timing)
        stats[1] = bwd_sec
        return None, None, grad_p, None, None


class PyCudaFeatsCosineLoss(nn.Module):
    """Mean cosine distance between voxel features and target features over the valid voxels.

    forward(voxel_label (X,Y,Z) f32, occ_gt_mask_camera (X,Y,Z) bool, d_grid_feats (X,Y,Z,C) f32,
            pseudo_dino_gt (X,Y,Z,C) f32) -> (loss (0-dim), stats (2,) CPU float32)
    A voxel is valid when the mask is set and its label is > 0; the loss is 0 when none is.  ``stats``
    holds the forward and backward device seconds, as for the voxelizer (``timing=False`` leaves them
    0 and skips the synchronisations).  ``voxel_size`` / ``voxel_range`` are kept for signature parity;
    the loss does not use them.  Reference: CudaGaussianVoxelizer/__init__.py:84-95.
    """

    def __init__(self, voxel_size=[0.4, 0.4, 0.4], voxel_range=[-40, -40, -1, 40, 40, 5.4], timing: bool = True):
        super().__init__()
        self.voxel_size = torch.tensor(voxel_size, dtype=torch.float32, device="cuda")
        self.voxel_range = torch.tensor(voxel_range, dtype=torch.float32, device="cuda")
        self.timing = timing

    def forward(self, voxel_label, occ_gt_mask_camera, d_grid_feats, pseudo_dino_gt):
        return _CudaFeatsCosinelossFunction.apply(voxel_label, occ_gt_mask_camera, d_grid_feats, pseudo_dino_gt,
                                                  self.timing)
