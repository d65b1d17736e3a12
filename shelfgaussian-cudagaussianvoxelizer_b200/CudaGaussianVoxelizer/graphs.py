"""CUDA-graph replay of the splat's forward and backward, for loops whose sizes stay fixed.

The eager path (``PyCudaGaussianVoxelizer``) synchronises once per forward to read the number of
(Gaussian, tile) pairs M and sizes its buffers from it.  Training loops with a fixed number of Gaussians
see nearly the same M every step, so this module measures M (and the backward's block-pair count) once
eagerly, keeps capacities with headroom, and from then on runs the capacity-capped entry points
(``g2v_forward_prepare_capped`` + splat + backward with the capacities as pair counts): no host
synchronisation and no size-dependent allocation, so the whole forward and the whole backward are each
captured once in a CUDA graph and replayed.  This is the density-only fast path of the reference's
training use (its recorded density-only forward/backward times are dominated by host synchronisations
and launch overhead), and it works with features too.

A step that needs more pairs than the capacities sets the capacity bit of the library's device error
word; its outputs are then invalid.  ``check()`` (one synchronisation) raises in that case; call it every
few steps, or let the next synchronising library call report it.  Outputs are the module's static
buffers (overwritten by the next forward), as with ``torch.cuda.make_graphed_callables``.
"""
from __future__ import annotations

import ctypes
import math

import torch
import torch.nn as nn

from . import _C, _lib

__all__ = ["GraphedGaussianVoxelizer"]


def _cap(v: int, headroom: float) -> int:
    return int(math.ceil(v * headroom)) + 1024


class _State:
    """Static buffers and the two captured graphs for one (N, C, device)."""

    def __init__(self, size_h, range_h, n, c, dev, max_pairs, max_block_pairs):
        self.size_h, self.range_h, self.n, self.c, self.dev = size_h, range_h, n, c, dev
        self.M, self.MB = int(max_pairs), int(max_block_pairs)
        (X, Y, Z), _ = _lib.grid_shape(size_h, range_h)
        self.dims = (X, Y, Z)
        f32 = dict(dtype=torch.float32, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        self.means = torch.zeros((n, 3), **f32)
        self.opacity = torch.zeros((n,), **f32)
        self.cov = torch.zeros((n, 9), **f32)
        self.cov[:, 0] = self.cov[:, 4] = self.cov[:, 8] = 1.0
        self.feats = torch.zeros((n, c), **f32) if c > 0 else None
        self.cov_inv = torch.empty((n, 9), **f32)
        self.lb = torch.empty((n, 3), **i32)
        self.ub = torch.empty((n, 3), **i32)
        self.nvox = torch.empty((n,), **i32)
        self.g2t_offsets = torch.empty((n + 1,), **i32)
        self.g2t_tile_ids = torch.empty((max(self.M, 1),), **i32)
        self.density = torch.empty((X, Y, Z), **f32)
        self.grid_feats = torch.empty((X, Y, Z, c), **f32)
        self.gD = torch.zeros((X, Y, Z), **f32)
        self.gF = torch.zeros((X, Y, Z, c), **f32) if c > 0 else None
        self.g_means = torch.empty((n, 3), **f32)
        self.g_cov = torch.empty((n, 9), **f32)
        self.g_op = torch.empty((n,), **f32)
        self.g_feat = torch.empty((n, c), **f32)
        lib = _lib.load()
        nb = ctypes.c_size_t()
        _lib.check(lib.g2v_forward_prepare_workspace_size(n, ctypes.byref(nb)), "g2v_forward_prepare_workspace_size")
        self.ws1 = _C._workspace(nb.value, dev)
        _lib.check(lib.g2v_forward_splat_workspace_size(n, self.M, _lib.i3(self.dims), c, ctypes.byref(nb)),
                   "g2v_forward_splat_workspace_size")
        self.ws2 = _C._workspace(nb.value, dev)
        _lib.check(lib.g2v_backward_workspace_size(n, self.M, self.MB, _lib.i3(self.dims), c, ctypes.byref(nb)),
                   "g2v_backward_workspace_size")
        self.ws3 = _C._workspace(nb.value, dev)
        self.fwd_graph = None
        self.bwd_graph = None

    # the two launch sequences (recorded into the graphs)
    def run_forward(self):
        lib, P = _lib.load(), _C._ptr
        sptr = ctypes.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)
        n, c = self.n, self.c
        _lib.check(lib.g2v_forward_prepare_capped(P(self.means), P(self.cov), n, _lib.f3(self.size_h),
                                                  _lib.f6(self.range_h), self.M, P(self.cov_inv), P(self.lb),
                                                  P(self.ub), P(self.nvox), P(self.g2t_offsets), P(self.ws1),
                                                  self.ws1.numel(), sptr), "g2v_forward_prepare_capped")
        fptr = None if self.feats is None else _C._features_ptr(self.feats, self.density)
        _lib.check(lib.g2v_forward_splat(P(self.means), P(self.opacity), fptr, n, c, _lib.f3(self.size_h),
                                         _lib.f6(self.range_h), P(self.cov_inv), P(self.lb), P(self.ub),
                                         P(self.g2t_offsets), self.M, P(self.g2t_tile_ids), P(self.density),
                                         P(self.grid_feats), 0, 0, P(self.ws2), self.ws2.numel(), sptr),
                   "g2v_forward_splat")

    def run_backward(self):
        lib, P = _lib.load(), _C._ptr
        sptr = ctypes.c_void_p(torch.cuda.current_stream(self.dev).cuda_stream)
        n, c = self.n, self.c
        fptr = None if self.feats is None else _C._features_ptr(self.feats, self.g_op)
        _lib.check(lib.g2v_backward(P(self.gD), P(self.gF) if c > 0 else None, P(self.means), P(self.opacity),
                                    P(self.cov_inv), fptr, n, c, _lib.f3(self.size_h), _lib.f6(self.range_h),
                                    _lib.i3(self.dims), P(self.lb), P(self.ub), P(self.g2t_offsets),
                                    P(self.g2t_tile_ids), self.M, self.MB if c > 0 else 0, P(self.density),
                                    P(self.grid_feats), P(self.g_means), P(self.g_cov), P(self.g_op),
                                    P(self.g_feat), 0, 0, P(self.ws3), self.ws3.numel(), sptr), "g2v_backward")

    def capture(self):
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):  # eager warm-up: loads every kernel before capture
            self.run_forward()
            self.run_backward()
        torch.cuda.current_stream(self.dev).wait_stream(side)
        torch.cuda.synchronize(self.dev)
        self.fwd_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.fwd_graph, capture_error_mode="relaxed"):
            self.run_forward()
        self.bwd_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.bwd_graph, capture_error_mode="relaxed"):
            self.run_backward()


class _GraphedVoxelizeFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, state, means3D, opacity, covariances, features):
        state.means.copy_(means3D)
        state.opacity.copy_(opacity)
        state.cov.copy_(covariances)
        if state.feats is not None:
            state.feats.copy_(features)
        state.fwd_graph.replay()
        ctx.state = state
        ctx.has_feats = features is not None
        stats = torch.zeros(2, dtype=torch.float32, device="cpu")
        ctx.mark_non_differentiable(stats)
        return state.density.detach(), state.grid_feats.detach(), stats

    @staticmethod
    def backward(ctx, grad_density, grad_feats, grad_stats):
        st = ctx.state
        if grad_density is None:
            st.gD.zero_()
        else:
            st.gD.copy_(grad_density)
        if st.gF is not None:
            if grad_feats is None:
                st.gF.zero_()
            else:
                st.gF.copy_(grad_feats)
        st.bwd_graph.replay()
        gf = st.g_feat.clone() if ctx.has_feats else None
        return None, st.g_means.clone(), st.g_op.clone(), st.g_cov.clone(), gf


class GraphedGaussianVoxelizer(nn.Module):
    """``PyCudaGaussianVoxelizer`` whose forward and backward replay CUDA graphs.

    Same call and outputs: ``forward(means3D (N,3), opacity (N,), covariances (N,9), features (N,C) or
    None) -> (density, grid_feats, stats)``; gradients flow to all four inputs.  The first call with a
    given (N, C, device) runs the eager path once to measure the pair counts, sets the capacities to
    ``headroom`` x those (+1024) unless ``max_pairs`` / ``max_block_pairs`` are given, and captures the
    graphs; later calls copy the inputs into static buffers and replay.  ``stats`` stays zero (timing
    events are not recorded inside graphs).
    """

    def __init__(self, voxel_size=[0.4, 0.4, 0.4], voxel_range=[-40, -40, -1, 40, 40, 5.4], headroom: float = 1.25,
                 max_pairs: int | None = None, max_block_pairs: int | None = None):
        super().__init__()
        self.voxel_size = torch.tensor(voxel_size, dtype=torch.float32, device="cuda")
        self.voxel_range = torch.tensor(voxel_range, dtype=torch.float32, device="cuda")
        self.size_h = _C._host_values(self.voxel_size, 3, "voxel_size")
        self.range_h = _C._host_values(self.voxel_range, 6, "voxel_range")
        self.headroom = float(headroom)
        self.max_pairs, self.max_block_pairs = max_pairs, max_block_pairs
        self._state = None

    def _build(self, means3D, opacity, covariances, features):
        n = int(means3D.shape[0])
        c = 0 if features is None else int(features.shape[1])
        dev = means3D.device
        M, MB = self.max_pairs, self.max_block_pairs
        if M is None or (c > 0 and MB is None):
            with torch.no_grad():
                out, mb = _C._forward_impl(means3D.detach(), opacity.detach(), covariances.detach(), self.size_h,
                                           self.range_h, None if features is None else features.detach(), False,
                                           plan=True)
            if M is None:
                M = _cap(int(out[7].numel()), self.headroom)
            if MB is None:
                MB = _cap(int(mb), self.headroom) if c > 0 else 0
        st = _State(self.size_h, self.range_h, n, c, dev, M, MB or 0)
        st.means.copy_(means3D.detach())
        st.opacity.copy_(opacity.detach())
        st.cov.copy_(covariances.detach())
        if st.feats is not None:
            st.feats.copy_(features.detach())
        st.capture()
        self._state = st

    def forward(self, means3D, opacity, covariances, features=None):
        st = self._state
        c = 0 if features is None else int(features.shape[1])
        if (st is None or st.n != means3D.shape[0] or st.c != c or st.dev != means3D.device or
                (st.feats is None) != (features is None)):
            self._build(means3D, opacity, covariances, features)
        return _GraphedVoxelizeFunction.apply(self._state, means3D, opacity, covariances, features)

    def check(self):
        """Synchronise and raise RuntimeError if a replay exceeded the capacities (or a bounded wait gave up)."""
        lib = _lib.load()
        word = ctypes.c_int(0)
        sptr = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        _lib.check(lib.g2v_device_error(sptr, ctypes.byref(word)), "g2v_device_error")
        if word.value:
            raise RuntimeError(f"GraphedGaussianVoxelizer: device error word 0x{word.value:x} "
                               "(8 = pair capacity exceeded; rebuild with larger max_pairs / max_block_pairs)")

    @property
    def capacities(self):
        return None if self._state is None else (self._state.M, self._state.MB)
