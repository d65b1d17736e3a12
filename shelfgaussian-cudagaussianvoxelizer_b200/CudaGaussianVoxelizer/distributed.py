"""One scene split across ranks (one process per GPU): x-slabs of tiles, one all-reduce of the gradients.

The tile grid is cut along x into contiguous slabs, one per rank.  Every rank holds all Gaussians (the
per-Gaussian preparation is replicated), splats only its slab into slab-local ``density`` (rows, Y, Z) and
``grid_feats`` (rows, Y, Z, C) arrays -- the slabs' outputs are disjoint, so the forward needs no
communication -- and in the backward computes the per-Gaussian gradient contributions of its slab's
voxels.  One sum all-reduce of the packed [N x (3 + 9 + 1 + C)] gradient buffer (NCCL over NVLink on
GPUs; any backend torch.distributed offers) gives every rank the whole-scene gradients.

This is the multi-device form of the reference's single-device call (CudaGaussianVoxelizer/__init__.py:
69-82); on one rank it computes exactly what ``PyCudaGaussianVoxelizer`` computes.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist
import torch.nn as nn

from . import _C, _lib

__all__ = ["slab_tiles", "slab_voxel_rows", "balanced_slab_bounds", "tile_pairs_per_column", "pack_grads",
           "unpack_grads", "allreduce_grads", "slab_forward", "slab_backward", "SlabGaussianVoxelizer"]


def slab_tiles(tiles_x: int, rank: int, world: int) -> tuple[int, int]:
    """Tile x range [b, e) of `rank`'s slab: contiguous, disjoint, covering [0, tiles_x), sizes differing
    by at most one tile (the first tiles_x % world ranks take one more)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    q, r = divmod(tiles_x, world)
    b = rank * q + min(rank, r)
    return b, b + q + (1 if rank < r else 0)


def balanced_slab_bounds(column_work, world: int) -> list[int]:
    """Slab boundaries [0 = b_0 < b_1 < ... < b_world = len(column_work)] over the tile x columns that split
    the work per column (the (Gaussian, tile) pairs of each column, tile_pairs_per_column) as evenly as
    contiguous slabs can: b_r is the column boundary whose running work is nearest r / world of the total,
    kept strictly increasing so that every slab has at least one column.  Plain host arithmetic on the
    given list, so every rank that passes the same counts gets the same slabs.  With equal work per column
    the slab sizes differ by at most one column."""
    work = [max(0, int(w)) for w in column_work]
    tiles_x = len(work)
    if world < 1 or tiles_x < world:
        raise ValueError(f"{tiles_x} tile columns cannot be split into {world} non-empty slabs")
    prefix = [0]
    for w in work:
        prefix.append(prefix[-1] + w)
    total = prefix[-1]
    if total == 0:
        return [slab_tiles(tiles_x, r, world)[0] for r in range(world)] + [tiles_x]
    bounds = [0]
    k = 0
    for r in range(1, world):
        target = total * r / world
        lo, hi = bounds[-1] + 1, tiles_x - (world - r)  # leave a column for each slab still to come
        k = max(k, lo)
        while k < hi and prefix[k + 1] <= target:
            k += 1
        if k < hi and abs(prefix[k + 1] - target) < abs(prefix[k] - target):
            k += 1
        bounds.append(min(max(k, lo), hi))
    bounds.append(tiles_x)
    return bounds


def tile_pairs_per_column(means3D, covariances, voxel_size, voxel_range) -> list[int]:
    """(Gaussian, tile) pairs of the scene per tile x column: the library's boxes (g2v_forward_prepare_plan
    on the Gaussians' device) and one read back to the host.  The same inputs give the same counts on every
    rank, so balanced_slab_bounds of them needs no communication."""
    lib = _lib.load()
    size_h = _C._host_values(voxel_size, 3, "voxel_size")
    range_h = _C._host_values(voxel_range, 6, "voxel_range")
    _C._need(means3D, "means3D", dim=2)
    dev = means3D.device
    n = means3D.shape[0]
    (X, _, _), tiles = _lib.grid_shape(size_h, range_h)
    if n == 0:
        return [0] * tiles[0]
    means3D, covariances = means3D.contiguous(), covariances.contiguous()
    i32 = dict(dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        sptr = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        cov_inv = torch.empty((n, 9), dtype=torch.float32, device=dev)
        lb = torch.empty((n, 3), **i32)
        ub = torch.empty((n, 3), **i32)
        nvox = torch.empty((n,), **i32)
        g2t_offsets = torch.empty((n + 1,), **i32)
        nbytes = ctypes.c_size_t()
        _lib.check(lib.g2v_forward_prepare_plan_workspace_size(n, ctypes.byref(nbytes)),
                   "g2v_forward_prepare_plan_workspace_size")
        ws = _C._workspace(nbytes.value, dev)
        m, mb = ctypes.c_int64(), ctypes.c_int64()
        _lib.check(lib.g2v_forward_prepare_plan(_C._ptr(means3D), _C._ptr(covariances), n, _lib.f3(size_h),
                                                _lib.f6(range_h), _C._ptr(cov_inv), _C._ptr(lb), _C._ptr(ub),
                                                _C._ptr(nvox), _C._ptr(g2t_offsets), 0, _C._ptr(ws), ws.numel(),
                                                sptr, ctypes.byref(m), ctypes.byref(mb)), "g2v_forward_prepare_plan")
        live = (ub >= lb).all(dim=1)
        tlo, thi = torch.div(lb, 4, rounding_mode="floor"), torch.div(ub, 4, rounding_mode="floor")
        per = ((thi[:, 1] - tlo[:, 1] + 1) * (thi[:, 2] - tlo[:, 2] + 1)).to(torch.int64) * live.to(torch.int64)
        diff = torch.zeros(tiles[0] + 1, dtype=torch.int64, device=dev)
        diff.index_add_(0, tlo[:, 0].to(torch.int64).clamp(0, tiles[0]), per)
        diff.index_add_(0, (thi[:, 0].to(torch.int64) + 1).clamp(0, tiles[0]), -per)
        return torch.cumsum(diff, 0)[:tiles[0]].tolist()


def slab_voxel_rows(dims_x: int, tile_range: tuple[int, int]) -> tuple[int, int]:
    """Voxel x rows [x0, x1) held by the slab-local arrays of the tile x range."""
    return min(tile_range[0] * 4, dims_x), min(tile_range[1] * 4, dims_x)


def pack_grads(grad_means, grad_cov, grad_opacity, grad_features) -> torch.Tensor:
    """One contiguous (N, 13 + C) float32 buffer: means (3) | covariances (9) | opacity (1) | features (C)."""
    n = grad_means.shape[0]
    parts = [grad_means.reshape(n, 3), grad_cov.reshape(n, 9), grad_opacity.reshape(n, 1)]
    if grad_features is not None and grad_features.numel() > 0:
        parts.append(grad_features.reshape(n, -1))
    return torch.cat(parts, dim=1).contiguous()


def unpack_grads(buf: torch.Tensor, c: int):
    """Inverse of pack_grads: (grad_means (N,3), grad_cov (N,9), grad_opacity (N,), grad_features (N,C))."""
    n = buf.shape[0]
    if buf.shape[1] != 13 + c:
        raise ValueError(f"packed gradient buffer has {buf.shape[1]} columns, expected {13 + c}")
    return (buf[:, 0:3].contiguous(), buf[:, 3:12].contiguous(), buf[:, 12].contiguous(),
            buf[:, 13:13 + c].contiguous().reshape(n, c))


# Optional timing of the all-reduce: when `allreduce_events` is a list, allreduce_grads appends a pair of
# CUDA events recorded on the current stream around each all-reduce (a benchmark reads the elapsed times).
allreduce_events = None


def allreduce_grads(grad_means, grad_cov, grad_opacity, grad_features, group=None):
    """Sum the slab-partial gradients of all ranks with one all-reduce of the packed buffer."""
    c = 0 if grad_features is None else int(grad_features.reshape(grad_means.shape[0], -1).shape[1])
    buf = pack_grads(grad_means, grad_cov, grad_opacity, grad_features)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        ev = None
        if allreduce_events is not None and buf.is_cuda:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
        if ev is not None:
            ev[1].record()
            allreduce_events.append(ev)
    return unpack_grads(buf, c)


def _check_inputs(means3D, opacity, covariances, features):
    _C._need(means3D, "means3D", dim=2)
    dev = means3D.device
    _C._need(opacity, "opacity", dim=1, device=dev)
    _C._need(covariances, "covariances", dim=2, device=dev)
    n = means3D.shape[0]
    if means3D.shape[1] != 3 or covariances.shape != (n, 9) or opacity.shape[0] != n:
        raise RuntimeError("expected means3D (N,3), opacity (N,), covariances (N,9)")
    if features is not None:
        _C._need(features, "features", dim=2, device=dev)
        if features.shape[0] != n:
            raise RuntimeError(f"features must have {n} rows, got {features.shape[0]}")
    return dev, n


def slab_forward(means3D, opacity, covariances, voxel_size, voxel_range, features, tile_range):
    """Preparation of all Gaussians plus the splat of the tile x range `tile_range` into slab-local arrays.

    Returns ``(density (rows,Y,Z), grid_feats (rows,Y,Z,C), state)``; `state` holds what slab_backward needs
    (cov_inv, lb, ub, num_voxels, g2t_offsets, g2t_tile_ids, the block-pair count and the grid dims).
    """
    lib = _lib.load()
    size_h = _C._host_values(voxel_size, 3, "voxel_size")
    range_h = _C._host_values(voxel_range, 6, "voxel_range")
    dev, n = _check_inputs(means3D, opacity, covariances, features)
    means3D, opacity, covariances = means3D.contiguous(), opacity.contiguous(), covariances.contiguous()
    if features is not None:
        features = features.contiguous()
    c = 0 if features is None else int(features.shape[1])
    (X, Y, Z), _ = _lib.grid_shape(size_h, range_h)
    tb, te = int(tile_range[0]), int(tile_range[1])
    x0, x1 = slab_voxel_rows(X, (tb, te))
    i32 = dict(dtype=torch.int32, device=dev)
    f32 = dict(dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        sptr = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        cov_inv = torch.empty((n, 9), **f32)
        lb = torch.empty((n, 3), **i32)
        ub = torch.empty((n, 3), **i32)
        nvox = torch.empty((n,), **i32)
        g2t_offsets = torch.empty((n + 1,), **i32)
        nbytes = ctypes.c_size_t()
        _lib.check(lib.g2v_forward_prepare_plan_workspace_size(n, ctypes.byref(nbytes)),
                   "g2v_forward_prepare_plan_workspace_size")
        ws1 = _C._workspace(nbytes.value, dev)
        m, mb = ctypes.c_int64(), ctypes.c_int64()
        _lib.check(lib.g2v_forward_prepare_plan(_C._ptr(means3D), _C._ptr(covariances), n, _lib.f3(size_h),
                                                _lib.f6(range_h), _C._ptr(cov_inv), _C._ptr(lb), _C._ptr(ub),
                                                _C._ptr(nvox), _C._ptr(g2t_offsets), c, _C._ptr(ws1), ws1.numel(),
                                                sptr, ctypes.byref(m), ctypes.byref(mb)), "g2v_forward_prepare_plan")
        m, mb = int(m.value), int(mb.value)
        g2t_tile_ids = torch.empty((m,), **i32)
        density = torch.empty((x1 - x0, Y, Z), **f32)
        grid_feats = torch.empty((x1 - x0, Y, Z, c), **f32)
        _lib.check(lib.g2v_forward_splat_workspace_size(n, m, _lib.i3((X, Y, Z)), c, ctypes.byref(nbytes)),
                   "g2v_forward_splat_workspace_size")
        ws2 = _C._workspace(nbytes.value, dev)
        _lib.check(lib.g2v_forward_splat_local(_C._ptr(means3D), _C._ptr(opacity), _C._features_ptr(features, density),
                                               n, c, _lib.f3(size_h), _lib.f6(range_h), _C._ptr(cov_inv),
                                               _C._ptr(lb), _C._ptr(ub), _C._ptr(g2t_offsets), m,
                                               _C._ptr(g2t_tile_ids), _C._ptr(density), _C._ptr(grid_feats), tb, te,
                                               _C._ptr(ws2), ws2.numel(), sptr), "g2v_forward_splat_local")
    state = (cov_inv, lb, ub, nvox, g2t_offsets, g2t_tile_ids, mb, (X, Y, Z))
    return density, grid_feats, state


def slab_backward(grad_density, grad_grid_feats, means3D, opacity, features, voxel_size, voxel_range, density,
                  grid_feats, state, tile_range):
    """The slab's partial per-Gaussian gradients (grad_means (N,3), grad_cov (N,9), grad_opacity (N,),
    grad_features (N,C)); slab-local volume arrays as returned by slab_forward."""
    lib = _lib.load()
    cov_inv, lb, ub, nvox, g2t_offsets, g2t_tile_ids, mb, dims = state
    size_h = _C._host_values(voxel_size, 3, "voxel_size")
    range_h = _C._host_values(voxel_range, 6, "voxel_range")
    dev = means3D.device
    n = means3D.shape[0]
    c = 0 if features is None else int(features.shape[1])
    tb, te = int(tile_range[0]), int(tile_range[1])
    x0, x1 = slab_voxel_rows(dims[0], (tb, te))
    rows = (x1 - x0, dims[1], dims[2])
    grad_density = grad_density.to(torch.float32).contiguous()
    if tuple(grad_density.shape) != rows or tuple(density.shape) != rows:
        raise RuntimeError(f"slab volume arrays must be {rows}")
    if c > 0:
        grad_grid_feats = grad_grid_feats.to(torch.float32).contiguous()
        if tuple(grad_grid_feats.shape) != rows + (c,):
            raise RuntimeError(f"grad_grid_feats must be {rows + (c,)}")
    m = g2t_tile_ids.numel()
    f32 = dict(dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        sptr = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        nbytes = ctypes.c_size_t()
        _lib.check(lib.g2v_backward_workspace_size(n, m, mb, _lib.i3(dims), c, ctypes.byref(nbytes)),
                   "g2v_backward_workspace_size")
        ws = _C._workspace(nbytes.value, dev)
        grad_means = torch.empty((n, 3), **f32)
        grad_cov = torch.empty((n, 9), **f32)
        grad_op = torch.empty((n,), **f32)
        grad_feats = torch.empty((n, c), **f32)
        fptr = _C._features_ptr(features, grad_op if grad_op.numel() else density)
        _lib.check(lib.g2v_backward_local(_C._ptr(grad_density), _C._ptr(grad_grid_feats) if c > 0 else None,
                                          _C._ptr(means3D), _C._ptr(opacity), _C._ptr(cov_inv), fptr, n, c,
                                          _lib.f3(size_h), _lib.f6(range_h), _lib.i3(dims), _C._ptr(lb), _C._ptr(ub),
                                          _C._ptr(g2t_offsets), _C._ptr(g2t_tile_ids), m, mb, _C._ptr(density),
                                          _C._ptr(grid_feats), _C._ptr(grad_means), _C._ptr(grad_cov),
                                          _C._ptr(grad_op), _C._ptr(grad_feats), tb, te, _C._ptr(ws), ws.numel(),
                                          sptr), "g2v_backward_local")
    return grad_means, grad_cov, grad_op, grad_feats


class _SlabVoxelizeFunction(torch.autograd.Function):
    """Autograd function of the split splat: slab-local forward, all-reduced whole-scene gradients."""

    @staticmethod
    def forward(ctx, means3D, opacity, covariances, voxel_size, voxel_range, features, tile_range, group):
        means3D, opacity, covariances = means3D.contiguous(), opacity.contiguous(), covariances.contiguous()
        if features is not None:
            features = features.contiguous()
        density, grid_feats, state = slab_forward(means3D, opacity, covariances, voxel_size, voxel_range, features,
                                                  tile_range)
        ctx.state = state
        ctx.tile_range = tile_range
        ctx.group = group
        ctx.has_features = features is not None
        ctx.save_for_backward(means3D, opacity, voxel_size, voxel_range, density, grid_feats,
                              features if features is not None else density.new_empty(0))
        return density, grid_feats

    @staticmethod
    def backward(ctx, grad_density, grad_grid_feats):
        means3D, opacity, voxel_size, voxel_range, density, grid_feats, features = ctx.saved_tensors
        if not ctx.has_features:
            features = None
        if grad_density is None:
            grad_density = torch.zeros_like(density)
        if grad_grid_feats is None:
            grad_grid_feats = torch.zeros_like(grid_feats)
        gm, gc, go, gf = slab_backward(grad_density, grad_grid_feats, means3D, opacity, features, voxel_size,
                                       voxel_range, density, grid_feats, ctx.state, ctx.tile_range)
        gm, gc, go, gf = allreduce_grads(gm, gc, go, gf, ctx.group)
        return gm, go, gc, None, None, (gf if features is not None else None), None, None


class SlabGaussianVoxelizer(nn.Module):
    """A scene split into x-slabs over the ranks of a process group (one rank per GPU).

    forward(means3D (N,3), opacity (N,), covariances (N,9), features (N,C) or None), identical on every
    rank, returns ``(density (rows,Y,Z), grid_feats (rows,Y,Z,C), (x0, x1))``: this rank's slab of the
    reference outputs, voxel x rows [x0, x1).  Gradients reaching the inputs are the whole scene's on every
    rank (one all-reduce inside backward).  With a single rank it is PyCudaGaussianVoxelizer without stats.
    The slabs hold equal numbers of tile columns unless ``tile_bounds`` (world + 1 increasing column
    boundaries from 0 to the grid's tile columns, e.g. balanced_slab_bounds of tile_pairs_per_column) gives
    them, the same list on every rank.
    """

    def __init__(self, voxel_size=[0.4, 0.4, 0.4], voxel_range=[-40, -40, -1, 40, 40, 5.4], group=None,
                 rank: int | None = None, world: int | None = None, tile_bounds=None):
        super().__init__()
        self.voxel_size = torch.tensor(voxel_size, dtype=torch.float32, device="cuda")
        self.voxel_range = torch.tensor(voxel_range, dtype=torch.float32, device="cuda")
        self.group = group
        on = dist.is_available() and dist.is_initialized()
        self.rank = rank if rank is not None else (dist.get_rank(group) if on else 0)
        self.world = world if world is not None else (dist.get_world_size(group) if on else 1)
        size_h = _C._host_values(self.voxel_size, 3, "voxel_size")
        range_h = _C._host_values(self.voxel_range, 6, "voxel_range")
        (X, _, _), tiles = _lib.grid_shape(size_h, range_h)
        if tile_bounds is None:
            self.tile_range = slab_tiles(tiles[0], self.rank, self.world)
        else:
            b = [int(v) for v in tile_bounds]
            if (len(b) != self.world + 1 or b[0] != 0 or b[-1] != tiles[0] or
                    any(e <= s for s, e in zip(b, b[1:]))):
                raise ValueError(f"tile_bounds must be {self.world + 1} increasing column boundaries from 0 to "
                                 f"{tiles[0]}, got {b}")
            self.tile_range = (b[self.rank], b[self.rank + 1])
        self.rows = slab_voxel_rows(X, self.tile_range)

    def forward(self, means3D, opacity, covariances, features=None):
        density, grid_feats = _SlabVoxelizeFunction.apply(means3D, opacity, covariances, self.voxel_size,
                                                          self.voxel_range, features, self.tile_range, self.group)
        return density, grid_feats, self.rows
