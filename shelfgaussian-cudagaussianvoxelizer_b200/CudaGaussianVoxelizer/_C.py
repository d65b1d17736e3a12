"""Drop-in replacement of the reference's ``CudaGaussianVoxelizer._C`` functions.

Same names, argument names, argument meaning and return tuples as the reference's pybind module
(src/bindings.cpp:8-100: the voxelizer forward/backward and the feature cosine loss forward/backward),
implemented over the C ABI of libg2v.so.  Outputs are allocated from the
torch caching allocator on ``means3D.device``; the library itself never allocates: every call passes
it a workspace tensor.  Failures raise ``RuntimeError`` (never exit the process).
"""
from __future__ import annotations

import ctypes
import weakref

import torch

from . import _lib

__all__ = ["gaussian_voxelizer_forward", "gaussian_voxelizer_backward", "grid_shape", "t2g_maps",
           "CudaFeatsCosinelossForward", "CudaFeatsCosinelossBackward", "covariance_from_scale_rot",
           "covariance_from_scale_rot_backward"]

# id(tensor) -> (weakref to the tensor, its _version, host values).  The weak reference makes sure a
# hit is the same live tensor object (an address or id can be reused after a tensor is freed).
_geom_cache: dict = {}


def _host_values(t, n: int, name: str):
    """Host floats of voxel_size / voxel_range; a tensor is read back once per (object, version)."""
    if isinstance(t, torch.Tensor):
        if t.numel() != n:
            raise RuntimeError(f"{name} must have {n} elements, got {t.numel()}")
        hit = _geom_cache.get(id(t))
        if hit is not None and hit[0]() is t and hit[1] == t._version:
            return hit[2]
        v = tuple(float(x) for x in t.detach().to("cpu", torch.float32).tolist())
        if len(_geom_cache) > 256:
            for k in [k for k, e in _geom_cache.items() if e[0]() is None]:
                del _geom_cache[k]
        _geom_cache[id(t)] = (weakref.ref(t), t._version, v)
        return v
    v = tuple(float(x) for x in t)
    if len(v) != n:
        raise RuntimeError(f"{name} must have {n} elements, got {len(v)}")
    return v


def _features_ptr(features, fallback):
    """Pointer for the C ABI's features argument.  NULL selects the density-only path, so a given but
    empty tensor (whose data_ptr() is 0) is passed as a non-NULL address the library never reads."""
    if features is None:
        return None
    p = features.data_ptr()
    return ctypes.c_void_p(p if p else fallback.data_ptr())


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None and t.numel() > 0 else ctypes.c_void_p(0)


def _need(t, name, dtype=torch.float32, dim=None, device=None):
    if not isinstance(t, torch.Tensor):
        raise RuntimeError(f"{name} must be a tensor")
    if t.dtype != dtype:
        raise RuntimeError(f"expected scalar type {dtype} for {name} but found {t.dtype}")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if device is not None and t.device != device:
        raise RuntimeError(f"{name} is on {t.device}, expected {device}")
    if dim is not None and t.dim() != dim:
        raise RuntimeError(f"{name} must have {dim} dimensions, got {t.dim()}")


def _need_contig(t, name, dtype, device):
    _need(t, name, dtype, None, device)
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def grid_shape(voxel_size, voxel_range):
    """((X, Y, Z), (Tx, Ty, Tz)) with the reference's float32 rule (cu:1512-1519)."""
    return _lib.grid_shape(_host_values(voxel_size, 3, "voxel_size"), _host_values(voxel_range, 6, "voxel_range"))


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def _scale_rot_inputs(scales, rotations, n, dev):
    """(N,3) scales and (N,4) rotation quaternions, float32 contiguous on ``dev``."""
    _need(scales, "scales", dim=2, device=dev)
    _need(rotations, "rotations", dim=2, device=dev)
    if tuple(scales.shape) != (n, 3) or tuple(rotations.shape) != (n, 4):
        raise RuntimeError(f"expected scales (N,3) and rotations (N,4) for N={n}; got {tuple(scales.shape)}, "
                           f"{tuple(rotations.shape)}")
    return scales.contiguous(), rotations.contiguous()


def _scene_offsets(scene_sizes, n, dev):
    """Device int32 offsets (B+1) of ragged scene sizes (a list of ints or a 1-D integer tensor)."""
    sizes = [int(v) for v in (scene_sizes.tolist() if isinstance(scene_sizes, torch.Tensor) else scene_sizes)]
    if not sizes or any(v < 0 for v in sizes) or sum(sizes) != n:
        raise RuntimeError(f"scene_sizes must be non-negative and sum to the {n} Gaussians, got {sizes}")
    off = [0]
    for v in sizes:
        off.append(off[-1] + v)
    return torch.tensor(off, dtype=torch.int32).to(dev, non_blocking=True), len(sizes)


def _forward_impl(means3D, opacity, covariances, voxel_size, voxel_range, features, timing, keep_t2g=False,
                  plan=False, scale_rot=None, scenes=None, caps=None, keep_units=None):
    """The forward; ``scale_rot=(scales, rotations)`` replaces ``covariances`` (then ``plan`` is implied and
    the covariances are formed inside the preparation kernel).  ``scenes=(scene_offsets (B+1) device int32,
    B)``: the Gaussians are a ragged batch of B scenes, splatted in one call into (B, X, Y, Z[, C]) volumes
    (boxes and tile ids in the coordinates of the scenes stacked along x; ``plan`` implied).
    ``caps=(max_pairs, max_block_pairs)``: capacity-capped, with no host synchronisation at all (the pair
    buffers are sized by the capacities; ``plan`` implied and the returned block-pair count is the cap), so
    the call can be captured in a CUDA graph; overflow is reported through the device error word.
    ``keep_units`` (True / False, with ``plan``): a third value is returned, the splat's unit lists
    ``(unit_offsets, unit_lists)`` when True and the splat built them, else None; they are for
    ``gaussian_voxelizer_backward(units=...)``, which then skips rebuilding them."""
    lib = _lib.load()
    size_h = _host_values(voxel_size, 3, "voxel_size")
    range_h = _host_values(voxel_range, 6, "voxel_range")
    _need(means3D, "means3D", dim=2)
    dev = means3D.device
    _need(opacity, "opacity", dim=1, device=dev)
    n = means3D.shape[0]
    if scale_rot is not None:
        plan = True
        scales, rotations = _scale_rot_inputs(scale_rot[0], scale_rot[1], n, dev)
        covariances = None
    else:
        _need(covariances, "covariances", dim=2, device=dev)
    if means3D.shape[1] != 3 or opacity.shape[0] != n or (covariances is not None and covariances.shape != (n, 9)):
        raise RuntimeError(f"expected means3D (N,3), opacity (N,), covariances (N,9); got {tuple(means3D.shape)}, "
                           f"{tuple(opacity.shape)}, {None if covariances is None else tuple(covariances.shape)}")
    if features is not None:
        _need(features, "features", dim=2, device=dev)
        if features.shape[0] != n:
            raise RuntimeError(f"features must have {n} rows, got {features.shape[0]}")
        features = features.contiguous()
    c = 0 if features is None else int(features.shape[1])
    means3D, opacity = means3D.contiguous(), opacity.contiguous()
    if covariances is not None:
        covariances = covariances.contiguous()
    (X, Y, Z), _ = _lib.grid_shape(size_h, range_h)
    nsc = 1
    if scenes is not None:
        plan = True
        scene_off, nsc = scenes
        if keep_t2g:
            raise RuntimeError("t2g maps are not exposed for batched scenes")
    if caps is not None:
        plan = True
        if scenes is not None or scale_rot is not None or keep_t2g or timing:
            raise RuntimeError("capacity-capped calls take covariances, one scene and timing=False")
    XS = X * nsc  # x rows of the stacked volume arrays
    i32 = dict(dtype=torch.int32, device=dev)
    f32 = dict(dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        sptr = ctypes.c_void_p(stream.cuda_stream)
        cov_inv = torch.empty((n, 9), **f32)
        lb = torch.empty((n, 3), **i32)
        ub = torch.empty((n, 3), **i32)
        nvox = torch.empty((n,), **i32)
        g2t_offsets = torch.empty((n + 1,), **i32)
        nbytes = ctypes.c_size_t()
        if plan:
            _lib.check(lib.g2v_forward_prepare_plan_workspace_size(n, ctypes.byref(nbytes)),
                       "g2v_forward_prepare_plan_workspace_size")
        else:
            _lib.check(lib.g2v_forward_prepare_workspace_size(n, ctypes.byref(nbytes)),
                       "g2v_forward_prepare_workspace_size")
        ws1 = _workspace(nbytes.value, dev)
        if timing:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
        m = ctypes.c_int64()
        mb = ctypes.c_int64()
        if caps is not None:  # no readback: the capacities size the pair buffers
            _lib.check(lib.g2v_forward_prepare_capped(_ptr(means3D), _ptr(covariances), n, _lib.f3(size_h),
                                                      _lib.f6(range_h), int(caps[0]), _ptr(cov_inv), _ptr(lb),
                                                      _ptr(ub), _ptr(nvox), _ptr(g2t_offsets), _ptr(ws1),
                                                      ws1.numel(), sptr), "g2v_forward_prepare_capped")
            m.value = int(caps[0])
            mb.value = int(caps[1]) if c > 0 else 0
        elif scenes is not None:
            _lib.check(lib.g2v_forward_prepare_plan_batched(
                _ptr(means3D), _ptr(covariances) if scale_rot is None else None,
                _ptr(scales) if scale_rot is not None else None, _ptr(rotations) if scale_rot is not None else None,
                _ptr(scene_off), nsc, n, _lib.f3(size_h), _lib.f6(range_h), _ptr(cov_inv), _ptr(lb), _ptr(ub),
                _ptr(nvox), _ptr(g2t_offsets), c, _ptr(ws1), ws1.numel(), sptr, ctypes.byref(m), ctypes.byref(mb)),
                "g2v_forward_prepare_plan_batched")
        elif scale_rot is not None:  # covariances formed in the preparation kernel
            _lib.check(lib.g2v_forward_prepare_plan_sr(_ptr(means3D), _ptr(scales), _ptr(rotations), n,
                                                       _lib.f3(size_h), _lib.f6(range_h), _ptr(cov_inv), _ptr(lb),
                                                       _ptr(ub), _ptr(nvox), _ptr(g2t_offsets), c, _ptr(ws1),
                                                       ws1.numel(), sptr, ctypes.byref(m), ctypes.byref(mb)),
                       "g2v_forward_prepare_plan_sr")
        elif plan:  # prepare + the backward's block-pair count, one synchronisation
            _lib.check(lib.g2v_forward_prepare_plan(_ptr(means3D), _ptr(covariances), n, _lib.f3(size_h),
                                                    _lib.f6(range_h), _ptr(cov_inv), _ptr(lb), _ptr(ub), _ptr(nvox),
                                                    _ptr(g2t_offsets), c, _ptr(ws1), ws1.numel(), sptr,
                                                    ctypes.byref(m), ctypes.byref(mb)), "g2v_forward_prepare_plan")
        else:
            _lib.check(lib.g2v_forward_prepare(_ptr(means3D), _ptr(covariances), n, _lib.f3(size_h),
                                               _lib.f6(range_h), _ptr(cov_inv), _ptr(lb), _ptr(ub), _ptr(nvox),
                                               _ptr(g2t_offsets), _ptr(ws1), ws1.numel(), sptr, ctypes.byref(m)),
                       "g2v_forward_prepare")
        m = int(m.value)
        g2t_tile_ids = torch.empty((m,), **i32)
        vshape = (X, Y, Z) if scenes is None else (nsc, X, Y, Z)
        density = torch.empty(vshape, **f32)
        grid_feats = torch.empty(vshape + (c,), **f32)
        _lib.check(lib.g2v_forward_splat_workspace_size(n, m, _lib.i3((XS, Y, Z)), c, ctypes.byref(nbytes)),
                   "g2v_forward_splat_workspace_size")
        ws2 = _workspace(nbytes.value, dev)
        if scenes is not None:
            _lib.check(lib.g2v_forward_splat_batched(nsc, _ptr(means3D), _ptr(opacity),
                                                     _features_ptr(features, density), n, c, _lib.f3(size_h),
                                                     _lib.f6(range_h), _ptr(cov_inv), _ptr(lb), _ptr(ub),
                                                     _ptr(g2t_offsets), m, _ptr(g2t_tile_ids), _ptr(density),
                                                     _ptr(grid_feats), 0, 0, _ptr(ws2), ws2.numel(), sptr),
                       "g2v_forward_splat_batched")
        else:
            _lib.check(lib.g2v_forward_splat(_ptr(means3D), _ptr(opacity), _features_ptr(features, density),
                                             n, c, _lib.f3(size_h), _lib.f6(range_h), _ptr(cov_inv), _ptr(lb),
                                             _ptr(ub), _ptr(g2t_offsets), m, _ptr(g2t_tile_ids), _ptr(density),
                                             _ptr(grid_feats), 0, 0, _ptr(ws2), ws2.numel(), sptr),
                       "g2v_forward_splat")
        sec = 0.0
        if timing:
            ev1.record(stream)
            ev1.synchronize()
            sec = ev0.elapsed_time(ev1) / 1000.0
        out = (density, cov_inv, lb, ub, nvox, grid_feats, g2t_offsets, g2t_tile_ids, sec)
        if keep_units is not None and plan:
            units = None
            nu = ctypes.c_int64()
            if keep_units and scenes is None and caps is None and c > 0 and lib.g2v_forward_splat_unit_lists(
                    None, n, m, _lib.i3((XS, Y, Z)), c, None, None, ctypes.byref(nu), sptr) == 0:
                uoff = torch.empty((int(nu.value) + 1,), **i32)
                ulist = torch.empty((max(m, 1),), **i32)
                _lib.check(lib.g2v_forward_splat_unit_lists(_ptr(ws2), n, m, _lib.i3((XS, Y, Z)), c, _ptr(uoff),
                                                            _ptr(ulist), ctypes.byref(nu), sptr),
                           "g2v_forward_splat_unit_lists")
                units = (uoff, ulist)
            return out, int(mb.value), units
        if plan:
            return out, int(mb.value)
        if keep_t2g:
            tiles = _lib.grid_shape(size_h, range_h)[1]
            nt = tiles[0] * tiles[1] * tiles[2]
            toff = torch.empty((nt + 1,), **i32)
            t2g = torch.empty((max(m, 1),), **i32)
            tb = ctypes.c_size_t()
            _lib.check(lib.g2v_build_t2g_workspace_size(n, m, _lib.i3((X, Y, Z)), ctypes.byref(tb)),
                       "g2v_build_t2g_workspace_size")
            ws3 = _workspace(tb.value, dev)
            _lib.check(lib.g2v_build_t2g(_ptr(lb), _ptr(ub), n, _lib.f3(size_h), _lib.f6(range_h), m, _ptr(toff),
                                         _ptr(t2g), _ptr(ws3), ws3.numel(), sptr), "g2v_build_t2g")
            return out, (toff, t2g[:m])
        return out


def gaussian_voxelizer_forward(means3D, opacity, covariances, voxel_size, voxel_range, features=None, *,
                               timing: bool = True):
    """Forward of the G2V splat (reference src/bindings.cpp:8-28, cu:1484-1918).

    Returns ``(density (X,Y,Z), cov_inv (N,9), valid_voxel_lb (N,3), valid_voxel_ub (N,3),
    num_voxels_per_gaussian (N,), grid_feats (X,Y,Z,C), g2t_offsets (N+1,), g2t_tile_ids (M,), fwd_sec)``.
    ``fwd_sec`` is the device time of the call (CUDA events; 0.0 with ``timing=False``, which also
    drops the end-of-call synchronisation).
    """
    return _forward_impl(means3D, opacity, covariances, voxel_size, voxel_range, features, timing)


def t2g_maps(means3D, opacity, covariances, voxel_size, voxel_range, features=None):
    """Forward outputs plus the reference's Tile->Gaussian CSR (g2v_build_t2g on the forward's boxes):
    (outputs, (tile_offsets, t2g_gaussians))."""
    return _forward_impl(means3D, opacity, covariances, voxel_size, voxel_range, features, False, keep_t2g=True)


def backward_plan(valid_voxel_lb, valid_voxel_ub, dims, channels) -> int:
    """Number of (Gaussian, tile block) pairs of the feature-gradient pass (one synchronisation)."""
    lib = _lib.load()
    dev = valid_voxel_lb.device
    n = valid_voxel_lb.shape[0]
    nbytes = ctypes.c_size_t()
    _lib.check(lib.g2v_backward_plan_workspace_size(n, ctypes.byref(nbytes)), "g2v_backward_plan_workspace_size")
    with torch.cuda.device(dev):
        ws = _workspace(nbytes.value, dev)
        mb = ctypes.c_int64()
        sptr = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(lib.g2v_backward_plan(_ptr(valid_voxel_lb), _ptr(valid_voxel_ub), n, _lib.i3(dims), int(channels),
                                         _ptr(ws), ws.numel(), sptr, ctypes.byref(mb)), "g2v_backward_plan")
    return int(mb.value)


def gaussian_voxelizer_backward(grad_output, grad_feats_output, means3D, opacity, cov_inv, voxel_size, voxel_range,
                                valid_voxel_lb, valid_voxel_ub, num_voxels_per_gaussian, g2t_offsets, g2t_tile_ids,
                                density, grid_feats, features=None, *, timing: bool = True,
                                num_block_pairs: int | None = None, tile_x_range=None, scale_rot=None,
                                num_scenes: int = 1, units=None):
    """Backward of the G2V splat (reference src/bindings.cpp:30-64, cu:1920-2057).

    Returns ``(grad_means3D (N,3), grad_cov (N,9), grad_opacity (N,), grad_feats (N,C), bwd_sec)``;
    ``grad_feats`` is (N,0) when ``features`` is None.  Inputs must be contiguous CUDA tensors of the
    reference's dtypes (RuntimeError otherwise, like the reference's TORCH_CHECKs, cu:1941-1954).
    ``tile_x_range=(b, e)`` restricts the gradient to the voxels of tiles with x in [b, e).
    ``scale_rot=(scales (N,3), rotations (N,4))``: the Gaussians' covariances came from them; the second
    output is then the pair ``(grad_scales (N,3), grad_rotations (N,4))`` in place of grad_cov (the chain
    rule runs inside the gradient reduction).
    ``num_scenes=B``: the state of a batched forward; grad_output / density are (B, X, Y, Z) and
    grad_feats_output / grid_feats (B, X, Y, Z, C).
    ``units=(unit_offsets, unit_lists)``: the forward splat's unit lists (``_forward_impl(keep_units=True)``)
    for the same Gaussians; the tile pass then uses them instead of rebuilding them (whole grid, one scene,
    covariance inputs).
    """
    lib = _lib.load()
    dev = means3D.device
    size_h = _host_values(voxel_size, 3, "voxel_size")
    range_h = _host_values(voxel_range, 6, "voxel_range")
    for t, name, dt in ((grad_output, "grad_output", torch.float32), (means3D, "means3D", torch.float32),
                        (opacity, "opacity", torch.float32), (cov_inv, "cov_inv", torch.float32),
                        (valid_voxel_lb, "valid_voxel_lb", torch.int32), (valid_voxel_ub, "valid_voxel_ub", torch.int32),
                        (num_voxels_per_gaussian, "num_voxels_per_gaussian", torch.int32),
                        (g2t_offsets, "g2t_offsets", torch.int32), (g2t_tile_ids, "g2t_tile_ids", torch.int32),
                        (density, "density", torch.float32), (grid_feats, "grid_feats", torch.float32)):
        _need_contig(t, name, dt, dev)
    n = means3D.shape[0]
    if g2t_offsets.numel() != n + 1:
        raise RuntimeError("g2t_offsets must have N+1 entries")
    c = 0
    if features is not None:
        _need_contig(features, "features", torch.float32, dev)
        c = int(features.shape[1])
        _need_contig(grad_feats_output, "grad_feats_output", torch.float32, dev)
    vdims = tuple(int(s) for s in grad_output.shape)
    if tuple(density.shape) != vdims or len(vdims) != (3 if num_scenes == 1 else 4) or (
            num_scenes > 1 and vdims[0] != num_scenes):
        raise RuntimeError("grad_output and density must be (X,Y,Z)" if num_scenes == 1 else
                           f"grad_output and density must be ({num_scenes},X,Y,Z)")
    if c > 0 and tuple(grad_feats_output.shape) != vdims + (c,):
        raise RuntimeError(f"grad_feats_output must be {vdims + (c,)}")
    dims = vdims if num_scenes == 1 else (vdims[0] * vdims[1], vdims[2], vdims[3])  # stacked along x
    m = g2t_tile_ids.numel()
    f32 = dict(dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        sptr = ctypes.c_void_p(stream.cuda_stream)
        if num_block_pairs is None:
            num_block_pairs = backward_plan(valid_voxel_lb, valid_voxel_ub, dims, c) if c > 0 else 0
        nbytes = ctypes.c_size_t()
        _lib.check(lib.g2v_backward_workspace_size(n, m, int(num_block_pairs), _lib.i3(dims), c, ctypes.byref(nbytes)),
                   "g2v_backward_workspace_size")
        ws = _workspace(nbytes.value, dev)
        grad_means = torch.empty((n, 3), **f32)
        if scale_rot is not None:
            scales, rotations = _scale_rot_inputs(scale_rot[0], scale_rot[1], n, dev)
            grad_cov = torch.empty((n, 3), **f32)  # grad_scales
            grad_rot = torch.empty((n, 4), **f32)
        else:
            grad_cov = torch.empty((n, 9), **f32)
        grad_op = torch.empty((n,), **f32)
        grad_feats = torch.empty((n, c), **f32)
        tb, te = (0, 0) if tile_x_range is None else (int(tile_x_range[0]), int(tile_x_range[1]))
        if timing:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
        fptr = _features_ptr(features, grad_op if grad_op.numel() else density)
        if num_scenes > 1:
            sr = scale_rot is not None
            _lib.check(lib.g2v_backward_batched(
                num_scenes, _ptr(grad_output), _ptr(grad_feats_output) if c > 0 else None, _ptr(means3D),
                _ptr(opacity), _ptr(scales) if sr else None, _ptr(rotations) if sr else None, _ptr(cov_inv), fptr, n,
                c, _lib.f3(size_h), _lib.f6(range_h), _lib.i3(dims), _ptr(valid_voxel_lb), _ptr(valid_voxel_ub),
                _ptr(g2t_offsets), _ptr(g2t_tile_ids), m, int(num_block_pairs), _ptr(density), _ptr(grid_feats),
                _ptr(grad_means), _ptr(grad_cov), _ptr(grad_rot) if sr else None, _ptr(grad_op), _ptr(grad_feats),
                tb, te, _ptr(ws), ws.numel(), sptr), "g2v_backward_batched")
        elif scale_rot is not None:
            _lib.check(lib.g2v_backward_sr(_ptr(grad_output), _ptr(grad_feats_output) if c > 0 else None,
                                           _ptr(means3D), _ptr(opacity), _ptr(scales), _ptr(rotations), _ptr(cov_inv),
                                           fptr, n, c, _lib.f3(size_h), _lib.f6(range_h), _lib.i3(dims),
                                           _ptr(valid_voxel_lb), _ptr(valid_voxel_ub), _ptr(g2t_offsets),
                                           _ptr(g2t_tile_ids), m, int(num_block_pairs), _ptr(density),
                                           _ptr(grid_feats), _ptr(grad_means), _ptr(grad_cov), _ptr(grad_rot),
                                           _ptr(grad_op), _ptr(grad_feats), tb, te, _ptr(ws), ws.numel(), sptr),
                       "g2v_backward_sr")
        elif units is not None and c > 0 and tile_x_range is None:
            _lib.check(lib.g2v_backward_units(_ptr(grad_output), _ptr(grad_feats_output), _ptr(means3D), _ptr(opacity),
                                              _ptr(cov_inv), fptr, n, c, _lib.f3(size_h), _lib.f6(range_h),
                                              _lib.i3(dims), _ptr(valid_voxel_lb), _ptr(valid_voxel_ub),
                                              _ptr(g2t_offsets), _ptr(g2t_tile_ids), m, int(num_block_pairs),
                                              _ptr(density), _ptr(grid_feats), _ptr(grad_means), _ptr(grad_cov),
                                              _ptr(grad_op), _ptr(grad_feats), _ptr(units[0]), _ptr(units[1]),
                                              _ptr(ws), ws.numel(), sptr), "g2v_backward_units")
        else:
            _lib.check(lib.g2v_backward(_ptr(grad_output), _ptr(grad_feats_output) if c > 0 else None,
                                        _ptr(means3D), _ptr(opacity), _ptr(cov_inv), fptr, n, c, _lib.f3(size_h),
                                        _lib.f6(range_h), _lib.i3(dims), _ptr(valid_voxel_lb), _ptr(valid_voxel_ub),
                                        _ptr(g2t_offsets), _ptr(g2t_tile_ids), m, int(num_block_pairs),
                                        _ptr(density), _ptr(grid_feats), _ptr(grad_means), _ptr(grad_cov),
                                        _ptr(grad_op), _ptr(grad_feats), tb, te, _ptr(ws), ws.numel(), sptr),
                       "g2v_backward")
        sec = 0.0
        if timing:
            ev1.record(stream)
            ev1.synchronize()
            sec = ev0.elapsed_time(ev1) / 1000.0
    if scale_rot is not None:
        return grad_means, (grad_cov, grad_rot), grad_op, grad_feats, sec
    return grad_means, grad_cov, grad_op, grad_feats, sec


def covariance_from_scale_rot(scales, rotations):
    """Covariances R(q/|q|) diag(s)^2 R(q/|q|)^T of (..., 3) scales and (..., 4) (r, x, y, z) quaternions,
    as (..., 3, 3) -- the front end of GaussTR pipelines, get_covariance(scales, quat_to_rotmat(rotations))
    (reference test/gaussian_voxelizer.py:14-37), on the device (no autograd; see
    ``CudaGaussianVoxelizer.covariance_from_scale_rot`` for the differentiable one)."""
    lib = _lib.load()
    _need(scales, "scales")
    dev = scales.device
    _need(rotations, "rotations", device=dev)
    lead = tuple(scales.shape[:-1])
    if scales.shape[-1:] != (3,) or tuple(rotations.shape) != lead + (4,):
        raise RuntimeError(f"expected scales (...,3) and rotations (...,4); got {tuple(scales.shape)}, "
                           f"{tuple(rotations.shape)}")
    s = scales.detach().reshape(-1, 3).contiguous()
    q = rotations.detach().reshape(-1, 4).contiguous()
    n = s.shape[0]
    with torch.cuda.device(dev):
        cov = torch.empty((n, 9), dtype=torch.float32, device=dev)
        sptr = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(lib.g2v_covariance_from_scale_rot(_ptr(s), _ptr(q), n, _ptr(cov), sptr),
                   "g2v_covariance_from_scale_rot")
    return cov.reshape(lead + (3, 3))


def covariance_from_scale_rot_backward(scales, rotations, grad_covariances):
    """(grad_scales (..., 3), grad_rotations (..., 4)) from grad_covariances (..., 3, 3) or (..., 9)."""
    lib = _lib.load()
    dev = scales.device
    lead = tuple(scales.shape[:-1])
    s = scales.detach().reshape(-1, 3).contiguous()
    q = rotations.detach().reshape(-1, 4).contiguous()
    n = s.shape[0]
    _need(grad_covariances, "grad_covariances", device=dev)
    if grad_covariances.numel() != 9 * n:
        raise RuntimeError(f"grad_covariances must have {9 * n} elements, got {grad_covariances.numel()}")
    g = grad_covariances.detach().reshape(n, 9).contiguous()
    with torch.cuda.device(dev):
        gs = torch.empty((n, 3), dtype=torch.float32, device=dev)
        gq = torch.empty((n, 4), dtype=torch.float32, device=dev)
        sptr = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(lib.g2v_covariance_from_scale_rot_backward(_ptr(s), _ptr(q), _ptr(g), n, _ptr(gs), _ptr(gq), sptr),
                   "g2v_covariance_from_scale_rot_backward")
    return gs.reshape(lead + (3,)), gq.reshape(lead + (4,))


def _loss_inputs(voxel_label, occ_gt_mask_camera, d_grid_feats, pseudo_dino_gt):
    """Checks of the reference (cuda_feats_loss.cu:150-153: dtype, contiguous, CUDA) plus the shape
    agreement the reference assumes: label and mask (X,Y,Z), features and targets (X,Y,Z,C)."""
    dev = d_grid_feats.device if isinstance(d_grid_feats, torch.Tensor) else None
    _need_contig(voxel_label, "voxel_label", torch.float32, dev)
    if not isinstance(occ_gt_mask_camera, torch.Tensor) or occ_gt_mask_camera.dtype not in (torch.bool, torch.uint8):
        raise RuntimeError("occ_gt_mask_camera must be a bool tensor")
    _need_contig(occ_gt_mask_camera, "occ_gt_mask_camera", occ_gt_mask_camera.dtype, dev)
    _need_contig(d_grid_feats, "d_grid_feats", torch.float32, dev)
    _need_contig(pseudo_dino_gt, "pseudo_dino_gt", torch.float32, dev)
    if d_grid_feats.dim() != 4:
        raise RuntimeError(f"d_grid_feats must be (X,Y,Z,C), got {tuple(d_grid_feats.shape)}")
    dims = tuple(d_grid_feats.shape[:3])
    if tuple(pseudo_dino_gt.shape) != tuple(d_grid_feats.shape):
        raise RuntimeError(f"pseudo_dino_gt {tuple(pseudo_dino_gt.shape)} must match d_grid_feats "
                           f"{tuple(d_grid_feats.shape)}")
    if tuple(voxel_label.shape) != dims or tuple(occ_gt_mask_camera.shape) != dims:
        raise RuntimeError(f"voxel_label {tuple(voxel_label.shape)} and occ_gt_mask_camera "
                           f"{tuple(occ_gt_mask_camera.shape)} must be {dims}")
    return dev, dims[0] * dims[1] * dims[2], int(d_grid_feats.shape[3])


def _cosine_loss_forward_impl(voxel_label, occ_gt_mask_camera, d_grid_feats, pseudo_dino_gt, timing):
    """(loss 0-dim f32, count (1,) int32, sec) on the device; no synchronisation unless ``timing``."""
    lib = _lib.load()
    dev, nv, c = _loss_inputs(voxel_label, occ_gt_mask_camera, d_grid_feats, pseudo_dino_gt)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        sptr = ctypes.c_void_p(stream.cuda_stream)
        nbytes = ctypes.c_size_t()
        _lib.check(lib.g2v_cosine_loss_workspace_size(nv, ctypes.byref(nbytes)), "g2v_cosine_loss_workspace_size")
        ws = _workspace(nbytes.value, dev)
        loss = torch.empty((), dtype=torch.float32, device=dev)
        count = torch.empty((1,), dtype=torch.int32, device=dev)
        if timing:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
        _lib.check(lib.g2v_cosine_loss_forward(_ptr(voxel_label), _ptr(occ_gt_mask_camera), _ptr(d_grid_feats),
                                               _ptr(pseudo_dino_gt), nv, c, _ptr(loss), _ptr(count), _ptr(ws),
                                               ws.numel(), sptr), "g2v_cosine_loss_forward")
        sec = 0.0
        if timing:
            ev1.record(stream)
            ev1.synchronize()
            sec = ev0.elapsed_time(ev1) / 1000.0
    return loss, count, sec


def CudaFeatsCosinelossForward(voxel_label, occ_gt_mask_camera, d_grid_feats, pseudo_dino_gt, *,
                               timing: bool = True):
    """Mean cosine loss over the valid voxels (reference src/bindings.cpp:67-80, cuda_feats_loss.cu:146-225).

    A voxel is valid when ``occ_gt_mask_camera`` and ``voxel_label > 0``.  Returns ``(loss (0-dim f32
    CUDA tensor), num_valid_voxel (int), fwd_sec)``; the int needs one synchronisation, as in the
    reference.  ``fwd_sec`` is the device time (CUDA events; 0.0 with ``timing=False``).
    """
    loss, count, sec = _cosine_loss_forward_impl(voxel_label, occ_gt_mask_camera, d_grid_feats, pseudo_dino_gt,
                                                 timing)
    return loss, int(count.item()), sec


def CudaFeatsCosinelossBackward(grad_output, voxel_label, occ_gt_mask_camera, d_grid_feats, pseudo_dino_gt,
                                num_valid_voxel, *, timing: bool = True):
    """Gradient of the loss with respect to ``d_grid_feats`` (reference src/bindings.cpp:82-100,
    cuda_feats_loss.cu:311-366).  Returns ``(grad_p (X,Y,Z,C), bwd_sec)``; invalid voxels get 0.

    ``grad_output`` is the upstream gradient (one element; read on the device, no synchronisation when
    it is a CUDA tensor).  ``num_valid_voxel`` is the forward's count: an int as in the reference, or a
    one-element int32 CUDA tensor (the count left on the device by the autograd path).
    """
    lib = _lib.load()
    dev, nv, c = _loss_inputs(voxel_label, occ_gt_mask_camera, d_grid_feats, pseudo_dino_gt)
    if isinstance(grad_output, torch.Tensor):
        if grad_output.numel() != 1:
            raise RuntimeError(f"grad_output must have one element, got {grad_output.numel()}")
        gout = grad_output.detach().to(device=dev, dtype=torch.float32).reshape(1).contiguous()
    else:
        gout = torch.full((1,), float(grad_output), dtype=torch.float32, device=dev)
    count_dev, count_host = None, 0
    if isinstance(num_valid_voxel, torch.Tensor):
        if num_valid_voxel.numel() != 1:
            raise RuntimeError("num_valid_voxel must have one element")
        count_dev = num_valid_voxel.detach().to(device=dev, dtype=torch.int32).reshape(1).contiguous()
    else:
        count_host = int(num_valid_voxel)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        sptr = ctypes.c_void_p(stream.cuda_stream)
        grad_p = torch.empty_like(d_grid_feats)
        if timing:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
        _lib.check(lib.g2v_cosine_loss_backward(_ptr(gout), _ptr(count_dev) if count_dev is not None else None,
                                                count_host, _ptr(voxel_label), _ptr(occ_gt_mask_camera),
                                                _ptr(d_grid_feats), _ptr(pseudo_dino_gt), nv, c, _ptr(grad_p), sptr),
                   "g2v_cosine_loss_backward")
        sec = 0.0
        if timing:
            ev1.record(stream)
            ev1.synchronize()
            sec = ev0.elapsed_time(ev1) / 1000.0
    return grad_p, sec
