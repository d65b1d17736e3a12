"""C-ABI checks that need no GPU: the library loads, exports what include/g2v.h declares, and its host
logic (grid rule, argument validation, workspace sizing) behaves like the reference's."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import REPO
from oracle import oracle

HEADER = os.path.join(REPO, "include", "g2v.h")


def declared_symbols():
    with open(HEADER) as fh:
        src = fh.read()
    return sorted(set(re.findall(r"^G2V_API\s+[\w\s\*]+?\b(g2v_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("g2v_forward_prepare", "g2v_forward_splat", "g2v_backward", "g2v_grid_shape"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    from CudaGaussianVoxelizer import _lib
    lib = _lib.load()
    for s in declared_symbols():
        assert hasattr(lib, s), s
    assert set(declared_symbols()) == set(_lib.SIGNATURES), "ctypes signatures out of sync with include/g2v.h"
    assert lib.g2v_abi_version() == 1


@pytest.mark.parametrize("size,rng", [
    ([0.4, 0.4, 0.4], [-40, -40, -1, 40, 40, 5.4]),
    ([0.2, 0.2, 0.2], [-40, -40, -1, 40, 40, 5.4]),
    ([0.4, 0.4, 0.4], [-8, -8, -1, 8, 8, 5.4]),
    ([0.25, 0.5, 0.375], [-3.0, -2.0, -1.5, 2.75, 2.0, 1.875]),
    ([0.3, 0.7, 0.11], [-5.0, -3.3, -0.5, 5.1, 4.4, 1.7]),
])
def test_grid_shape_matches_float32_rule(size, rng):
    from CudaGaussianVoxelizer import _lib
    dims, tiles = _lib.grid_shape(size, rng)
    odims, otiles = oracle.grid_shape(size, rng)
    assert dims == odims and tiles == otiles
    # float32 division, truncation (cu:1512-1514)
    exp = tuple(int(np.float32(np.float32(rng[3 + a]) - np.float32(rng[a])) / np.float32(size[a])) for a in range(3))
    assert dims == exp


def test_headline_grid_is_200x200x16():
    from CudaGaussianVoxelizer import _lib
    assert _lib.grid_shape([0.4] * 3, [-40, -40, -1, 40, 40, 5.4]) == ((200, 200, 16), (50, 50, 4))
    assert _lib.grid_shape([0.2] * 3, [-40, -40, -1, 40, 40, 5.4]) == ((400, 400, 32), (100, 100, 8))


def test_invalid_grid_is_an_error_not_an_exit():
    from CudaGaussianVoxelizer import _lib
    with pytest.raises(_lib.G2VError, match="INVALID_VALUE"):
        _lib.grid_shape([0.4, 0.4, 0.4], [1, 1, 1, 0, 0, 0])
    with pytest.raises(_lib.G2VError):
        _lib.grid_shape([0.0, 0.4, 0.4], [0, 0, 0, 1, 1, 1])


def test_workspace_queries_and_too_small_workspace():
    from CudaGaussianVoxelizer import _lib
    lib = _lib.load()
    nb = ctypes.c_size_t()
    assert lib.g2v_forward_prepare_workspace_size(18000, ctypes.byref(nb)) == 0 and nb.value > 18000 * 4
    assert lib.g2v_forward_splat_workspace_size(18000, 1_900_000, _lib.i3((200, 200, 16)), 1024, ctypes.byref(nb)) == 0
    assert nb.value >= 2 * 1_900_000 * 4
    assert lib.g2v_backward_workspace_size(18000, 1_900_000, 137_000, _lib.i3((200, 200, 16)), 1024,
                                           ctypes.byref(nb)) == 0
    assert nb.value >= 1_900_000 * 40 + 137_000 * 1024 * 4
    # too-small workspace is rejected before any device work (no GPU needed for this path)
    m = ctypes.c_int64()
    dummy = ctypes.c_void_p(256)
    rc = lib.g2v_forward_prepare(dummy, dummy, 10, _lib.f3([0.4] * 3), _lib.f6([-4, -4, -1, 4, 4, 2.2]), dummy, dummy,
                                 dummy, dummy, dummy, ctypes.c_void_p(256), 16, None, ctypes.byref(m))
    assert rc == 2, lib.g2v_last_error()
    assert b"workspace" in lib.g2v_last_error()
    # negative sizes are invalid
    assert lib.g2v_forward_prepare_workspace_size(-1, ctypes.byref(nb)) == 1


def test_slab_range_validation():
    from CudaGaussianVoxelizer import _lib
    lib = _lib.load()
    p = ctypes.c_void_p(256)
    rc = lib.g2v_forward_splat(p, p, None, 1, 0, _lib.f3([0.4] * 3), _lib.f6([-4, -4, -1, 4, 4, 2.2]), p, p, p, p, 0,
                               None, p, None, 3, 99, p, 1 << 20, None)
    assert rc == 1 and b"tile x range" in lib.g2v_last_error()


def test_python_api_rejects_cpu_tensors():
    import torch
    from CudaGaussianVoxelizer import _C
    m = torch.zeros(4, 3)
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.gaussian_voxelizer_forward(m, torch.zeros(4), torch.zeros(4, 9), [0.4] * 3, [-4, -4, -1, 4, 4, 2.2])
    with pytest.raises(RuntimeError, match="scalar type"):
        _C.gaussian_voxelizer_forward(m.double(), torch.zeros(4), torch.zeros(4, 9), [0.4] * 3,
                                      [-4, -4, -1, 4, 4, 2.2])


def test_geometry_cache_never_serves_a_freed_tensor():
    """Host copies of voxel_size/voxel_range are cached per live tensor object; a new tensor that reuses
    the address (or id) of a freed one must be read again."""
    import gc
    import torch
    from CudaGaussianVoxelizer import _C
    for i in range(50):
        t = torch.tensor([0.4, 0.4, 0.1 * (i + 1)])
        assert _C._host_values(t, 3, "voxel_size")[2] == pytest.approx(0.1 * (i + 1), rel=1e-6)
        del t
        gc.collect()
    t = torch.tensor([1.0, 2.0, 3.0])
    assert _C._host_values(t, 3, "voxel_size") == (1.0, 2.0, 3.0)
    t.mul_(2)  # in-place change bumps the version
    assert _C._host_values(t, 3, "voxel_size") == (2.0, 4.0, 6.0)
