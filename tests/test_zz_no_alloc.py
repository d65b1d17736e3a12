"""g2v_forward_prepare_static: the forward's first stage for callers that cannot allocate device memory.

Such callers (a serving process that reserves all device memory up front and must not call cudaMalloc
later, a plugin whose host application owns every allocation) cannot pass the workspace that
g2v_forward_prepare needs; this entry point keeps its scratch in a fixed array inside the library.
The test calls it through the C ABI and checks that, on two calls in a row with different inputs
(a large scene, then a smaller one, so stale scratch from the first call would show), it returns
exactly what g2v_forward_prepare returns.  The first size (200000 Gaussians, above the 65536 counts
the one-block scan handles) takes the three-kernel scan through the block-sum region of the static
scratch; the second takes the one-block scan.  It also checks the size limit, and that a grid the
workspace entry point rejects is rejected here too.  The file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

SIZE = [0.4, 0.4, 0.4]
RANGE = [-40.0, -40.0, -1.0, 40.0, 40.0, 5.4]


def _outputs(n, dev):
    return (torch.empty((n, 9), dtype=torch.float32, device=dev), torch.empty((n, 3), dtype=torch.int32, device=dev),
            torch.empty((n, 3), dtype=torch.int32, device=dev), torch.empty((n,), dtype=torch.int32, device=dev),
            torch.empty((n + 1,), dtype=torch.int32, device=dev))


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _with_workspace(lib, _lib, means, cov, n, stream):
    outs = _outputs(n, means.device)
    nb = ctypes.c_size_t()
    _lib.check(lib.g2v_forward_prepare_workspace_size(n, ctypes.byref(nb)), "workspace size")
    ws = torch.empty(nb.value, dtype=torch.uint8, device=means.device)
    m = ctypes.c_int64()
    _lib.check(lib.g2v_forward_prepare(_p(means), _p(cov), n, _lib.f3(SIZE), _lib.f6(RANGE), *[_p(t) for t in outs],
                                       _p(ws), ws.numel(), stream, ctypes.byref(m)), "g2v_forward_prepare")
    return outs, m.value


def _static(lib, _lib, means, cov, n, stream):
    outs = _outputs(n, means.device)
    m = ctypes.c_int64()
    _lib.check(lib.g2v_forward_prepare_static(_p(means), _p(cov), n, _lib.f3(SIZE), _lib.f6(RANGE),
                                              *[_p(t) for t in outs], stream, ctypes.byref(m)),
               "g2v_forward_prepare_static")
    return outs, m.value


@pytest.mark.parametrize("sizes", [(200000, 700)])
def test_static_prepare_matches_workspace_prepare_twice(sizes):
    from CudaGaussianVoxelizer import _lib
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    for call, n in enumerate(sizes):
        m, _, c, _ = oracle.generate_inputs(n, None, RANGE, seed=40 + call, num_outside=n // 20)
        n = m.shape[0]
        means, cov = m.to(dev), c.to(dev)
        ref, m_ref = _with_workspace(lib, _lib, means, cov, n, stream)
        got, m_got = _static(lib, _lib, means, cov, n, stream)
        torch.cuda.synchronize()
        assert m_got == m_ref > 0
        for name, a, b in zip(("cov_inv", "lb", "ub", "num_voxels", "g2t_offsets"), got, ref):
            np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy(), err_msg=f"call {call}: {name}")


def test_static_prepare_rejects_oversized_input():
    from CudaGaussianVoxelizer import _lib
    lib = _lib.load()
    m = ctypes.c_int64()
    dummy = ctypes.c_void_p(256)
    n = 262144 + 1
    rc = lib.g2v_forward_prepare_static(dummy, dummy, n, _lib.f3(SIZE), _lib.f6(RANGE), dummy, dummy, dummy, dummy,
                                        dummy, None, ctypes.byref(m))
    assert rc == 3  # G2V_ERROR_SIZE_LIMIT, before any device work
    assert b"at most 262144" in lib.g2v_last_error()


def test_static_prepare_rejects_the_grids_the_workspace_path_rejects():
    """Grid limits are shared with g2v_forward_prepare: a grid of more than INT32_MAX / 2 tiles fails
    with the same status on both entry points, before any device work."""
    from CudaGaussianVoxelizer import _lib
    lib = _lib.load()
    m = ctypes.c_int64()
    dummy = ctypes.c_void_p(256)
    size, rng = [1e-3] * 3, [-500.0, -500.0, -500.0, 500.0, 500.0, 500.0]
    rc_ws = lib.g2v_forward_prepare(dummy, dummy, 10, _lib.f3(size), _lib.f6(rng), dummy, dummy, dummy, dummy,
                                    dummy, dummy, 1 << 20, None, ctypes.byref(m))
    rc_st = lib.g2v_forward_prepare_static(dummy, dummy, 10, _lib.f3(size), _lib.f6(rng), dummy, dummy, dummy,
                                           dummy, dummy, None, ctypes.byref(m))
    assert rc_ws == rc_st == 3  # G2V_ERROR_SIZE_LIMIT
    assert b"too large" in lib.g2v_last_error()
