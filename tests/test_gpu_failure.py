"""Failure detection without a GPU fault: a bounded wait that runs out (an mbarrier nothing arrives at)
gives up after its time limit, reports through the device error word, and the context stays usable."""
import ctypes
import time

import numpy as np
import pytest
import torch

from gpu_util import assert_close, dev
from oracle import oracle

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_context_survives():
    from CudaGaussianVoxelizer import _C, _lib
    lib = _lib.load()
    sptr = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    word = ctypes.c_int(0)
    _lib.check(lib.g2v_device_error(sptr, ctypes.byref(word)), "g2v_device_error")  # start from a clear word
    gave_up = ctypes.c_int(-1)
    t0 = time.perf_counter()
    _lib.check(lib.g2v_debug_wait_timeout(sptr, ctypes.byref(gave_up)), "g2v_debug_wait_timeout")
    elapsed = time.perf_counter() - t0
    assert gave_up.value == 1
    assert 1.0 < elapsed < 60.0, elapsed  # the limit is ~2 s of %globaltimer
    _lib.check(lib.g2v_device_error(sptr, ctypes.byref(word)), "g2v_device_error")
    assert word.value & 1, word.value  # the timeout bit
    _lib.check(lib.g2v_device_error(sptr, ctypes.byref(word)), "g2v_device_error")
    assert word.value == 0  # read-and-clear
    # the context is intact: a splat right after matches the oracle
    size, rng = [0.4] * 3, [-4.0, -4.0, -1.0, 4.0, 4.0, 2.2]
    m, o, cv, f = (t.numpy() for t in oracle.generate_inputs(200, 8, rng, seed=3))
    out = _C.gaussian_voxelizer_forward(*dev(m, o, cv), size, rng, dev(f)[0], timing=False)
    torch.cuda.synchronize()
    lb, ub = out[2].cpu().numpy(), out[3].cpu().numpy()
    dims = oracle.grid_shape(size, rng)[0]
    dref, fref = oracle.forward(m, o, cv, f, lb, ub, size, rng, dims)
    assert_close("density", out[0].cpu().numpy(), dref)
    assert_close("grid_feats", out[5].cpu().numpy(), fref)


def test_error_word_fails_the_next_synchronising_call():
    """A set word makes the next forward_prepare fail loudly (and clears it)."""
    from CudaGaussianVoxelizer import _C, _lib
    lib = _lib.load()
    sptr = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    gave_up = ctypes.c_int(-1)
    _lib.check(lib.g2v_debug_wait_timeout(sptr, ctypes.byref(gave_up)), "g2v_debug_wait_timeout")
    size, rng = [0.4] * 3, [-4.0, -4.0, -1.0, 4.0, 4.0, 2.2]
    m, o, cv, f = (t.numpy() for t in oracle.generate_inputs(50, 4, rng, seed=1))
    with pytest.raises(RuntimeError, match="bounded wait"):
        _C.gaussian_voxelizer_forward(*dev(m, o, cv), size, rng, dev(f)[0], timing=False)
    out = _C.gaussian_voxelizer_forward(*dev(m, o, cv), size, rng, dev(f)[0], timing=False)  # clear again
    assert np.isfinite(out[0].cpu().numpy()).all()
