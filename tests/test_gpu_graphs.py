"""GPU checks of the capacity-capped, graph-replayed path (GraphedGaussianVoxelizer).

* Outputs and gradients bit-identical to the eager PyCudaGaussianVoxelizer (the capped calls run the
  same kernels; the capacities only bound the offsets), density-only and with features, including
  replays after the inputs changed (a different number of pairs below the capacity).
* A capacity below the needed pairs is reported through the device error word (check() raises) -- the
  offsets are clamped and every CSR store and read is bounded by the capacity, so nothing is written
  or read out of bounds -- and the library's next call works normally.
* The sync-free prepare itself: g2v_forward_prepare_capped writes the same boxes / offsets as
  g2v_forward_prepare when the capacity suffices.
"""
import ctypes

import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

SIZE, RNG = [0.4] * 3, [-8.0, -8.0, -1.0, 8.0, 8.0, 5.4]


def _inputs(n, c, seed):
    m, o, cov, f = oracle.generate_inputs(n, max(c, 1), RNG, seed=seed, num_outside=4)
    return m.cuda(), o.cuda(), cov.cuda(), (f[:, :c].contiguous().cuda() if c > 0 else None)


def _fwd_bwd(vox, m, o, cov, f, seed):
    leaves = [t.clone().requires_grad_(True) for t in (m, o, cov)]
    fl = f.clone().requires_grad_(True) if f is not None else None
    density, grid_feats, _ = vox(*leaves, fl)
    gen = torch.Generator("cuda").manual_seed(seed)
    gD = torch.randn(density.shape, device="cuda", generator=gen)
    outs, ups = [density], [gD]
    if f is not None:
        outs.append(grid_feats)
        ups.append(torch.randn(grid_feats.shape, device="cuda", generator=gen))
    torch.autograd.backward(outs, ups)
    torch.cuda.synchronize()
    res = [density.detach().clone(), grid_feats.detach().clone()] + [t.grad.clone() for t in leaves]
    if fl is not None:
        res.append(fl.grad.clone())
    return res


@pytest.mark.parametrize("c", [0, 16])
def test_graph_replay_is_bit_identical_to_eager(c):
    from CudaGaussianVoxelizer import GraphedGaussianVoxelizer, PyCudaGaussianVoxelizer
    eager = PyCudaGaussianVoxelizer(voxel_size=SIZE, voxel_range=RNG)
    graphed = GraphedGaussianVoxelizer(voxel_size=SIZE, voxel_range=RNG)
    for step, seed in enumerate([1, 1, 2, 3]):  # capture, replay, then new inputs (different M)
        m, o, cov, f = _inputs(600, c, seed)
        a = _fwd_bwd(eager, m, o, cov, f, seed=10 + step)
        b = _fwd_bwd(graphed, m, o, cov, f, seed=10 + step)
        for i, (x, y) in enumerate(zip(a, b)):
            assert torch.equal(x, y), f"step {step}: output {i}"
    graphed.check()
    M, MB = graphed.capacities
    assert M > 0 and (MB > 0) == (c > 0)


def test_capacity_overflow_is_reported_not_overrun():
    from CudaGaussianVoxelizer import GraphedGaussianVoxelizer, PyCudaGaussianVoxelizer
    m, o, cov, f = _inputs(500, 8, 5)
    graphed = GraphedGaussianVoxelizer(voxel_size=SIZE, voxel_range=RNG, max_pairs=64, max_block_pairs=32)
    _fwd_bwd(graphed, m, o, cov, f, seed=3)
    with pytest.raises(RuntimeError, match="capacity"):
        graphed.check()
    graphed.check()  # the word was cleared by the read
    # the library is healthy afterwards: an eager call matches the oracle's boxes
    eager = PyCudaGaussianVoxelizer(voxel_size=SIZE, voxel_range=RNG)
    density, _, _ = eager(m, o, cov, f)
    torch.cuda.synchronize()
    assert torch.isfinite(density).all()


def test_capped_prepare_matches_prepare():
    from CudaGaussianVoxelizer import _C, _lib
    lib = _lib.load()
    m, o, cov, _ = _inputs(700, 0, 7)
    n = m.shape[0]
    ref = _C.gaussian_voxelizer_forward(m, o, cov, SIZE, RNG, None, timing=False)
    M = int(ref[7].numel())
    i32 = dict(dtype=torch.int32, device="cuda")
    cov_inv = torch.empty((n, 9), device="cuda")
    lb, ub = torch.empty((n, 3), **i32), torch.empty((n, 3), **i32)
    nvox, off = torch.empty((n,), **i32), torch.empty((n + 1,), **i32)
    nb = ctypes.c_size_t()
    _lib.check(lib.g2v_forward_prepare_workspace_size(n, ctypes.byref(nb)), "ws")
    ws = torch.empty(nb.value, dtype=torch.uint8, device="cuda")
    P = _C._ptr
    sptr = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.g2v_forward_prepare_capped(P(m), P(cov), n, _lib.f3(SIZE), _lib.f6(RNG), M + 5, P(cov_inv), P(lb),
                                              P(ub), P(nvox), P(off), P(ws), ws.numel(), sptr), "capped")
    torch.cuda.synchronize()
    for x, y in ((cov_inv, ref[1]), (lb, ref[2]), (ub, ref[3]), (nvox, ref[4]), (off, ref[6])):
        assert torch.equal(x, y)


@pytest.mark.parametrize("c", [0, 16])
def test_whole_step_capture_with_capped_module(c):
    """A training step (forward, loss, backward) through PyCudaGaussianVoxelizer(max_pairs=...) captured in
    one torch CUDA graph reproduces the eager step bit for bit, and keeps doing so for new inputs copied
    into the static tensors."""
    from CudaGaussianVoxelizer import PyCudaGaussianVoxelizer, _C
    m, o, cov, f = _inputs(500, c, 21)
    out0, mb0 = _C._forward_impl(m, o, cov, SIZE, RNG, f, False, plan=True)
    caps = (2 * int(out0[7].numel()) + 64, 2 * mb0 + 64)
    capped = PyCudaGaussianVoxelizer(voxel_size=SIZE, voxel_range=RNG, timing=False, max_pairs=caps[0],
                                     max_block_pairs=caps[1])
    eager = PyCudaGaussianVoxelizer(voxel_size=SIZE, voxel_range=RNG)
    static = [t.clone().requires_grad_(True) for t in (m, o, cov)] + ([f.clone().requires_grad_(True)] if c else [])

    def step(vox, ls):
        density, grid_feats, _ = vox(*ls[:3], ls[3] if c else None)
        loss = (density * density).sum() + (grid_feats.sum() if c else 0.0)
        return torch.autograd.grad(loss, ls)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            step(capped, static)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="relaxed"):
        out = step(capped, static)
    for seed in (21, 22):
        m, o, cov, f = _inputs(500, c, seed)
        with torch.no_grad():
            for t, v in zip(static, (m, o, cov, f)):
                t.copy_(v)
        g.replay()
        ref = step(eager, [t.detach().clone().requires_grad_(True) for t in static])
        torch.cuda.synchronize()
        for i, (x, y) in enumerate(zip(out, ref)):
            assert torch.equal(x, y), f"seed {seed}: grad {i}"
    from CudaGaussianVoxelizer import GraphedGaussianVoxelizer
    GraphedGaussianVoxelizer(voxel_size=SIZE, voxel_range=RNG).check()
