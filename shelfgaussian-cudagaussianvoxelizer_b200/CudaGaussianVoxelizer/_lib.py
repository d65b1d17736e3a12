"""ctypes binding of libg2v.so (the C ABI declared in include/g2v.h).

The library is built in-tree by ``csrc/build.py`` (``__graft_entry__.build()`` runs it) and loaded from
this directory.  There is no fallback: if the library is missing or fails to load, importing
``CudaGaussianVoxelizer`` raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libg2v.so")

P = ctypes.c_void_p
I32 = ctypes.c_int
I64 = ctypes.c_int64
SZ = ctypes.c_size_t
F3 = ctypes.c_float * 3
F6 = ctypes.c_float * 6
I3 = ctypes.c_int * 3

# name -> (restype, argtypes); mirrors include/g2v.h
SIGNATURES = {
    "g2v_abi_version": (I32, []),
    "g2v_status_string": (ctypes.c_char_p, [I32]),
    "g2v_last_error": (ctypes.c_char_p, []),
    "g2v_grid_shape": (I32, [F3, F6, I3, I3]),
    "g2v_forward_prepare_workspace_size": (I32, [I64, ctypes.POINTER(SZ)]),
    "g2v_forward_prepare": (I32, [P, P, I64, F3, F6, P, P, P, P, P, P, SZ, P, ctypes.POINTER(I64)]),
    "g2v_forward_prepare_static": (I32, [P, P, I64, F3, F6, P, P, P, P, P, P, ctypes.POINTER(I64)]),
    "g2v_forward_prepare_capped": (I32, [P, P, I64, F3, F6, I64, P, P, P, P, P, P, SZ, P]),
    "g2v_forward_prepare_plan_workspace_size": (I32, [I64, ctypes.POINTER(SZ)]),
    "g2v_forward_prepare_plan": (I32, [P, P, I64, F3, F6, P, P, P, P, P, I64, P, SZ, P, ctypes.POINTER(I64),
                                       ctypes.POINTER(I64)]),
    "g2v_forward_prepare_plan_sr": (I32, [P, P, P, I64, F3, F6, P, P, P, P, P, I64, P, SZ, P, ctypes.POINTER(I64),
                                          ctypes.POINTER(I64)]),
    "g2v_forward_prepare_plan_batched": (I32, [P, P, P, P, P, I32, I64, F3, F6, P, P, P, P, P, I64, P, SZ, P,
                                               ctypes.POINTER(I64), ctypes.POINTER(I64)]),
    "g2v_forward_splat_batched": (I32, [I32, P, P, P, I64, I64, F3, F6, P, P, P, P, I64, P, P, P, I32, I32, P, SZ,
                                        P]),
    "g2v_backward_batched": (I32, [I32, P, P, P, P, P, P, P, P, I64, I64, F3, F6, I3, P, P, P, P, I64, I64, P, P, P,
                                   P, P, P, P, I32, I32, P, SZ, P]),
    "g2v_covariance_from_scale_rot": (I32, [P, P, I64, P, P]),
    "g2v_covariance_from_scale_rot_backward": (I32, [P, P, P, I64, P, P, P]),
    "g2v_forward_splat_workspace_size": (I32, [I64, I64, I3, I64, ctypes.POINTER(SZ)]),
    "g2v_forward_splat": (I32, [P, P, P, I64, I64, F3, F6, P, P, P, P, I64, P, P, P, I32, I32, P, SZ, P]),
    "g2v_forward_splat_local": (I32, [P, P, P, I64, I64, F3, F6, P, P, P, P, I64, P, P, P, I32, I32, P, SZ, P]),
    "g2v_backward_local": (I32, [P, P, P, P, P, P, I64, I64, F3, F6, I3, P, P, P, P, I64, I64, P, P, P, P, P, P, I32,
                                 I32, P, SZ, P]),
    "g2v_backward_sr": (I32, [P, P, P, P, P, P, P, P, I64, I64, F3, F6, I3, P, P, P, P, I64, I64, P, P, P, P, P, P,
                              P, I32, I32, P, SZ, P]),
    "g2v_backward_units": (I32, [P, P, P, P, P, P, I64, I64, F3, F6, I3, P, P, P, P, I64, I64, P, P, P, P, P, P, P,
                                 P, P, SZ, P]),
    "g2v_forward_splat_unit_lists": (I32, [P, I64, I64, I3, I64, P, P, ctypes.POINTER(I64), P]),
    "g2v_backward_plan": (I32, [P, P, I64, I3, I64, P, SZ, P, ctypes.POINTER(I64)]),
    "g2v_backward_plan_workspace_size": (I32, [I64, ctypes.POINTER(SZ)]),
    "g2v_backward_workspace_size": (I32, [I64, I64, I64, I3, I64, ctypes.POINTER(SZ)]),
    "g2v_backward": (I32, [P, P, P, P, P, P, I64, I64, F3, F6, I3, P, P, P, P, I64, I64, P, P, P, P, P, P, I32, I32,
                           P, SZ, P]),
    "g2v_cosine_loss_workspace_size": (I32, [I64, ctypes.POINTER(SZ)]),
    "g2v_cosine_loss_forward": (I32, [P, P, P, P, I64, I64, P, P, P, SZ, P]),
    "g2v_cosine_loss_backward": (I32, [P, P, I32, P, P, P, P, I64, I64, P, P]),
    "g2v_build_t2g_workspace_size": (I32, [I64, I64, I3, ctypes.POINTER(SZ)]),
    "g2v_build_t2g": (I32, [P, P, I64, F3, F6, I64, P, P, P, SZ, P]),
    "g2v_device_error": (I32, [P, ctypes.POINTER(I32)]),
    "g2v_debug_wait_timeout": (I32, [P, ctypes.POINTER(I32)]),
    "g2v_profile_enable": (I32, [I32]),
    "g2v_profile_read": (I32, [I32, ctypes.c_char_p, SZ, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(I64)]),
}

_lib = None


def load():
    """Load libg2v.so once; raise if it is missing (no silent fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libg2v.so not found at {LIB_PATH}; build it with "
                          "`python shelfgaussian-cudagaussianvoxelizer_b200/csrc/build.py` "
                          "(or __graft_entry__.build())")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.g2v_abi_version() != 1:
        raise ImportError("libg2v.so ABI version mismatch")
    _lib = lib
    return lib


class G2VError(RuntimeError):
    """A libg2v.so call failed (RuntimeError, like the reference's c10::Error / TORCH_CHECK)."""


def check(status: int, what: str) -> None:
    if status != 0:
        lib = load()
        name = lib.g2v_status_string(status).decode()
        msg = lib.g2v_last_error().decode()
        raise G2VError(f"{what} failed: {name}: {msg}")


def f3(v) -> F3:
    return F3(*[float(x) for x in v])


def f6(v) -> F6:
    return F6(*[float(x) for x in v])


def i3(v) -> I3:
    return I3(*[int(x) for x in v])


def grid_shape(voxel_size, voxel_range):
    """(dims, tiles) from the library's float32 rule."""
    lib = load()
    d, t = I3(), I3()
    check(lib.g2v_grid_shape(f3(voxel_size), f6(voxel_range), d, t), "g2v_grid_shape")
    return tuple(d), tuple(t)


def profile_enable(enabled: bool) -> None:
    """Start (clearing old records) or stop per-kernel CUDA-event timing inside the library."""
    check(load().g2v_profile_enable(1 if enabled else 0), "g2v_profile_enable")


def profile_read() -> dict:
    """{kernel name: (total milliseconds, launches)} of the launches recorded since profile_enable(True)."""
    lib = load()
    out = {}
    i = 0
    buf = ctypes.create_string_buffer(128)
    ms = ctypes.c_double()
    n = I64()
    while True:
        rc = lib.g2v_profile_read(i, buf, 128, ctypes.byref(ms), ctypes.byref(n))
        if rc == 1:
            break
        check(rc, "g2v_profile_read")
        out[buf.value.decode()] = (ms.value, int(n.value))
        i += 1
    return out
