"""Build the reference's CUDA voxelizer into oracle/_ref/ -- TEST INFRASTRUCTURE ONLY.

    python oracle/build_ref.py            # needs the reference checkout: $G2V_REFERENCE_ROOT, else a "reference" folder beside the repo

Compiles the reference's src/cuda_gaussian_voxelizer.cu and src/cuda_feats_loss.cu where they lie
(nothing is copied into this repository) together with oracle/ref_bindings.cpp, with the reference's own nvcc flags
(-O3 --use_fast_math, setup.py:19-20) for sm_100a.  The reference's build system (setup.py / CMake) is
not run.  The result, oracle/_ref/g2v_reference_ext*.so, is git-ignored but travels to the GPU box,
where tests/ use it as the bit-exact pin of the CSR maps and the comparator of the feature loss, and
bench.py's reference arm may time it.
Nothing on the product path imports it.
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
# the reference checkout: $G2V_REFERENCE_ROOT, else the folder "reference" next to this repository
REF = os.environ.get("G2V_REFERENCE_ROOT") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
NAME = "g2v_reference_ext"


def build(verbose=True):
    srcs = [os.path.join(REF, "src", f) for f in ("cuda_gaussian_voxelizer.cu", "cuda_feats_loss.cu")]
    for src in srcs:
        if not os.path.exists(src):
            raise FileNotFoundError(f"reference source not found: {src}")
    os.makedirs(OUT, exist_ok=True)
    from torch.utils import cpp_extension
    return cpp_extension.load(
        name=NAME, sources=[os.path.join(HERE, "ref_bindings.cpp"), *srcs],
        extra_include_paths=[os.path.join(REF, "include")],
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=["-O3", "--use_fast_math", "-gencode", "arch=compute_100a,code=sm_100a"],
        build_directory=OUT, verbose=verbose)


_loaded = None


def load():
    """Import the prebuilt reference extension from oracle/_ref/ (no rebuild; loaded once per process)."""
    global _loaded
    if _loaded is not None:
        return _loaded
    import importlib.util
    import glob
    import torch  # noqa: F401  (the extension links libtorch)
    cands = sorted(glob.glob(os.path.join(OUT, NAME + "*.so")))
    if not cands:
        return None
    spec = importlib.util.spec_from_file_location(NAME, cands[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    _loaded = mod
    return mod


if __name__ == "__main__":
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    build(verbose="-q" not in sys.argv)
    print("built", OUT)
