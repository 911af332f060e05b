"""Compile the reference implementation, unmodified, into oracle/_ref/.

TEST INFRASTRUCTURE ONLY.  Builds the reference's own torch extension from
its sources where they lie (core/bindings.cpp, core/torch_ops.cu,
core/quantize.cu under the reference checkout) with the reference's own nvcc
flags (setup.py:27-33: -O3 --expt-relaxed-constexpr, default fmad) plus an
sm_100a target, so the GPU parity tests can run the reference kernels on a
B200.  Outputs go only to oracle/_ref/ (git-ignored; it travels to the GPU
machine with the rest of the tree).

The module is named ``memboost_ref_C`` and exposes exactly the reference's
``memboost._C`` functions (core/bindings.cpp:6-39).

Usage: python oracle/build_ref.py [REFERENCE_ROOT]
(default: $MEMBOOST_REFERENCE_DIR; reference_dir() below)
"""
from __future__ import annotations

import glob
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "memboost_ref_C"


def reference_dir() -> str | None:
    """The reference checkout this recipe reads: $MEMBOOST_REFERENCE_DIR, else
    the build container's mount point; None where neither holds core/."""
    for d in (os.environ.get("MEMBOOST_REFERENCE_DIR"), "/root/reference"):
        if d and os.path.isdir(os.path.join(d, "core")):
            return d
    return None


def built_path() -> str | None:
    hits = sorted(glob.glob(os.path.join(OUT, NAME + "*.so")))
    return hits[0] if hits else None


def build(ref_root: str | None = None, verbose: bool = False) -> str:
    ref_root = ref_root or reference_dir()
    if ref_root is None:
        raise FileNotFoundError("reference checkout not found (set MEMBOOST_REFERENCE_DIR)")
    core = os.path.join(ref_root, "core")
    srcs = [os.path.join(core, f) for f in ("bindings.cpp", "torch_ops.cu", "quantize.cu")]
    for s in srcs:
        if not os.path.exists(s):
            raise FileNotFoundError(s)
    newest_src = max(os.path.getmtime(s) for s in srcs + [os.path.abspath(__file__)])
    prev = built_path()
    if prev and os.path.getmtime(prev) >= newest_src:
        return prev
    from torch.utils import cpp_extension

    bdir = os.path.join(OUT, "build")
    os.makedirs(bdir, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    cpp_extension.load(
        name=NAME,
        sources=srcs,
        extra_include_paths=[core],
        extra_cflags=["-O3"],
        extra_cuda_cflags=["-O3", "--expt-relaxed-constexpr", "-UTTEST_QUANTIZE",
                           "-gencode=arch=compute_100a,code=sm_100a"],
        build_directory=bdir,
        verbose=verbose,
        is_python_module=True,
    )
    so = os.path.join(bdir, NAME + ".so")
    dst = os.path.join(OUT, NAME + ".so")
    shutil.copy2(so, dst)
    return dst


def load():
    """Import the compiled reference module from oracle/_ref/ (no rebuild)."""
    import importlib.util

    import torch  # noqa: F401  (the extension links against libtorch)

    path = built_path()
    if path is None:
        raise ImportError("reference extension not built (run oracle/build_ref.py)")
    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True))
