"""Build recipe for the reference solution's own CUDA kernel (same-box baseline).

Compiles the reference's unchanged sources solution/cuda/kernel.cu and
solution/cuda/main.cpp, where they lie in the reference checkout, into a
Python extension module ``moe_ref_ext`` under baseline/_ref/ (git-ignored;
the built .so travels to the GPU box with the tree, the sources do not).
The flags are the reference's own (solution/cuda/main.py:11-29: -O3,
-std=c++20, --expt-relaxed-constexpr, sm_100a, the four no-half-operator
defines), with the architecture given as -gencode compute_100a/sm_100a.
This is our recipe around torch.utils.cpp_extension.load, not the
reference's import-time build (which also deletes the torch extension
cache); nothing from the reference is copied into this repository.

    python baseline/build_reference.py [path/to/reference/checkout]

``load_built()`` imports the built module (bench.py's same-box leg and the
reference-kernel test use it); it raises when the module was not built.
"""
from __future__ import annotations

import glob
import importlib.machinery
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "moe_ref_ext"
DEFAULT_REF = "/root/reference"

CUDA_FLAGS = [
    "-O3",
    "-std=c++20",
    "--expt-relaxed-constexpr",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-D__CUDA_NO_HALF_OPERATORS__",
    "-D__CUDA_NO_HALF_CONVERSIONS__",
    "-D__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-D__CUDA_NO_HALF2_OPERATORS__",
]
CXX_FLAGS = ["-O3", "-std=c++20", "-fPIC"]


def build(ref_root: str = DEFAULT_REF, verbose: bool = False) -> str:
    """Compiles the reference kernel into baseline/_ref; returns the .so path."""
    src = os.path.join(ref_root, "solution", "cuda")
    sources = [os.path.join(src, "main.cpp"), os.path.join(src, "kernel.cu")]
    for s in sources:
        if not os.path.exists(s):
            raise FileNotFoundError(f"reference source {s} not found")
    os.makedirs(OUT, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load

    load(name=NAME, sources=sources, extra_cuda_cflags=CUDA_FLAGS, extra_cflags=CXX_FLAGS,
         build_directory=OUT, verbose=verbose, is_python_module=True)
    return built_path()


def built_path() -> str | None:
    found = sorted(glob.glob(os.path.join(OUT, f"{NAME}*.so")))
    return found[0] if found else None


def load_built():
    """The built reference extension (``run(...)`` with the reference's
    signature, solution/cuda/main.py:31-54)."""
    import torch  # noqa: F401  (the extension links against torch)

    path = built_path()
    if path is None:
        raise RuntimeError(f"reference extension not built in {OUT} (run baseline/build_reference.py)")
    loader = importlib.machinery.ExtensionFileLoader(NAME, path)
    spec = importlib.util.spec_from_loader(NAME, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else DEFAULT_REF, verbose="-v" in sys.argv))
