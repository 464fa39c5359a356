"""The solution directory builds its CUDA library from source on import.

The reference compiles its extension when its entry module is imported
(solution/cuda/main.py:6-29), and the contest accepts compiled code only when
it is compiled from source during evaluation. Here a copy of the package
without any built file is imported in a fresh process: importing ``main``
must compile libmoe_b200.so from csrc/ (nvcc cross-compiles sm_100a without
a GPU) and load it. A change to a source file must mark the build stale.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

import pytest

from conftest import PKG, ROOT


def _copy_tree(dst_root: str) -> str:
    pkg_name = os.path.basename(PKG)
    shutil.copytree(os.path.join(ROOT, "include"), os.path.join(dst_root, "include"))
    skip = shutil.ignore_patterns("*.so", "*.stamp", "_build", "__pycache__", "*.tmp*")
    shutil.copytree(PKG, os.path.join(dst_root, pkg_name), ignore=skip)
    return os.path.join(dst_root, pkg_name)


def _run(pkg: str, code: str) -> str:
    env = dict(os.environ)
    env.pop("PYTHONPATH", None)
    res = subprocess.run([sys.executable, "-c", code], cwd=pkg, env=env, capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0, res.stdout + res.stderr
    return res.stdout


@pytest.mark.skipif(shutil.which("nvcc") is None and not os.path.exists("/usr/local/cuda/bin/nvcc"),
                    reason="needs nvcc")
def test_import_builds_the_library_from_source(tmp_path):
    pkg = _copy_tree(str(tmp_path))
    lib = os.path.join(pkg, "libmoe_b200.so")
    assert not os.path.exists(lib)
    out = _run(pkg, "import sys; sys.path.insert(0, '.'); import main, moe_host; "
                    "print(moe_host.load_library()._name); print(moe_host.load_library().moe_b200_abi_version())")
    name, abi = out.split()[-2:]
    assert os.path.samefile(name, lib) and int(abi) >= 7
    assert os.path.exists(lib + ".stamp")
    # the build is current: a second import compiles nothing
    out = _run(pkg, "import sys; sys.path.insert(0, '.'); import moe_host; "
                    "print(moe_host._build_module().needs_build())")
    assert out.split()[-1] == "False"
    # a changed source makes it stale
    with open(os.path.join(pkg, "csrc", "epilogue.cu"), "a") as f:
        f.write("\n// edited\n")
    out = _run(pkg, "import sys; sys.path.insert(0, '.'); import moe_host; "
                    "print(moe_host._build_module().needs_build())")
    assert out.split()[-1] == "True"
