"""Build recipe for libmoe_b200.so (the C-ABI library of this package).

Compiles every CUDA source under ``csrc/`` for sm_100a only and links them
into ``libmoe_b200.so`` next to this file, so the library travels with the
source tree. A stamp file beside the library records a digest of every
source, header and compiler flag it was built from; the library is rebuilt
when it is missing or when that digest no longer matches (contents, not
modification times, so copies of the tree keep a valid build). Concurrent
builders (several processes importing the package at once) serialise on a
lock file. Run ``python build.py [-v] [-f]`` or call :func:`build`.

The package's entry module builds the library this way on import when it
is missing or stale, as the reference solution compiles its extension on
import (solution/cuda/main.py:6-29).
"""
from __future__ import annotations

import concurrent.futures as cf
import fcntl
import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIB_NAME = "libmoe_b200.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
STAMP_PATH = LIB_PATH + ".stamp"
OBJ_DIR = os.path.join(HERE, "_build")
LOCK_PATH = os.path.join(OBJ_DIR, ".build.lock")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-I" + INCLUDE,
]
LINK_LIBS = ["-lcudart_static", "-ldl", "-lrt", "-lpthread"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the MoE CUDA library cannot be built")
    return cand


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps() -> list[str]:
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    files += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    files.append(os.path.abspath(__file__))
    return sorted(files)


def source_digest() -> str:
    """SHA-256 over the names and contents of every build input and the flags."""
    h = hashlib.sha256()
    h.update(" ".join(NVCC_FLAGS[:-1] + LINK_LIBS).encode())
    for f in _deps():
        h.update(os.path.basename(f).encode() + b"\0")
        with open(f, "rb") as fh:
            h.update(fh.read())
        h.update(b"\0")
    return h.hexdigest()


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH) or not os.path.exists(STAMP_PATH):
        return True
    with open(STAMP_PATH) as f:
        return f.read().strip() != source_digest()


def _compile_and_link(verbose: bool, ptxas_info: bool) -> None:
    nvcc = _nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []

    def compile_one(src: str) -> str:
        obj = os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or ptxas_info or res.returncode != 0:
            sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}")
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = f"{LIB_PATH}.tmp{os.getpid()}"
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", tmp, *objs, *LINK_LIBS]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError("linking libmoe_b200.so failed")
    os.replace(tmp, LIB_PATH)


def build(verbose: bool = False, force: bool = False, ptxas_info: bool = False) -> str:
    """Compile csrc/*.cu for sm_100a into libmoe_b200.so when it is missing
    or stale (or always with ``force``); returns its path."""
    if not force and not ptxas_info and not needs_build():
        return LIB_PATH
    os.makedirs(OBJ_DIR, exist_ok=True)
    with open(LOCK_PATH, "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        try:
            # another process may have finished the same build meanwhile
            if force or ptxas_info or needs_build():
                digest = source_digest()
                _compile_and_link(verbose, ptxas_info)
                with open(STAMP_PATH + ".tmp", "w") as f:
                    f.write(digest + "\n")
                os.replace(STAMP_PATH + ".tmp", STAMP_PATH)
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)
    return LIB_PATH


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv, ptxas_info="--ptxas" in sys.argv)
    print(LIB_PATH)
