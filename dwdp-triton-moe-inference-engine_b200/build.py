"""Build the in-tree C-ABI library ``libdwdp_b200.so`` with nvcc for sm_100a.

Every ``csrc/*.cu`` / ``csrc/*.cpp`` file is compiled to an object (in parallel)
and linked into one shared library beside this file, so the built library
travels with the source tree. Run ``python build.py [--force]`` or call ``build()``.
"""
from __future__ import annotations

import concurrent.futures
import os
import pathlib
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
LIB_NAME = "libdwdp_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}",
          "--expt-relaxed-constexpr"] + os.environ.get("DWDP_NVCC_FLAGS", "").split()  # e.g. a diagnostic -D


def _sources() -> list[pathlib.Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def library_path() -> pathlib.Path:
    return HERE / LIB_NAME


def _stale(lib: pathlib.Path) -> bool:
    if not lib.exists():
        return True
    deps = _sources() + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max(p.stat().st_mtime for p in deps) > lib.stat().st_mtime


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    lib = library_path()
    if not force and not _stale(lib):
        return lib
    objdir = HERE / "_build"
    objdir.mkdir(exist_ok=True)

    def compile_one(src: pathlib.Path) -> pathlib.Path:
        obj = objdir / (src.name + ".o")
        cmd = [NVCC, *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
        return obj

    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        objs = list(pool.map(compile_one, _sources()))
    tmp = lib.with_suffix(".so.tmp")
    cmd = [NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
