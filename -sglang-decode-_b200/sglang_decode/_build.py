"""Build ``libsgld_sm100.so`` (the C-ABI kernel library) in-tree with nvcc.

The library holds every GPU kernel of the decode hot path, compiled for sm_100a
only.  It is written next to this file (``_lib/``) so it travels with the source
tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE.parent / "csrc"
INCLUDE = PACKAGE.parent.parent / "include"
LIB_DIR = PACKAGE / "_lib"
LIB_NAME = "libsgld_sm100.so"
OPS_NAME = "libsgld_torch_ops.so"        # torch operator library over the C ABI
OPS_SOURCE = "sgld_torch_ops.cpp"
SOURCES = ("sgld_plan.cu", "sgld_decode.cu", "sgld_decode_tc.cu", "sgld_merge.cu", "sgld_kvwrite.cu",
           "sgld_capi.cu", "sgld_noalloc.cu")
ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def library_path() -> Path:
    return LIB_DIR / LIB_NAME


def ops_library_path() -> Path:
    return LIB_DIR / OPS_NAME


def _inputs():
    files = [CSRC / s for s in SOURCES] + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    return files


def is_stale() -> bool:
    lib = library_path()
    if not lib.exists():
        return True
    built = lib.stat().st_mtime
    return any(f.stat().st_mtime > built for f in _inputs())


def ops_is_stale() -> bool:
    ops = ops_library_path()
    if not ops.exists():
        return True
    inputs = [CSRC / OPS_SOURCE, library_path()] + sorted(INCLUDE.glob("*.h"))
    return any(f.stat().st_mtime > ops.stat().st_mtime for f in inputs)


def build_ops(force: bool = False, verbose: bool = False) -> Path:
    """Compile the torch operator library (host C++ only) against torch's headers, linked to
    the C-ABI library beside it (rpath $ORIGIN)."""
    ops = ops_library_path()
    if not force and not ops_is_stale():
        return ops
    import torch
    from torch.utils import cpp_extension
    cuda_home = Path(cpp_extension.CUDA_HOME or "/usr/local/cuda")
    includes = cpp_extension.include_paths() + [str(cuda_home / "include"), str(INCLUDE)]
    cmd = [shutil.which("g++") or "g++", "-O2", "-std=c++17", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           *[f"-I{p}" for p in includes], str(CSRC / OPS_SOURCE), "-o", str(ops.with_suffix(".so.tmp")),
           f"-L{LIB_DIR}", "-lsgld_sm100", *[f"-L{p}" for p in cpp_extension.library_paths()],
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", f"-L{cuda_home / 'lib64'}", "-lcudart",
           "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed: {' '.join(cmd)}\n{res.stdout.decode(errors='replace')}")
    os.replace(ops.with_suffix(".so.tmp"), ops)
    return ops


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the CUDA sources and link the shared library (parallel nvcc jobs)."""
    lib = library_path()
    if not force and not is_stale():
        return lib
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    obj_dir = LIB_DIR / "obj"
    obj_dir.mkdir(parents=True, exist_ok=True)
    flags = [ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}",
             "--expt-relaxed-constexpr", "-diag-suppress=177"]
    procs = []
    for src in SOURCES:
        obj = obj_dir / (Path(src).stem + ".o")
        cmd = [nvcc, *flags, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    for cmd, proc in procs:
        out, _ = proc.communicate()
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{out.decode(errors='replace')}")
    tmp = lib.with_suffix(".so.tmp")
    link = [nvcc, "-shared", ARCH, "-Xlinker", f"-soname={LIB_NAME}", "-o", str(tmp),
            *[str(obj_dir / (Path(s).stem + ".o")) for s in SOURCES]]
    res = subprocess.run(link, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    if res.returncode != 0:
        raise RuntimeError(f"link failed: {' '.join(link)}\n{res.stdout.decode(errors='replace')}")
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
    print(build_ops(force="--force" in sys.argv, verbose=True))
