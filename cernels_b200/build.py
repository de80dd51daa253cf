"""Builds the in-tree shared library ``cernels_b200/_C/libcernels_b200.so`` with nvcc.

The library holds every CUDA kernel of the package (sm_100a only) behind the C ABI
declared in ``include/cernels_b200.h``. It has no torch dependency: the Python layer
binds it with ctypes. Run ``python -m cernels_b200.build`` (or ``__graft_entry__.build()``).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
OUT_DIR = PKG_DIR / "_C"
LIB_NAME = "libcernels_b200.so"
SOURCES = ["capi.cu", "route.cu", "permute.cu", "grouped_gemm.cu", "decode.cu", "capi_noalloc.cu", "router.cu", "router_gemm.cu", "ep_p2p.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build cernels_b200")
    return cand


def lib_path() -> Path:
    return OUT_DIR / LIB_NAME


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compiles every .cu under csrc/ into one shared library; returns its path."""
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh"))
    deps.append(REPO_DIR / "include" / "cernels_b200.h")
    target = lib_path()
    if not force and not _stale(target, deps):
        return target
    nvcc = nvcc_path()
    objs = []
    build_dir = OUT_DIR / "obj"
    build_dir.mkdir(exist_ok=True)
    common = [
        nvcc, *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
        "--expt-relaxed-constexpr", "-I", str(REPO_DIR / "include"),
    ]
    if ptxas_verbose:
        common += ["-Xptxas", "-v"]
    procs = []
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        objs.append(obj)
        cmd = common + ["-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if out and (verbose or ptxas_verbose or p.returncode):
            print(out, file=sys.stderr)
        if p.returncode:
            failed.append(src)
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    tmp = target.with_suffix(".so.tmp")
    link = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
    if verbose:
        print(" ".join(link), flush=True)
    subprocess.run(link, check=True)
    os.replace(tmp, target)
    return target


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv, ptxas_verbose="--ptxas" in sys.argv))
