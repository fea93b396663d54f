"""Build the sm_100a shared library ``triton_fused_rmsnorm_qkv/libfqkv.so``.

Every ``csrc/*.cu`` file is compiled with nvcc for ``sm_100a`` (in parallel) and
linked into one position-independent shared object with the CUDA runtime linked
statically, so the library needs only the NVIDIA driver at run time.  The library is
built in-tree (next to the Python package that loads it).  ``csrc/fqkv_pycall.c``, the
package's CPython fast path for ``fqkv_launch``, is compiled with the host C compiler
when the Python headers are present (the package falls back to ctypes otherwise).

Usage: ``python build.py [--verbose] [--ptxas-info]``
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT_DIR = HERE / "triton_fused_rmsnorm_qkv"
LIB = OUT_DIR / "libfqkv.so"
BUILD = HERE / "_build"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fvisibility=hidden", "-I", str(INCLUDE)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put it on PATH)")


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"command failed ({res.returncode}): {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return res.stdout + res.stderr


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> Path:
    """Compile and link the library; returns its path.  Skips work when up to date."""
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    if LIB.exists() and not force:
        newest = max(p.stat().st_mtime for p in sources + headers + [Path(__file__)])
        if LIB.stat().st_mtime >= newest:
            pycall = sorted(OUT_DIR.glob("_fqkv_pycall*.so"))
            src = CSRC / "fqkv_pycall.c"
            if not pycall or (src.exists() and pycall[-1].stat().st_mtime < src.stat().st_mtime):
                build_pycall(verbose)
            return LIB
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []

    def compile_one(src: Path) -> tuple[Path, str]:
        obj = BUILD / (src.stem + ".o")
        out = _run([cc, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)], verbose)
        return obj, out

    with ThreadPoolExecutor(max_workers=min(len(sources), os.cpu_count() or 4)) as ex:
        results = list(ex.map(compile_one, sources))
    if ptxas_info:
        for _, out in results:
            print(out)
    tmp = LIB.with_suffix(".so.tmp")
    _run([cc, *ARCH, "-shared", "-rdc=true", "-cudart", "static", "-o", str(tmp), *[str(o) for o, _ in results]], verbose)
    os.replace(tmp, LIB)
    build_pycall(verbose)
    return LIB


def build_pycall(verbose: bool = False) -> Path | None:
    """Compile the CPython fast path (``_fqkv_pycall``) next to the package, or return None
    when the host compiler or the Python headers are missing."""
    src = CSRC / "fqkv_pycall.c"
    include = sysconfig.get_paths().get("include", "")
    cc = shutil.which(os.environ.get("CC", "gcc")) or shutil.which("cc")
    if not src.exists() or not cc or not (Path(include) / "Python.h").exists():
        return None
    dst = OUT_DIR / ("_fqkv_pycall" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))
    tmp = dst.with_name(dst.name + ".tmp")
    _run([cc, "-O2", "-shared", "-fPIC", "-I", include, str(src), "-o", str(tmp)], verbose)
    os.replace(tmp, dst)
    return dst


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / smem per kernel")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, ptxas_info=a.ptxas_info, force=a.force or a.ptxas_info))
    return 0


if __name__ == "__main__":
    sys.exit(main())
