"""Build the sm_100a kernel library libp3dcuda.so in-tree.

    python -m pixal3d.cpp_b200.build [--force] [-v]

Every .cu under csrc/ is compiled with
    nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3
into _build/*.o (parallel, incremental on source/header mtimes) and linked
into pixal3d/cpp_b200/libp3dcuda.so with a static CUDA runtime.  The C++17
host layer (host/*.cpp: the reference's include/pixal3d API on top of the
C ABI) is linked into libpixal3d_b200.so next to it.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent.parent
CSRC = PKG / "csrc"
HOST = PKG / "host"
BUILD = PKG / "_build"
LIB = PKG / "libp3dcuda.so"
HOST_LIB = PKG / "libpixal3d_b200.so"
INCLUDE = REPO / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                     "-Xptxas", "-warn-spills", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers(root: Path):
    return list(root.glob("*.cuh")) + list(root.glob("*.h")) + list(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, deps) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps])


def _run(cmd, verbose):
    if verbose:
        print(" ".join(map(str, cmd)), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(map(str, cmd))}\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr)
    return r


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    nv = nvcc()
    srcs = sorted(CSRC.glob("*.cu"))
    deps = _headers(CSRC)
    jobs = []
    objs = []
    for s in srcs:
        o = BUILD / (s.stem + ".o")
        objs.append(o)
        if force or ptxas_info or _stale(o, s, deps):
            flags = NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_info else [])
            jobs.append([nv, *flags, "-c", str(s), "-o", str(o)])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        outs = list(ex.map(lambda c: _run(c, verbose), jobs))
    if ptxas_info:
        for r in outs:
            print(r.stderr)
    if jobs or not LIB.exists():
        _run([nv, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)], verbose)
    # C++17 host layer (reference API) over the C ABI.
    hsrcs = sorted(HOST.glob("*.cpp")) if HOST.exists() else []
    if hsrcs:
        hdeps = list((HOST / "include").rglob("*.h")) + list(INCLUDE.glob("*.h"))
        if force or not HOST_LIB.exists() or any(_stale(HOST_LIB, s, hdeps) for s in hsrcs) or \
                LIB.stat().st_mtime > HOST_LIB.stat().st_mtime:
            _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-I{HOST / 'include'}", f"-I{INCLUDE}",
                  "-I/usr/local/cuda/include", *map(str, hsrcs), "-o", str(HOST_LIB),
                  f"-L{PKG}", "-lp3dcuda", "-Wl,-rpath,$ORIGIN"], verbose)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v register/spill/smem info")
    a = ap.parse_args()
    p = build(a.force, a.verbose, a.ptxas_info)
    print("built", p)


if __name__ == "__main__":
    sys.exit(main())
