"""Builds the sm_100a kernel library and the C++ host runtime in-tree.

    python -m ml_engine_b200.build          # or __graft_entry__.build()

Outputs (git-ignored, shipped with the source tree):
    ml_engine_b200/lib/libmle_kernels.so   C ABI of include/mle_kernels.h
    ml_engine_b200/lib/libmle_engine.so    C++ runtime + C ABI of include/mle_engine.h

Every CUDA translation unit is compiled with
    -gencode arch=compute_100a,code=sm_100a -lineinfo -O3
Objects go to ml_engine_b200/_build/; a unit is rebuilt when it or any header
it can see is newer than its object.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a kernels cannot be built")


def _headers(dirs):
    out = []
    for d in dirs:
        for ext in ("*.h", "*.cuh", "*.hpp"):
            out.extend(Path(d).glob(ext))
    return out


def _stale(obj: Path, src: Path, headers) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    if src.stat().st_mtime > t:
        return True
    return any(h.stat().st_mtime > t for h in headers)


def _compile(src: Path, obj: Path, includes, extra) -> None:
    cmd = [nvcc(), *NVCC_FLAGS, *[f"-I{i}" for i in includes], *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        print(f"[build] {src.name}: {r.stderr.strip()}", file=sys.stderr)


def _build_lib(name: str, sources, includes, extra_compile=(), link_libs=(), rpath_origin=False, verbose=False):
    BUILD.mkdir(exist_ok=True)
    LIB.mkdir(exist_ok=True)
    headers = _headers(includes)
    objs, jobs = [], []
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        for src in sources:
            obj = BUILD / (name + "__" + src.stem + ".o")
            objs.append(obj)
            if _stale(obj, src, headers):
                if verbose:
                    print(f"[build] nvcc {src.relative_to(ROOT)}")
                jobs.append(ex.submit(_compile, src, obj, includes, list(extra_compile)))
        for j in jobs:
            j.result()
    out = LIB / f"lib{name}.so"
    if out.exists() and not jobs and all(o.stat().st_mtime <= out.stat().st_mtime for o in objs) and \
            Path(__file__).stat().st_mtime <= out.stat().st_mtime:
        return out
    # calls inside the library bind to its own functions, whatever else the
    # process has loaded (the reference's runtime defines the same C++ names)
    cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-Xlinker", "-Bsymbolic-functions", "-o", str(out),
           *map(str, objs), *link_libs]
    if rpath_origin:
        cmd += ["-Xlinker", "-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed for {out.name}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return out


def build(verbose: bool = False) -> list[Path]:
    kdir = CSRC / "kernels"
    kernels = _build_lib("mle_kernels", sorted(kdir.glob("*.cu")), [INCLUDE, kdir], verbose=verbose)
    outs = [kernels]
    edir = CSRC / "engine"
    engine_srcs = sorted(edir.glob("*.cu"))
    if engine_srcs:
        outs.append(_build_lib("mle_engine", engine_srcs, [INCLUDE, edir], link_libs=[f"-L{LIB}", "-lmle_kernels"],
                               rpath_origin=True, verbose=verbose))
    return outs


if __name__ == "__main__":
    for p in build(verbose=True):
        print(p)
