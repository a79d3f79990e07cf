"""Build recipe for the test-only checkers.

  * oracle/lib/libmle_oracle.so -- the C restatement (mle_oracle.c), gcc + OpenMP.
  * oracle/_ref/libmle_ref.so   -- the reference's own Engine/kernels.cu compiled
    from the ML_Engine source tree together with ref_harness.cu (nvcc, sm_100a).
  * oracle/_ref/librefstep.so  -- the reference's whole runtime (engine, kernels,
    debug, transformer) with ref_step.cu: the reference's own training step.
    Built only where the reference tree is present; the binary then travels with
    the repository snapshot (it is git-ignored, not copied into history).

The reference tree is located through $MLE_REFERENCE_DIR, else through the
`reference_path` key of BASELINE.json at the repository root.  None of the
reference's sources are copied: nvcc reads them where they lie and writes
objects only under oracle/_ref/.
"""
from __future__ import annotations

import json
import os
import shutil
import subprocess
from pathlib import Path

ORACLE = Path(__file__).resolve().parent
ROOT = ORACLE.parent
LIBDIR = ORACLE / "lib"
REFDIR = ORACLE / "_ref"


def reference_dir() -> Path | None:
    cand = os.environ.get("MLE_REFERENCE_DIR")
    if not cand:
        try:
            cand = json.loads((ROOT / "BASELINE.json").read_text()).get("reference_path")
        except (OSError, ValueError):
            cand = None
    if cand and (Path(cand) / "Engine" / "kernels.cu").exists():
        return Path(cand)
    return None


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(map(str, cmd))}\n{r.stdout}\n{r.stderr}")


def _export_only(prefix: str, name: str) -> list[str]:
    """Linker flags that export only the C entry points starting with
    `prefix`: every other symbol (the reference's C++ API, whose names equal
    the ones libmle_engine.so defines on purpose) becomes local, so neither
    library's calls can bind to the other's definitions when both are loaded
    in one process."""
    REFDIR.mkdir(exist_ok=True)
    vs = REFDIR / f"{name}.map"
    vs.write_text("{\n  global: " + prefix + "*;\n  local: *;\n};\n")
    return ["-Xlinker", f"--version-script={vs}", "-Xlinker", "-Bsymbolic"]


def build_oracle() -> Path:
    LIBDIR.mkdir(exist_ok=True)
    out = LIBDIR / "libmle_oracle.so"
    src = ORACLE / "mle_oracle.c"
    if out.exists() and out.stat().st_mtime >= src.stat().st_mtime:
        return out
    _run([shutil.which("gcc") or "gcc", "-O2", "-fopenmp", "-shared", "-fPIC", "-std=c11", "-o", str(out), str(src),
          "-lm"])
    return out


def build_ref() -> Path | None:
    ref = reference_dir()
    out = REFDIR / "libmle_ref.so"
    if ref is None:
        return out if out.exists() else None
    REFDIR.mkdir(exist_ok=True)
    srcs = [ref / "Engine" / "kernels.cu", ORACLE / "ref_harness.cu"]
    if out.exists() and all(out.stat().st_mtime >= s.stat().st_mtime for s in srcs + [Path(__file__)]):
        return out
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    flags = ["-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC",
             f"-I{ref / 'Includes'}", "-w"]
    objs = []
    for s in srcs:
        o = REFDIR / (s.stem + ".o")
        _run([nvcc, *flags, "-c", str(s), "-o", str(o)])
        objs.append(str(o))
    _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(out), *objs,
          *_export_only("ref_", "libmle_ref")])
    return out


def build_ref_step() -> Path | None:
    """oracle/_ref/librefstep.so: the reference's own runtime (Engine/engine.cu,
    kernels.cu, debug.cu, transformer.cu, compiled from the reference tree)
    with ref_step.cu, which builds the BASELINE graphs through the
    reference's API and times its training step."""
    ref = reference_dir()
    out = REFDIR / "librefstep.so"
    if ref is None:
        return out if out.exists() else None
    REFDIR.mkdir(exist_ok=True)
    srcs = [ref / "Engine" / f"{u}.cu" for u in ("engine", "kernels", "debug", "transformer")]
    srcs.append(ORACLE / "ref_step.cu")
    if out.exists() and all(out.stat().st_mtime >= s.stat().st_mtime for s in srcs + [Path(__file__)]):
        return out
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    flags = ["-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC",
             f"-I{ref / 'Includes'}", "-w"]
    import concurrent.futures as cf
    objs = [REFDIR / f"step_{s.stem}.o" for s in srcs]
    with cf.ThreadPoolExecutor(max_workers=len(srcs)) as ex:
        for f in [ex.submit(_run, [nvcc, *flags, "-c", str(s), "-o", str(o)]) for s, o in zip(srcs, objs)]:
            f.result()
    _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(out), *map(str, objs),
          *_export_only("refstep_", "librefstep")])
    return out


def build() -> dict:
    return {"oracle": build_oracle(), "ref": build_ref(), "ref_step": build_ref_step()}


if __name__ == "__main__":
    print(build())
