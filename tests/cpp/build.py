"""Builds a C++ program written against the reference's engine API
(tests/cpp/*.cu) with this repository's headers and libmle_engine.so:
    python tests/cpp/build.py <source.cu> <output binary>
Used by tests/test_dropin_cpp.py."""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]


def build(src: Path, out: Path) -> None:
    sys.path.insert(0, str(ROOT))
    from ml_engine_b200 import build as b
    b.build()
    lib = ROOT / "ml_engine_b200" / "lib"
    cmd = [b.nvcc(), "-std=c++17", "-O2", "-gencode", "arch=compute_100a,code=sm_100a",
           f"-I{ROOT / 'include'}", f"-I{ROOT / 'ml_engine_b200' / 'csrc' / 'engine'}", str(src), "-o", str(out),
           f"-L{lib}", "-lmle_engine", "-lmle_kernels", "-Xlinker", f"-rpath,{lib}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


if __name__ == "__main__":
    build(Path(sys.argv[1]), Path(sys.argv[2]))
