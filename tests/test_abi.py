"""CPU checks of the drop-in boundary: the C-ABI libraries load without a GPU
and export every entry point their headers declare; the header prototypes
parse into complete ctypes signatures; the oracle agrees with numpy on the
formulas it restates."""
import ctypes
import os
from pathlib import Path

import numpy as np
import pytest

from conftest import rel_err

ROOT = Path(__file__).resolve().parents[1]


def _declared(header):
    from ml_engine_b200._lib import parse_header
    return parse_header(ROOT / "include" / header)


def test_kernel_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(ROOT / "ml_engine_b200" / "lib" / "libmle_kernels.so"))
    names = _declared("mle_kernels.h")
    assert len(names) >= 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_engine_library_exports_every_declared_symbol():
    hdr = ROOT / "include" / "mle_engine.h"
    if not hdr.exists():
        pytest.skip("engine ABI not declared yet")
    lib = ctypes.CDLL(str(ROOT / "ml_engine_b200" / "lib" / "libmle_engine.so"), mode=ctypes.RTLD_GLOBAL)
    missing = [n for n in _declared("mle_engine.h") if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_load_without_gpu():
    from ml_engine_b200 import kernels
    k = kernels()
    assert k.mle_abi_version() == 1
    assert k.dll.mle_status_string(0) == b"ok"


def test_argument_validation_needs_no_gpu():
    from ml_engine_b200 import kernels
    k = kernels()
    # invalid arguments are rejected on the host before any launch
    assert k.mle_fill(None, 0.0, 10, None) == 1
    assert k.mle_gemm(None, None, None, None, 1, 4, 4, 4, 4, 4, 4, 0, 0, 0, 0, 0, 1.0, 0.0, None) == 1
    assert k.mle_act_fwd(99, None, None, 4, None) == 1


def test_oracle_bcmm_matches_numpy(rng):
    from oracle import ops as orc
    b, c, m, n, p = 2, 3, 5, 7, 4
    A = rng.standard_normal((b, c, n, m)).astype(np.float32)   # ATB: A stored [n, m]
    B = rng.standard_normal((b, c, n, p)).astype(np.float32)
    C = np.zeros((b, c, m, p), np.float32)
    orc.bcmm(2, A, B, C, b, c, m, n, p, 0, 3, 3, 3, 2.0)
    ref = 2.0 * np.einsum("bcnm,bcnp->bcmp", A.astype(np.float64), B)
    assert rel_err(C, ref) <= 1e-6
    # everything broadcast, accumulate: the product is added b*c times
    A2 = rng.standard_normal((m, n)).astype(np.float32)
    B2 = rng.standard_normal((n, p)).astype(np.float32)
    C2 = np.zeros((m, p), np.float32)
    orc.bcmm(0, A2, B2, C2, b, c, m, n, p, 1, 0, 0, 0, 1.0)
    assert rel_err(C2, b * c * (A2.astype(np.float64) @ B2)) <= 1e-6


def test_oracle_softmax_and_layernorm_match_numpy(rng):
    from oracle import ops as orc
    x = rng.standard_normal((3, 6, 9)).astype(np.float32)
    y = orc.softmax_fwd(x, 3, 6, 9, 1)
    e = np.exp(x - x.max(axis=1, keepdims=True))
    assert rel_err(y, e / e.sum(axis=1, keepdims=True)) <= 1e-6
    z = rng.standard_normal((4, 32)).astype(np.float32)
    yn, mean, sq = orc.layernorm_fwd(z, 4, 1, 1, 32)
    mu = z.mean(axis=1, keepdims=True)
    ref = (z - mu) / np.sqrt(((z - mu) ** 2).mean(axis=1, keepdims=True) + 1e-5)
    assert rel_err(yn, ref) <= 1e-5


def test_oracle_adamw_matches_closed_form(rng):
    from oracle import ops as orc
    n, t, lr = 50, 3, 1e-3
    w = rng.standard_normal(n).astype(np.float32)
    g = rng.standard_normal(n).astype(np.float32)
    m = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    w0 = w.copy()
    orc.adam(w, g, m, v, t, lr, True)
    m_ref = 0.1 * g.astype(np.float64)
    v_ref = 0.001 * g.astype(np.float64) ** 2
    mh, vh = m_ref / (1 - 0.9 ** t), v_ref / (1 - 0.999 ** t)
    w_ref = w0 - lr * (mh / (np.sqrt(vh) + 1e-8) + 0.01 * w0)
    assert rel_err(w, w_ref) <= 1e-6


def test_reference_runtime_never_binds_to_this_library():
    """The reference's runtime (oracle/_ref/librefstep.so, the baseline the
    bench and the parity tests run) defines the same C++ names as
    libmle_engine.so (the drop-in API).  Loaded into one process, neither
    library may call into the other: librefstep.so exports only its
    refstep_* entry points and binds its own calls locally, and
    libmle_engine.so binds its own functions at link time
    (-Bsymbolic-functions).  Checked with the dynamic linker's binding trace,
    every symbol bound at load (LD_BIND_NOW)."""
    import subprocess
    import sys
    so = ROOT / "oracle" / "_ref" / "librefstep.so"
    if not so.exists():
        pytest.skip("oracle/_ref/librefstep.so not built")
    code = ("import sys; sys.path.insert(0, sys.argv[1]);"
            "from ml_engine_b200._lib import engine, kernels; engine(); kernels();"
            "from oracle import ref; ref.step_lib(); ref.lib()")
    env = dict(os.environ, LD_BIND_NOW="1", LD_DEBUG="bindings", CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, "-c", code, str(ROOT)], capture_output=True, text=True, env=env,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    bad = []
    for line in out.stderr.splitlines():
        if "binding file" not in line:
            continue
        src, _, dst = line.partition(" to ")
        ours_src = "libmle_engine" in src or "libmle_kernels" in src
        ref_src = "librefstep" in src or "libmle_ref" in src
        if (ref_src and ("libmle_engine" in dst or "libmle_kernels" in dst)) or \
                (ours_src and ("librefstep" in dst or "libmle_ref" in dst)):
            bad.append(line.strip())
    assert not bad, bad[:5]
    exported = subprocess.run(["nm", "-D", "--defined-only", str(so)], capture_output=True, text=True).stdout
    names = [ln.split()[-1] for ln in exported.splitlines() if ln.strip()]
    assert names and all(n.startswith("refstep_") for n in names), [n for n in names if not n.startswith("refstep_")][:5]
