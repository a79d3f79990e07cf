"""ctypes bindings of the C ABI in include/*.h.

The prototypes are read from the headers themselves, so the Python side and
the C side cannot drift apart.  Loading never touches the GPU; a missing
library raises instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
INCLUDE = ROOT / "include"
LIBDIR = PKG / "lib"


class MLEError(RuntimeError):
    """A C-ABI entry point returned a non-zero mle_status."""


class mle_param_view(ctypes.Structure):
    _fields_ = [
        ("w", ctypes.c_void_p), ("g", ctypes.c_void_p), ("m", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("n", ctypes.c_int64), ("t", ctypes.c_void_p),
        ("b1", ctypes.c_float), ("b2", ctypes.c_float), ("eps", ctypes.c_float), ("weight_decay", ctypes.c_float),
    ]


_SCALARS = {
    "int": ctypes.c_int, "int64_t": ctypes.c_int64, "int32_t": ctypes.c_int32, "float": ctypes.c_float,
    "double": ctypes.c_double, "uint64_t": ctypes.c_uint64, "size_t": ctypes.c_size_t,
    "mle_stream_t": ctypes.c_void_p, "mle_session_t": ctypes.c_void_p,
}


def _ctype(decl: str):
    decl = decl.strip()
    if decl == "void" or not decl:
        return None
    if "*" in decl:
        base = decl.replace("const", "").replace("*", " ").split()
        if base and base[0] == "char" and decl.count("*") == 1 and "const" in decl:
            return ctypes.c_char_p
        return ctypes.c_void_p
    words = decl.replace("const", "").split()
    typ = words[0] if len(words) == 1 else " ".join(words[:-1]) if words[-1] not in _SCALARS else words[-1]
    for w in words:
        if w in _SCALARS:
            return _SCALARS[w]
    raise ValueError(f"unsupported C type in prototype: {decl!r} ({typ})")


_PROTO = re.compile(r"^\s*(?!typedef)([A-Za-z_][\w\s\*]*?)\s*\b(mle_\w+)\s*\(([^)]*)\)\s*;", re.M)


def parse_header(path: Path) -> dict[str, tuple]:
    """name -> (restype, [argtypes]) for every mle_* prototype in a header."""
    text = path.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    out = {}
    for m in _PROTO.finditer(text):
        ret, name, args = m.group(1), m.group(2), m.group(3)
        argtypes = []
        if args.strip() and args.strip() != "void":
            for a in args.split(","):
                a = a.strip()
                # drop the parameter name
                mm = re.match(r"(.*?)(\b\w+)\s*$", a)
                typ = mm.group(1) if mm and mm.group(1).strip() else a
                argtypes.append(_ctype(typ))
        out[name] = (_ctype(ret), argtypes)
    return out


class _Lib:
    def __init__(self, so: Path, headers: list[Path]):
        if not so.exists():
            raise MLEError(f"{so.name} is not built ({so}); run `python -m ml_engine_b200.build`")
        self.path = so
        self.dll = ctypes.CDLL(str(so), mode=ctypes.RTLD_GLOBAL)
        self.protos = {}
        for h in headers:
            self.protos.update(parse_header(h))
        for name, (res, args) in self.protos.items():
            fn = getattr(self.dll, name)
            fn.restype = res
            fn.argtypes = args

    def __getattr__(self, name):
        if name.startswith("mle_"):
            return getattr(self.dll, name)
        raise AttributeError(name)

    def call(self, name: str, *args):
        st = getattr(self.dll, name)(*args)
        if st != 0:
            k = kernels()   # status strings and the CUDA error live in the kernel library
            raise MLEError(f"{name} -> status {st} ({k.dll.mle_status_string(st).decode()}), "
                           f"cuda error {k.dll.mle_last_cuda_error()}")
        return st


_kernels = None
_engine = None


def kernels() -> _Lib:
    global _kernels
    if _kernels is None:
        _kernels = _Lib(LIBDIR / "libmle_kernels.so", [INCLUDE / "mle_kernels.h"])
        _kernels.dll.mle_status_string.restype = ctypes.c_char_p
    return _kernels


def engine() -> _Lib:
    global _engine
    if _engine is None:
        kernels()
        _engine = _Lib(LIBDIR / "libmle_engine.so", [INCLUDE / "mle_engine.h"])
    return _engine
