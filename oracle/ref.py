"""Binding of the reference's own CUDA kernels (oracle/_ref/libmle_ref.so).

Test infrastructure only: the library is the ML_Engine Engine/kernels.cu
compiled from source plus ref_harness.cu, which launches those kernels the
way the reference's graph lambdas do.  Arguments are torch CUDA tensors.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

_HERE = Path(__file__).resolve().parent
_LIB = None

I, L, F, D, P = ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.c_double, ctypes.c_void_p

_SIGS = {
    "ref_bcmm": [I, P, P, P, I, I, I, I, I, I, I, I, I, F],
    "ref_linear_fwd": [P, P, P, P, I, I, I, I, I, I],
    "ref_linear_bwd": [P, P, P, P, P, P, I, I, I, I, I, I],
    "ref_act_fwd": [I, P, P, I],
    "ref_act_bwd": [I, P, P, P, I],
    "ref_accumulate": [P, P, L, D],
    "ref_scale_write": [P, P, L, F],
    "ref_bcompress": [P, P, I, I, I, I],
    "ref_headify": [P, P, I, I, I, I, I],
    "ref_matpe": [P, P, I, I, I, I],
    "ref_layernorm_fwd": [P, P, P, P, I, I, I, I],
    "ref_layernorm_bwd": [P, P, P, P, P, P, P, P, I, I, I, I],
    "ref_groupnorm_fwd": [P, P, P, P, I, I, I, I, I],
    "ref_groupnorm_bwd": [P, P, P, P, P, P, P, P, I, I, I, I, I],
    "ref_softmax_fwd": [P, P, P, P, I, I, I, I, I, I],
    "ref_softmax_bwd": [P, P, P, I, I, I, I, I],
    "ref_smce_fwd": [P, P, P, P, P, P, I, I, I, I],
    "ref_smce_bwd": [P, P, P, L, I],
    "ref_mse_fwd": [P, P, P, L],
    "ref_mse_bwd": [P, P, P, P, L],
    "ref_channel_squeeze": [P, P, I, I, I, I],
    "ref_sumsq": [P, P, L],
    "ref_clip_finalize": [P],
    "ref_clip_apply": [P, P, L],
    "ref_adam": [P, P, I, I, P, P, F, F, F, F, F, I],
    "ref_conv2d_fwd": [P, P, P, P, I, I, I, I, I, I, I, I, I],
    "ref_conv2d_bwd_k": [P, P, P, I, I, I, I, I, I, I, I, I],
    "ref_conv2d_bwd_x": [P, P, P, I, I, I, I, I, I, I, I, I],
    "ref_convT2d_fwd": [P, P, P, P, I, I, I, I, I, I, I, I, I],
    "ref_convT2d_bwd_w": [P, P, P, I, I, I, I, I, I, I, I, I],
    "ref_convT2d_bwd_x": [P, P, P, I, I, I, I, I, I, I, I, I],
    "ref_key_update": [P, P, P, I, I, I, F, L],
    "ref_sync": [],
}


_STEP_SIGS = {
    "refstep_create": (I, [I, I, I, I, I, I, I, I, I, I, I]),
    "refstep_destroy": (I, []),
    "refstep_param_count": (I, []),
    "refstep_param_numel": (L, [I]),
    "refstep_param_step": (I, [I]),
    "refstep_param_write": (I, [I, I, P]),
    "refstep_param_read": (I, [I, I, P]),
    "refstep_embedding_count": (I, []),
    "refstep_embedding_write": (I, [I, P, L]),
    "refstep_embedding_read": (I, [I, P, L]),
    "refstep_set_embed_update": (I, [I, F]),
    "refstep_input_write": (I, [ctypes.c_char_p, P, L]),
    "refstep_step": (I, [F, I, F, P]),
    "refstep_time": (I, [I, I, F, I, F, P]),
    "refstep_graph_gb": (D, []),
}
_STEP = None


def step_available() -> bool:
    return (_HERE / "_ref" / "librefstep.so").exists()


def step_lib():
    """The reference's own runtime with the BASELINE graphs (ref_step.cu)."""
    global _STEP
    if _STEP is None:
        so = _HERE / "_ref" / "librefstep.so"
        if not so.exists():
            raise RuntimeError("oracle/_ref/librefstep.so is not built (needs the reference source tree)")
        _STEP = ctypes.CDLL(str(so))
        for name, (res, args) in _STEP_SIGS.items():
            fn = getattr(_STEP, name)
            fn.restype = res
            fn.argtypes = args
    return _STEP


def available() -> bool:
    return (_HERE / "_ref" / "libmle_ref.so").exists()


def lib():
    global _LIB
    if _LIB is None:
        so = _HERE / "_ref" / "libmle_ref.so"
        if not so.exists():
            raise RuntimeError("oracle/_ref/libmle_ref.so is not built (needs the reference source tree)")
        _LIB = ctypes.CDLL(str(so))
        for name, args in _SIGS.items():
            fn = getattr(_LIB, name)
            fn.restype = I
            fn.argtypes = args
    return _LIB


# Tensors whose pointers were handed out since the last call(): they must
# stay alive until the launched kernels finished, or the caching allocator
# hands their memory to the next temporary.
_alive = []


def ptr(t):
    if t is None:
        return None
    _alive.append(t)
    return t.data_ptr()


def call(name, *args):
    try:
        st = getattr(lib(), name)(*args)
        if st != 0:
            raise RuntimeError(f"{name}: cuda error {st}")
        st = lib().ref_sync()
        if st != 0:
            raise RuntimeError(f"{name}: cuda error {st} after sync")
    finally:
        _alive.clear()
