"""numpy face of the C oracle (mle_oracle.c).  Test infrastructure only.

Every function takes and returns float32 numpy arrays; "accumulate" outputs
are updated in place, exactly like the reference kernel they restate (see the
citation in mle_oracle.c next to each C function).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

_LIB = None
_HERE = Path(__file__).resolve().parent

F = ctypes.c_float
D = ctypes.c_double
I = ctypes.c_int
L = ctypes.c_int64
P = ctypes.c_void_p

_SIGS = {
    "oracle_conv2d_fwd": (None, [P, P, P, P, I, I, I, I, I, I, I, I, I]),
    "oracle_conv2d_bwd_k": (None, [P, P, P, I, I, I, I, I, I, I, I, I]),
    "oracle_conv2d_bwd_x": (None, [P, P, P, I, I, I, I, I, I, I, I, I]),
    "oracle_convT2d_fwd": (None, [P, P, P, P, I, I, I, I, I, I, I, I, I]),
    "oracle_convT2d_bwd_w": (None, [P, P, P, I, I, I, I, I, I, I, I, I]),
    "oracle_convT2d_bwd_x": (None, [P, P, P, I, I, I, I, I, I, I, I, I]),
    "oracle_act_fwd": (None, [I, P, P, L]),
    "oracle_act_bwd": (None, [I, P, P, P, L]),
    "oracle_accumulate": (None, [P, P, L, D]),
    "oracle_scale_add": (None, [P, P, P, F, L]),
    "oracle_scale_write": (None, [P, P, L, F]),
    "oracle_bias_add": (None, [P, P, L, L]),
    "oracle_bias_grad": (None, [P, P, L, L, F]),
    "oracle_channel_bias_fwd": (None, [P, P, P, I, I, L]),
    "oracle_channel_bias_bwd": (None, [P, P, P, I, I, L]),
    "oracle_matpe": (None, [P, P, I, I, I, I]),
    "oracle_timestep_pe": (None, [P, I, I]),
    "oracle_headify": (None, [P, P, I, I, I, I, I]),
    "oracle_channel_concat": (None, [P, P, P, I, I, I, L]),
    "oracle_channel_split": (None, [P, P, P, I, I, I, L]),
    "oracle_embedding_gather": (None, [P, P, P, L, I]),
    "oracle_one_hot": (None, [P, P, L, I]),
    "oracle_key_update": (None, [P, P, P, I, I, I, F, L]),
    "oracle_bcmm": (None, [I, P, P, P, I, I, I, I, I, I, I, I, I, F]),
    "oracle_gemm": (None, [P, P, P, L, L, L, I, I, I]),
    "oracle_layernorm_fwd": (None, [P, P, P, P, I, I, I, I, F]),
    "oracle_groupnorm_fwd": (None, [P, P, P, P, I, I, I, I, I, F]),
    "oracle_layernorm_bwd": (None, [P, P, P, P, I, I, I, I, F]),
    "oracle_groupnorm_bwd": (None, [P, P, P, P, I, I, I, I, I, F]),
    "oracle_softmax_fwd": (None, [P, P, L, I, I, I, I]),
    "oracle_softmax_bwd": (None, [P, P, P, L, I, I, I]),
    "oracle_smce_fwd": (F, [P, P, P, L, I]),
    "oracle_smce_bwd": (None, [P, P, P, P, F, L]),
    "oracle_mse_fwd": (F, [P, P, L]),
    "oracle_mse_bwd": (None, [P, P, P, P, L]),
    "oracle_sumsq": (None, [P, P, L]),
    "oracle_clip_finalize": (None, [P]),
    "oracle_clip_apply": (None, [P, L, P]),
    "oracle_adam": (None, [P, P, P, P, L, I, F, F, F, F, F, I]),
}


def lib():
    global _LIB
    if _LIB is None:
        so = _HERE / "lib" / "libmle_oracle.so"
        if not so.exists():
            from . import build
            build.build_oracle()
        _LIB = ctypes.CDLL(str(so))
        for name, (res, args) in _SIGS.items():
            fn = getattr(_LIB, name)
            fn.restype = res
            fn.argtypes = args
    return _LIB


def _p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


ACT = {"relu": 0, "leaky_relu": 1, "silu": 2, "tanh": 3, "gelu": 4, "sigmoid": 5}


def act_fwd(kind, x):
    x = f32(x)
    y = np.empty_like(x)
    lib().oracle_act_fwd(kind, _p(x), _p(y), x.size)
    return y


def act_bwd(kind, x, gy, gx):
    lib().oracle_act_bwd(kind, _p(f32(x)), _p(f32(gy)), _p(gx), gx.size)
    return gx


def accumulate(x, y, scale=1.0):
    lib().oracle_accumulate(_p(f32(x)), _p(y), y.size, scale)
    return y


def scale_add(x, y, scale):
    x, y = f32(x), f32(y)
    z = np.empty_like(x)
    lib().oracle_scale_add(_p(x), _p(y), _p(z), scale, x.size)
    return z


def scale_write(x, scale):
    x = f32(x)
    y = np.empty_like(x)
    lib().oracle_scale_write(_p(x), _p(y), x.size, scale)
    return y


def bias_add(x, b):
    x = f32(x).copy()
    lib().oracle_bias_add(_p(x), _p(f32(b)), x.size // b.size, b.size)
    return x


def bias_grad(g, db, scale=1.0):
    cols = db.size
    lib().oracle_bias_grad(_p(f32(g)), _p(db), g.size // cols, cols, scale)
    return db


def channel_bias_fwd(x, b, batch, channels, spatial):
    x = f32(x)
    y = np.empty_like(x)
    lib().oracle_channel_bias_fwd(_p(x), _p(f32(b)), _p(y), batch, channels, spatial)
    return y


def channel_bias_bwd(g, gx, gb, batch, channels, spatial):
    lib().oracle_channel_bias_bwd(_p(f32(g)), _p(gx), _p(gb), batch, channels, spatial)


def matpe(x, batch, rows, cols, start_idx=0):
    x = f32(x)
    y = np.empty_like(x)
    lib().oracle_matpe(_p(x), _p(y), batch, rows, cols, start_idx)
    return y


def timestep_pe(t, dim):
    y = np.empty(dim, np.float32)
    lib().oracle_timestep_pe(_p(y), t, dim)
    return y


def headify(inp, out, b, heads, seq, head_dim, flag):
    lib().oracle_headify(_p(f32(inp)), _p(out), b, heads, seq, head_dim, flag)
    return out


def channel_concat(a, b, batch, c1, c2, spatial):
    c = np.empty(batch * (c1 + c2) * spatial, np.float32)
    lib().oracle_channel_concat(_p(f32(a)), _p(f32(b)), _p(c), batch, c1, c2, spatial)
    return c


def channel_split(ga, gb, gc, batch, c1, c2, spatial):
    lib().oracle_channel_split(_p(ga), _p(gb), _p(f32(gc)), batch, c1, c2, spatial)


def embedding_gather(keys, table):
    keys = np.ascontiguousarray(keys, np.int32)
    out = np.empty((keys.size, table.shape[-1]), np.float32)
    lib().oracle_embedding_gather(_p(keys), _p(f32(table)), _p(out), keys.size, table.shape[-1])
    return out


def key_update(table, grad, keys, clen, max_clen, lr):
    """table (modified in place) -= lr * grad rows at their keys (KeyUpdate)."""
    keys = np.ascontiguousarray(keys, np.int32)
    lib().oracle_key_update(_p(table), _p(f32(grad)), _p(keys), clen, max_clen, table.shape[-1], lr, grad.size)
    return table


def one_hot(keys, vocab):
    keys = np.ascontiguousarray(keys, np.int32)
    out = np.zeros((keys.size, vocab), np.float32)
    lib().oracle_one_hot(_p(keys), _p(out), keys.size, vocab)
    return out


def bcmm(variant, A, B, C, batch, channels, m, n, p, backward, A_case, B_case, C_case, scale=1.0):
    lib().oracle_bcmm(variant, _p(f32(A)), _p(f32(B)), _p(C), batch, channels, m, n, p, backward, A_case, B_case,
                      C_case, scale)
    return C


def set_threads(n):
    """OpenMP threads of the oracle's loops (n <= 0: query); returns the count."""
    return int(lib().oracle_set_threads(int(n)))


def gemm(A, B, C, M, N, K, trans_a=0, trans_b=0, accumulate=False):
    lib().oracle_gemm(_p(f32(A)), _p(f32(B)), _p(C), M, N, K, trans_a, trans_b, int(accumulate))
    return C


def layernorm_fwd(x, batch, channels, row, col, eps=1e-5):
    x = f32(x)
    y = np.empty_like(x)
    mean = np.empty(batch, np.float32)
    sq = np.empty(batch, np.float32)
    lib().oracle_layernorm_fwd(_p(x), _p(y), _p(mean), _p(sq), batch, channels, row, col, eps)
    return y, mean, sq


def layernorm_bwd(y, gy, sq, gx, batch, channels, row, col, eps=1e-5):
    lib().oracle_layernorm_bwd(_p(f32(y)), _p(f32(gy)), _p(f32(sq)), _p(gx), batch, channels, row, col, eps)
    return gx


def groupnorm_fwd(x, batch, channels, groups, row, col, eps=1e-5):
    x = f32(x)
    y = np.empty_like(x)
    mean = np.empty(batch * groups, np.float32)
    sq = np.empty(batch * groups, np.float32)
    lib().oracle_groupnorm_fwd(_p(x), _p(y), _p(mean), _p(sq), batch, channels, groups, row, col, eps)
    return y, mean, sq


def groupnorm_bwd(y, gy, sq, gx, batch, channels, groups, row, col, eps=1e-5):
    lib().oracle_groupnorm_bwd(_p(f32(y)), _p(f32(gy)), _p(f32(sq)), _p(gx), batch, channels, groups, row, col, eps)
    return gx


def softmax_fwd(x, bc, rows, cols, axis, causal=0):
    x = f32(x)
    y = np.empty_like(x)
    lib().oracle_softmax_fwd(_p(x), _p(y), bc, rows, cols, axis, causal)
    return y


def softmax_bwd(y, gy, gx, bc, rows, cols, axis):
    lib().oracle_softmax_bwd(_p(f32(y)), _p(f32(gy)), _p(gx), bc, rows, cols, axis)
    return gx


def smce_fwd(logits, target, rows, cols):
    logits, target = f32(logits), f32(target)
    probs = np.empty_like(logits)
    loss = lib().oracle_smce_fwd(_p(logits), _p(target), _p(probs), rows, cols)
    return probs, loss


def smce_bwd(probs, target, batch_div, upstream=None):
    probs = f32(probs)
    grad = np.empty_like(probs)
    up = None if upstream is None else np.asarray([upstream], np.float32)
    lib().oracle_smce_bwd(_p(probs), _p(f32(target)), _p(up), _p(grad), batch_div, probs.size)
    return grad


def mse_fwd(x, t):
    x, t = f32(x), f32(t)
    return lib().oracle_mse_fwd(_p(x), _p(t), x.size)


def mse_bwd(x, t, gx, upstream=None):
    up = None if upstream is None else np.asarray([upstream], np.float32)
    lib().oracle_mse_bwd(_p(f32(x)), _p(f32(t)), _p(up), _p(gx), gx.size)
    return gx


def sumsq(acc, g):
    lib().oracle_sumsq(_p(acc), _p(f32(g)), g.size)
    return acc


def clip_finalize(acc):
    lib().oracle_clip_finalize(_p(acc))
    return acc


def clip_apply(g, acc):
    lib().oracle_clip_apply(_p(g), g.size, _p(acc))
    return g


def adam(w, g, m, v, t, lr, adamw=True, b1=0.9, b2=0.999, eps=1e-8, wd=0.01):
    lib().oracle_adam(_p(w), _p(f32(g)), _p(m), _p(v), w.size, t, b1, b2, eps, wd, lr, int(adamw))
    return w, m, v


def _cgeom(x, k):
    N, Cin, H, W = x.shape
    Cout, _, KH, KW = k.shape
    return N, Cout, Cin, H, W, KH, KW


def conv2d_fwd(x, k, bias, pad, stride):
    N, Cout, Cin, H, W, KH, KW = _cgeom(x, k)
    OH, OW = (2 * pad + H - KH) // stride + 1, (2 * pad + W - KW) // stride + 1
    y = np.zeros((N, Cout, OH, OW), np.float32)
    lib().oracle_conv2d_fwd(_p(f32(x)), _p(f32(k)), _p(None if bias is None else f32(bias)), _p(y), N, Cout, Cin, H,
                            W, KH, KW, pad, stride)
    return y


def conv2d_bwd_k(x, dz, kshape, pad, stride):
    Cout, Cin, KH, KW = kshape
    N, _, H, W = x.shape
    dk = np.zeros(kshape, np.float32)
    lib().oracle_conv2d_bwd_k(_p(f32(x)), _p(f32(dz)), _p(dk), N, Cout, Cin, H, W, KH, KW, pad, stride)
    return dk


def conv2d_bwd_x(dy, k, dx, pad, stride):
    N, Cin, H, W = dx.shape
    Cout, _, KH, KW = k.shape
    lib().oracle_conv2d_bwd_x(_p(f32(dy)), _p(f32(k)), _p(dx), N, Cout, Cin, H, W, KH, KW, pad, stride)
    return dx


def convT2d_fwd(x, w, bias, pad, stride):
    N, Cout, Cin, H, W, KH, KW = _cgeom(x, w)
    OH, OW = (H - 1) * stride - 2 * pad + KH, (W - 1) * stride - 2 * pad + KW
    y = np.zeros((N, Cout, OH, OW), np.float32)
    lib().oracle_convT2d_fwd(_p(f32(x)), _p(f32(w)), _p(None if bias is None else f32(bias)), _p(y), N, Cout, Cin,
                             H, W, KH, KW, pad, stride)
    return y


def convT2d_bwd_w(x, gout, wshape, pad, stride):
    Cout, Cin, KH, KW = wshape
    N, _, H, W = x.shape
    gw = np.zeros(wshape, np.float32)
    lib().oracle_convT2d_bwd_w(_p(f32(x)), _p(f32(gout)), _p(gw), N, Cout, Cin, H, W, KH, KW, pad, stride)
    return gw


def convT2d_bwd_x(gout, w, xshape, pad, stride):
    N, Cin, H, W = xshape
    Cout, _, KH, KW = w.shape
    gx = np.zeros(xshape, np.float32)
    lib().oracle_convT2d_bwd_x(_p(f32(gout)), _p(f32(w)), _p(gx), N, Cout, Cin, H, W, KH, KW, pad, stride)
    return gx
