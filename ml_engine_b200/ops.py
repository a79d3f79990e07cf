"""Python face of the sm_100a kernels (include/mle_kernels.h).

Thin wrappers over the C ABI for torch CUDA tensors: every function checks
dtype/contiguity/device, passes raw pointers and the current torch stream,
and raises MLEError on a non-zero status.  Argument names and the
accumulate/assign behaviour follow the reference kernels each entry point
replaces (cited in the header).
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import MLEError, kernels, mle_param_view

RELU, LEAKY_RELU, SILU, TANH, GELU, SIGMOID = range(6)
GEMM_AB, GEMM_ABT, GEMM_ATB, GEMM_ATBT = range(4)


def _p(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise MLEError("ml_engine_b200 kernels need CUDA tensors")
    if t.dtype not in (torch.float32, torch.int32, torch.float64):
        raise MLEError(f"unsupported dtype {t.dtype}")
    if not t.is_contiguous():
        raise MLEError("ml_engine_b200 kernels need contiguous tensors")
    return t.data_ptr()


def _s():
    return torch.cuda.current_stream().cuda_stream


def _call(name, *args):
    kernels().call(name, *args)


def fill(x, value):
    _call("mle_fill", _p(x), value, x.numel(), _s())


def copy(x, y):
    _call("mle_copy", _p(x), _p(y), x.numel(), _s())


def accumulate(x, y, scale=1.0):
    _call("mle_accumulate", _p(x), _p(y), y.numel(), scale, _s())


def add_bwd(g, ga, gb):
    _call("mle_add_bwd", _p(g), _p(ga), _p(gb), g.numel(), _s())


def scale_write(x, y, scale):
    _call("mle_scale_write", _p(x), _p(y), x.numel(), scale, _s())


def scale_add(x, y, z, scale):
    _call("mle_scale_add", _p(x), _p(y), _p(z), scale, x.numel(), _s())


def act_fwd(kind, x, y):
    _call("mle_act_fwd", kind, _p(x), _p(y), x.numel(), _s())


def act_bwd(kind, x, gy, gx, bias_grad=None, assign=False):
    """gx += gy * f'(x) (assign=True: gx = ...; mle_act_bwd_assign)."""
    cols = bias_grad.numel() if bias_grad is not None else 0
    rows = x.numel() // cols if cols else 0
    _call("mle_act_bwd_assign" if assign else "mle_act_bwd", kind, _p(x), _p(gy), _p(gx), x.numel(), _p(bias_grad),
          rows, cols, _s())


def bias_add_fwd(x, bias, y):
    _call("mle_bias_add_fwd", _p(x), _p(bias), _p(y), x.numel() // bias.numel(), bias.numel(), _s())


def bias_grad(g, db, scale=1.0):
    _call("mle_bias_grad", _p(g), _p(db), g.numel() // db.numel(), db.numel(), scale, _s())


def channel_bias_fwd(x, b, y, batch, channels, spatial):
    _call("mle_channel_bias_fwd", _p(x), _p(b), _p(y), batch, channels, spatial, _s())


def channel_bias_bwd(g, gx, gb, batch, channels, spatial):
    _call("mle_channel_bias_bwd", _p(g), _p(gx), _p(gb), batch, channels, spatial, _s())


def channel_bias_bwd_first(g, gb, batch, channels, first, spatial):
    _call("mle_channel_bias_bwd_first", _p(g), _p(gb), batch, channels, first, spatial, _s())


def matpe_fwd(x, y, batch, rows, cols, start_idx=0):
    _call("mle_matpe_fwd", _p(x), _p(y), batch, rows, cols, start_idx, _s())


def timestep_pe(y, t):
    _call("mle_timestep_pe", _p(y), t, y.numel(), _s())


def headify(inp, out, batch, heads, seq, head_dim, flag):
    _call("mle_headify", _p(inp), _p(out), batch, heads, seq, head_dim, flag, _s())


def channel_concat(a, b, c, batch, c1, c2, spatial):
    _call("mle_channel_concat", _p(a), _p(b), _p(c), batch, c1, c2, spatial, _s())


def channel_split(ga, gb, gc, batch, c1, c2, spatial):
    _call("mle_channel_split", _p(ga), _p(gb), _p(gc), batch, c1, c2, spatial, _s())


def embedding_gather(keys, table, out):
    _call("mle_embedding_gather", _p(keys), _p(table), _p(out), keys.numel(), table.shape[-1], _s())


def embedding_update(keys, grad, table, row_len, lr, key_stride=None, gsum=None):
    """table[k] -= lr * (sum of the grad rows whose key is k); int32 keys,
    token t of batch b at keys[b * key_stride + t]."""
    vocab, dim = table.shape[0], table.shape[-1]
    rows = grad.numel() // dim
    if gsum is None:
        gsum = torch.empty_like(table)
    _call("mle_embedding_update", _p(keys), _p(grad), _p(table), _p(gsum), vocab, rows, dim, row_len,
          key_stride if key_stride is not None else row_len, lr, _s())


def one_hot(keys, out, vocab):
    _call("mle_one_hot", _p(keys), _p(out), keys.numel(), vocab, _s())


def layernorm_fwd(x, y, mean, sqdev, batch, channels, row, col, eps=1e-5):
    _call("mle_layernorm_fwd", _p(x), _p(y), _p(mean), _p(sqdev), batch, channels, row, col, eps, _s())


def add_layernorm_fwd(x, r, xr, y, mean, sqdev, batch, channels, row, col, eps=1e-5):
    """xr = x + r and the LayerNorm of xr, in one pass."""
    _call("mle_add_layernorm_fwd", _p(x), _p(r), _p(xr), _p(y), _p(mean), _p(sqdev), batch, channels, row, col, eps,
          _s())


def layernorm_bwd(y, gy, sqdev, gx, batch, channels, row, col, eps=1e-5):
    _call("mle_layernorm_bwd", _p(y), _p(gy), _p(sqdev), _p(gx), batch, channels, row, col, eps, _s())


def groupnorm_fwd(x, y, mean, sqdev, batch, channels, groups, row, col, eps=1e-5):
    _call("mle_groupnorm_fwd", _p(x), _p(y), _p(mean), _p(sqdev), batch, channels, groups, row, col, eps, _s())


def groupnorm_bwd(y, gy, sqdev, gx, batch, channels, groups, row, col, eps=1e-5):
    _call("mle_groupnorm_bwd", _p(y), _p(gy), _p(sqdev), _p(gx), batch, channels, groups, row, col, eps, _s())


def softmax_fwd(x, y, bc, rows, cols, axis, causal=0):
    _call("mle_softmax_fwd", _p(x), _p(y), bc, rows, cols, axis, causal, _s())


def softmax_bwd(y, gy, gx, bc, rows, cols, axis):
    _call("mle_softmax_bwd", _p(y), _p(gy), _p(gx), bc, rows, cols, axis, _s())


def softmax_ce_fwd(logits, target, probs, loss, grad, batch_div, rows, cols):
    _call("mle_softmax_ce_fwd", _p(logits), _p(target), _p(probs), _p(loss), _p(grad), batch_div, rows, cols, _s())


def softmax_ce_bwd(probs, target, grad, batch_div, upstream=None):
    _call("mle_softmax_ce_bwd", _p(probs), _p(target), _p(upstream), _p(grad), batch_div, probs.numel(), _s())


def softmax_ce_index_fwd(logits, labels, probs, loss, grad, batch_div, rows, cols):
    """labels: int32, one class index per row."""
    _call("mle_softmax_ce_index_fwd", _p(logits), _p(labels), _p(probs), _p(loss), _p(grad), batch_div, rows, cols,
          _s())


def softmax_ce_index_bwd(probs, labels, grad, batch_div, rows, cols, upstream=None):
    _call("mle_softmax_ce_index_bwd", _p(probs), _p(labels), _p(upstream), _p(grad), batch_div, rows, cols, _s())


def mse_fwd(x, target, loss):
    _call("mle_mse_fwd", _p(x), _p(target), _p(loss), x.numel(), _s())


def mse_bwd(x, target, gx, upstream=None):
    _call("mle_mse_bwd", _p(x), _p(target), _p(upstream), _p(gx), x.numel(), _s())


def bcmm(variant, A, B, C, batch, channels, m, n, p, backward, A_case, B_case, C_case, scale=1.0):
    _call("mle_bcmm", variant, _p(A), _p(B), _p(C), batch, channels, m, n, p, backward, A_case, B_case, C_case,
          scale, _s())


def gemm(A, B, C, M, N, K, trans_a=0, trans_b=0, alpha=1.0, beta=0.0, bias=None, batch=1, lda=None, ldb=None,
         ldc=None, stride_a=0, stride_b=0, stride_c=0):
    lda = lda if lda is not None else (M if trans_a else K)
    ldb = ldb if ldb is not None else (K if trans_b else N)
    ldc = ldc if ldc is not None else N
    _call("mle_gemm", _p(A), _p(B), _p(C), _p(bias), batch, M, N, K, lda, ldb, ldc, stride_a, stride_b, stride_c,
          trans_a, trans_b, alpha, beta, _s())


def linear_fwd(X, W, bias, Y, rows, in_features, out_features):
    _call("mle_linear_fwd", _p(X), _p(W), _p(bias), _p(Y), rows, in_features, out_features, _s())


def linear_bwd(X, W, dY, dX, dW, dB, rows, in_features, out_features):
    _call("mle_linear_bwd", _p(X), _p(W), _p(dY), _p(dX), _p(dW), _p(dB), rows, in_features, out_features, _s())


KEYGRAD_REFERENCE, KEYGRAD_TRUE = 0, 1
HEAD_MAJOR, TOKEN_MAJOR = 0, 1


def attention_fwd(Q, K, V, P, O, batch, heads, seq_q, seq_k, head_dim, scale, causal=0, softmax_axis=1,
                  layout=HEAD_MAJOR):
    _call("mle_attention_fwd", _p(Q), _p(K), _p(V), _p(P), _p(O), batch, heads, seq_q, seq_k, head_dim, scale, causal,
          softmax_axis, layout, _s())


def attention_bwd(Q, K, V, P, dO, dQ, dK, dV, dP, dS, batch, heads, seq_q, seq_k, head_dim, scale, causal=0,
                  softmax_axis=1, key_grad_mode=KEYGRAD_REFERENCE, layout=HEAD_MAJOR, workspace=None):
    """workspace: batch*heads*seq_q*seq_k floats for the fused and the
    tensor-core paths; made here when not given."""
    if workspace is None:
        workspace = torch.empty(batch * heads * seq_q * seq_k, device=Q.device, dtype=torch.float32)
    _call("mle_attention_bwd", _p(Q), _p(K), _p(V), _p(P), _p(dO), _p(dQ), _p(dK), _p(dV), _p(dP), _p(dS),
          _p(workspace), batch, heads, seq_q, seq_k, head_dim, scale, causal, softmax_axis, key_grad_mode, layout,
          _s())


def attention_flash_fwd(Q, K, V, O, stats, batch, heads, seq_q, seq_k, head_dim, scale, causal=0,
                        layout=HEAD_MAJOR):
    """Column-softmax attention without the score matrices in HBM:
    writes O and stats (2 * batch*heads*seq_k floats: column max, then
    inverse column sum)."""
    _call("mle_attention_flash_fwd", _p(Q), _p(K), _p(V), _p(O), _p(stats), batch, heads, seq_q, seq_k, head_dim,
          scale, causal, layout, _s())


def attention_flash_bwd(Q, K, V, dO, stats, dQ, dK, dV, batch, heads, seq_q, seq_k, head_dim, scale, causal=0,
                        key_grad_mode=KEYGRAD_REFERENCE, layout=HEAD_MAJOR, assign_mask=0, dvec=None):
    """Backward of attention_flash_fwd from its stats; dvec
    (batch*heads*seq_k floats of workspace) is made here when not given."""
    if dvec is None:
        dvec = torch.empty(batch * heads * seq_k, device=Q.device, dtype=torch.float32)
    _call("mle_attention_flash_bwd", _p(Q), _p(K), _p(V), _p(dO), _p(stats), _p(dvec), _p(dQ), _p(dK), _p(dV),
          batch, heads, seq_q, seq_k, head_dim, scale, causal, key_grad_mode, layout, assign_mask, _s())


def attention_flash_supported(seq_q, seq_k, head_dim, softmax_axis=1, key_grad_mode=KEYGRAD_REFERENCE):
    return bool(kernels().mle_attention_flash_supported(seq_q, seq_k, head_dim, softmax_axis, key_grad_mode))


def attention_fused_supported(seq_q, seq_k, head_dim, softmax_axis=1, key_grad_mode=KEYGRAD_REFERENCE):
    return bool(kernels().mle_attention_fused_supported(seq_q, seq_k, head_dim, softmax_axis, key_grad_mode))


ATTN_PATH_AUTO, ATTN_PATH_FUSED, ATTN_PATH_TENSOR = 0, 1, 2


def set_attention_path(path):
    """Attention implementation on this thread (mle_set_attention_path);
    returns the previous one."""
    old = kernels().mle_get_attention_path()
    _call("mle_set_attention_path", path)
    return old


def attention_tensor_supported(seq_q, seq_k, head_dim, softmax_axis=1, key_grad_mode=KEYGRAD_REFERENCE,
                               backward=True):
    """Whether ATTN_PATH_TENSOR runs these sizes on the tensor cores (TF32
    GEMM mode)."""
    ok = softmax_axis == 1 and seq_q % 4 == 0 and seq_k % 4 == 0 and head_dim % 4 == 0
    if backward and key_grad_mode == KEYGRAD_REFERENCE:
        ok = ok and seq_q == seq_k and head_dim % 32 == 0 and seq_k % head_dim == 0
    return ok


def matpe_table(table, rows, cols, start_idx=0):
    _call("mle_matpe_table", _p(table), rows, cols, start_idx, _s())


def rows_add_table(x, table, y, batch):
    _call("mle_rows_add_table", _p(x), _p(table), _p(y), batch, table.numel(), _s())


def param_views(params):
    """params: list of dicts with w, g, m, v (float32 CUDA tensors), t (int32
    CUDA tensor of one element) and optional b1, b2, eps, weight_decay."""
    arr = (mle_param_view * len(params))()
    for i, p in enumerate(params):
        arr[i].w, arr[i].g, arr[i].m, arr[i].v = _p(p["w"]), _p(p["g"]), _p(p["m"]), _p(p["v"])
        arr[i].n = p["w"].numel()
        arr[i].t = _p(p["t"])
        arr[i].b1 = p.get("b1", 0.9)
        arr[i].b2 = p.get("b2", 0.999)
        arr[i].eps = p.get("eps", 1e-8)
        arr[i].weight_decay = p.get("weight_decay", 0.01)
    return arr


# `params` below is a list of dicts (see param_views) or an array already
# made by param_views, which callers that repeat the update can keep.
def _views(params):
    return params if isinstance(params, ctypes.Array) else param_views(params)


def grad_sumsq(params, norm_ws, scale=1.0):
    views = _views(params)
    _call("mle_grad_sumsq", ctypes.cast(views, ctypes.c_void_p), len(views), _p(norm_ws), scale, _s())


def clip_finalize(norm_ws, max_norm=1.0):
    _call("mle_clip_finalize", _p(norm_ws), max_norm, _s())


def clip_apply(params, norm_ws):
    views = _views(params)
    _call("mle_clip_apply", ctypes.cast(views, ctypes.c_void_p), len(views), _p(norm_ws), _s())


def adam_update(params, lr, adamw=True, clip_ws=None, pre_scale=1.0, write_back_grad=True):
    views = _views(params)
    _call("mle_adam_update", ctypes.cast(views, ctypes.c_void_p), len(views), _p(clip_ws), pre_scale, lr,
          int(adamw), int(write_back_grad), _s())


def clip_adam_workspace(params):
    """Device workspace of the one-launch norm + clip + update for this
    parameter list, its tensor table filled (stream ordered)."""
    views = _views(params)
    nbytes = kernels().mle_clip_adam_ws_bytes(len(views))
    if nbytes <= 0:
        raise MLEError("mle_clip_adam_ws_bytes: no tensors")
    ws = torch.zeros((nbytes + 7) // 8, dtype=torch.float64, device="cuda")
    _call("mle_clip_adam_prepare", ctypes.cast(views, ctypes.c_void_p), len(views), _p(ws), ws.numel() * 8, _s())
    return ws


def clip_adam(ws, lr, max_norm=1.0, pre_scale=1.0, adamw=True, write_back_grad=True):
    """One launch: the gradient norm over every tensor of the workspace's
    table, the Sqrt_Scale clip with max_norm (<= 0: none), Adam/AdamW and
    t += 1."""
    _call("mle_clip_adam_run", _p(ws), max_norm, pre_scale, lr, int(adamw), int(write_back_grad), _s())


def clip_adam_status(ws):
    """The workspace's barrier status (0: every barrier met in time)."""
    out = ctypes.c_int(0)
    kernels().mle_clip_adam_status(_p(ws), ctypes.addressof(out), _s())
    return out.value


def watchdog():
    flag = ctypes.c_int(0)
    _call("mle_watchdog_read", ctypes.addressof(flag), _s())
    return flag.value


# ----------------------------------------------------------- convolutions
def conv_out_size(n, k, pad, stride):
    return kernels().mle_conv_out_size(n, k, pad, stride)


def convT_out_size(n, k, pad, stride):
    return kernels().mle_convT_out_size(n, k, pad, stride)


def conv2d_workspace(x, w, pad, stride):
    n, cin, h, wd = x.shape
    cout, _, kh, kw = w.shape
    nf = kernels().mle_conv2d_workspace_floats(n, cin, h, wd, cout, kh, kw, pad, stride)
    if nf < 0:
        raise MLEError("conv2d: kernel does not fit the input")
    return torch.empty(nf, device=x.device, dtype=torch.float32)


def conv2d_fwd(x, w, bias, y, ws, pad, stride):
    """x [N,Cin,H,W], w [Cout,Cin,KH,KW], y [N,Cout,OH,OW] (assigned);
    ws keeps what conv2d_bwd reads of x."""
    n, cin, h, wd = x.shape
    cout, _, kh, kw = w.shape
    _call("mle_conv2d_fwd", _p(x), _p(w), _p(bias), _p(y), _p(ws), n, cin, h, wd, cout, kh, kw, pad, stride, _s())


def conv2d_bwd(x, w, dy, dx, dw, db, ws, pad, stride):
    """dw assigned, db and dx accumulated; x and ws as given to conv2d_fwd.
    Any of dx, dw, db may be None; the dx part and the dw/db part may run as
    two calls on two streams."""
    n, cin, h, wd = x.shape
    cout, _, kh, kw = w.shape
    _call("mle_conv2d_bwd", _p(x), _p(w), _p(dy), _p(dx), _p(dw), _p(db), _p(ws), n, cin, h, wd, cout, kh, kw, pad,
          stride, _s())


def convT2d_workspace(x, w, pad, stride):
    n, cin, h, wd = x.shape
    cout, _, kh, kw = w.shape
    nf = kernels().mle_convT2d_workspace_floats(n, cin, h, wd, cout, kh, kw, pad, stride)
    if nf < 0:
        raise MLEError("convT2d: bad geometry")
    return torch.empty(nf, device=x.device, dtype=torch.float32)


def convT2d_fwd(x, w, bias, y, ws, pad, stride):
    n, cin, h, wd = x.shape
    cout, _, kh, kw = w.shape
    _call("mle_convT2d_fwd", _p(x), _p(w), _p(bias), _p(y), _p(ws), n, cin, h, wd, cout, kh, kw, pad, stride, _s())


def convT2d_bwd(x, w, dy, dx, dw, db, ws, pad, stride):
    """dw and dx assigned, db accumulated."""
    n, cin, h, wd = x.shape
    cout, _, kh, kw = w.shape
    _call("mle_convT2d_bwd", _p(x), _p(w), _p(dy), _p(dx), _p(dw), _p(db), _p(ws), n, cin, h, wd, cout, kh, kw, pad,
          stride, _s())
