"""Whole training steps of the benchmark graphs on the CPU oracle.

TEST INFRASTRUCTURE: every step below is the reference's graph executed node
by node with the oracle ops (oracle/mle_oracle.c), forward in topological
order and backward in reverse, with the reference's accumulate/assign
conventions:

  * Linear (Engine/engine.cu:3534-3563): Y = X W + b; dX += dY W^T,
    dW += X^T dY, db += colsum(dY)
  * MultiHeadAttention::forward (Engine/transformer.cu:647-661): Headify,
    BMMABT, Scale(1/sqrt(hd)), SOFTMAX(type 1), BMM, DeHeadify; its backward
    keeps BMMABT's key gradient as the reference computes it, bcmmT(Q, dS)
    (Engine/engine.cu:2307)
  * LayerNorm per token via the [B*S,1,1,D] reshape (Engine/engine.cu:3079-3130)
  * SoftMaxCrossEntropy, last=true (Engine/engine.cu:2063-2111)
  * clip = accumulate + Sqrt_Scale + clipNorm (Engine/engine.cu:3362-3368)
  * AdamW per tensor with its own step counter (Engine/engine.cu:283-292)

Parameters are lists of float32 arrays in the order the native session
reports them (W then b for each Linear, in construction order).
"""
from __future__ import annotations

import math

import numpy as np

from . import ops as o


def _lin_fwd(X, W, b):
    rows, fin = X.shape
    Y = np.zeros((rows, W.shape[1]), np.float32)
    o.gemm(X, W, Y, rows, W.shape[1], fin)
    return o.bias_add(Y, b)


def _lin_bwd(X, W, dY, dX, dW, db):
    rows, fin = X.shape
    fout = W.shape[1]
    if dX is not None:
        o.gemm(dY, W, dX, rows, fin, fout, 0, 1, accumulate=True)
    o.gemm(X, dY, dW, fin, fout, rows, 1, 0, accumulate=True)
    o.bias_grad(dY, db)


def clip_and_update(params, grads, steps, lr, clip_norm=1.0, adamw=True, moments=None):
    """Clip (if clip_norm > 0) then AdamW/Adam.  Returns (clip factor,
    new params, m, v); grads are clipped in place."""
    acc = np.zeros(1, np.float64)
    if clip_norm > 0:
        for g in grads:
            o.sumsq(acc, g)
        x = acc[0]
        if x == x:
            s = math.sqrt(x)
            acc[0] = s / clip_norm if s > clip_norm else 1.0
        for g in grads:
            o.clip_apply(g, acc)
    new_p, ms, vs = [], [], []
    for i, (p, g) in enumerate(zip(params, grads)):
        w = p.copy()
        m = np.zeros_like(w) if moments is None else moments[0][i].copy()
        v = np.zeros_like(w) if moments is None else moments[1][i].copy()
        o.adam(w, g, m, v, steps[i], lr, adamw)
        new_p.append(w)
        ms.append(m)
        vs.append(v)
    return float(acc[0]), new_p, ms, vs


# ============================================================== MLP (config 1)
def mlp_step(params, x, labels, classes=10, lr=1e-3, clip_norm=1.0, steps=None, update=True):
    W1, b1, W2, b2 = [p.reshape(s) for p, s in zip(params, [(x.shape[1], -1), (-1,), (-1, classes), (-1,)])]
    B = x.shape[0]
    h = _lin_fwd(x, W1, b1)
    a = o.act_fwd(0, h)
    logits = _lin_fwd(a, W2, b2)
    target = o.one_hot(labels, classes)
    probs, loss = o.smce_fwd(logits, target, B, classes)
    dlogits = o.smce_bwd(probs, target, float(B)).reshape(B, classes)
    da = np.zeros_like(a)
    gW2, gb2 = np.zeros_like(W2), np.zeros_like(b2)
    _lin_bwd(a, W2, dlogits, da, gW2, gb2)
    dh = o.act_bwd(0, h, da, np.zeros_like(h))
    gW1, gb1 = np.zeros_like(W1), np.zeros_like(b1)
    _lin_bwd(x, W1, dh, np.zeros_like(x), gW1, gb1)
    grads = [g.ravel().copy() for g in (gW1, gb1, gW2, gb2)]
    if not update:
        return dict(loss=loss, grads=grads)
    raw = [g.copy() for g in grads]
    steps = steps or [1] * 4
    clip, new_p, m, v = clip_and_update([p.ravel() for p in params], grads, steps, lr, clip_norm)
    return dict(loss=loss, grads=raw, clipped=grads, clip=clip, params=new_p, m=m, v=v)


# ======================================================== transformer blocks
class _Tape:
    """Records backward closures in forward order; replays them reversed."""

    def __init__(self):
        self.ops = []

    def add(self, fn):
        self.ops.append(fn)

    def backward(self):
        for fn in reversed(self.ops):
            fn()


def _layernorm_tokens(tape, x, dx, rows, D):
    y, _, sq = o.layernorm_fwd(x, rows, 1, 1, D)
    y = y.reshape(rows, D)
    dy = np.zeros_like(y)

    def bwd():
        o.layernorm_bwd(y, dy, sq, dx, rows, 1, 1, D)

    tape.add(bwd)
    return y, dy


def _linear(tape, X, dX, W, b, gW, gb):
    Y = _lin_fwd(X, W, b)
    dY = np.zeros_like(Y)

    def bwd():
        _lin_bwd(X, W, dY, dX, gW, gb)

    tape.add(bwd)
    return Y, dY


def _attention(tape, hq, dhq, hkv, dhkv, P_, G_, B, Sq, Sk, D, H, scale, mask):
    """q/k/v/o Linears around the reference's attention ops.  P_/G_ are the
    four (W, b) parameter and gradient pairs."""
    hd = D // H
    (Wq, bq, Wk, bk, Wv, bv, Wo, bo) = P_
    (gWq, gbq, gWk, gbk, gWv, gbv, gWo, gbo) = G_
    q, dq = _linear(tape, hq, dhq, Wq, bq, gWq, gbq)
    k, dk = _linear(tape, hkv, dhkv, Wk, bk, gWk, gbk)
    v, dv = _linear(tape, hkv, dhkv, Wv, bv, gWv, gbv)
    Qh = o.headify(q, np.zeros(B * Sq * D, np.float32), B, H, Sq, hd, 0)
    Kh = o.headify(k, np.zeros(B * Sk * D, np.float32), B, H, Sk, hd, 0)
    Vh = o.headify(v, np.zeros(B * Sk * D, np.float32), B, H, Sk, hd, 0)
    scores = o.bcmm(1, Qh, Kh, np.zeros(B * H * Sq * Sk, np.float32), B, H, Sq, hd, Sk, 0, 3, 3, 3)
    scaled = o.scale_write(scores, scale)
    P = o.softmax_fwd(scaled, B * H, Sq, Sk, 1, 1 if (mask and Sq > 1) else 0)
    Oh = o.bcmm(0, P, Vh, np.zeros(B * H * Sq * hd, np.float32), B, H, Sq, Sk, hd, 0, 3, 3, 3)
    c = o.headify(Oh, np.zeros(B * Sq * D, np.float32), B, H, Sq, hd, 2).reshape(B * Sq, D)
    dc = np.zeros_like(c)
    dQh, dKh, dVh = (np.zeros(n, np.float32) for n in (B * Sq * D, B * Sk * D, B * Sk * D))

    def attn_bwd():
        dOh = o.headify(dc, np.zeros(B * Sq * D, np.float32), B, H, Sq, hd, 3)
        dP = o.bcmm(1, dOh, Vh, np.zeros(B * H * Sq * Sk, np.float32), B, H, Sq, hd, Sk, 1, 3, 3, 3)
        o.bcmm(2, P, dOh, dVh, B, H, Sk, Sq, hd, 1, 3, 3, 3)
        dsc = o.softmax_bwd(P, dP, np.zeros(B * H * Sq * Sk, np.float32), B * H, Sq, Sk, 1)
        dS = o.accumulate(dsc, np.zeros_like(dsc), scale)
        o.bcmm(0, dS, Kh, dQh, B, H, Sq, Sk, hd, 1, 3, 3, 3)
        o.bcmm(3, Qh, dS, dKh, B, H, hd, Sq, Sk, 1, 3, 3, 3)  # the reference's bcmmT key gradient
        o.headify(dQh, dq, B, H, Sq, hd, 1)
        o.headify(dKh, dk, B, H, Sk, hd, 1)
        o.headify(dVh, dv, B, H, Sk, hd, 1)

    tape.add(attn_bwd)
    a, da = _linear(tape, c, dc, Wo, bo, gWo, gbo)
    return a, da


def _add(tape, a, da, b, db):
    y = o.scale_add(a, b, 1.0)
    dy = np.zeros_like(y)

    def bwd():
        np.add(da, dy, out=da)
        np.add(db, dy, out=db)

    tape.add(bwd)
    return y, dy


def _ffn(tape, h, dh, W1, b1, W2, b2, g):
    f1, df1 = _linear(tape, h, dh, W1, b1, g[0], g[1])
    a = o.act_fwd(4, f1)
    da = np.zeros_like(a)

    def gelu_bwd():
        o.act_bwd(4, f1, da, df1)

    tape.add(gelu_bwd)
    f2, df2 = _linear(tape, a, da, W2, b2, g[2], g[3])
    return f2, df2


def encoder_step(params, table, tokens, targets, batch, seq, d_model, heads, ffn, layers, vocab, lr=1e-3, update=True,
                 clip_norm=1.0, steps=None):
    """One step of the ENCODER session graph on the oracle."""
    B, S, D, H = batch, seq, d_model, heads
    rows = B * S
    shapes = []
    for _ in range(layers):
        shapes += [(D, D), (D,)] * 4 + [(D, ffn), (ffn,), (ffn, D), (D,)]
    shapes += [(D, vocab), (vocab,)]
    P = [p.reshape(s) for p, s in zip(params, shapes)]
    G = [np.zeros_like(p) for p in P]
    tape = _Tape()
    emb = o.embedding_gather(tokens.ravel(), table.reshape(vocab, D))
    x = o.matpe(emb, B, S, D).reshape(rows, D)
    dx = np.zeros_like(x)
    demb = np.zeros_like(x)

    def pe_bwd(dx0=dx):  # bound now: `dx` is rebound per layer below
        np.add(demb, dx0, out=demb)

    tape.add(pe_bwd)
    for layer in range(layers):
        base = layer * 12
        h, dh = _layernorm_tokens(tape, x, dx, rows, D)
        a, da = _attention(tape, h, dh, h, dh, P[base:base + 8], G[base:base + 8], B, S, S, D, H,
                           1.0 / math.sqrt(D // H), False)
        x1, dx1 = _add(tape, x, dx, a, da)
        h2, dh2 = _layernorm_tokens(tape, x1, dx1, rows, D)
        f, df = _ffn(tape, h2, dh2, P[base + 8], P[base + 9], P[base + 10], P[base + 11], G[base + 8:base + 12])
        x, dx = _add(tape, x1, dx1, f, df)
    logits, dlogits = _linear(tape, x, dx, P[-2], P[-1], G[-2], G[-1])
    target = o.one_hot(targets.ravel(), vocab)
    probs, loss = o.smce_fwd(logits, target, rows, vocab)
    dlogits[:] = o.smce_bwd(probs, target, float(B)).reshape(rows, vocab)
    tape.backward()
    grads = [g.ravel().copy() for g in G]
    if not update:
        return dict(loss=loss, grads=grads)
    raw = [g.copy() for g in grads]
    steps = steps or [1] * len(grads)
    clip, new_p, m, v = clip_and_update([p.ravel() for p in P], grads, steps, lr, clip_norm)
    return dict(loss=loss, grads=raw, clipped=grads, clip=clip, params=new_p, m=m, v=v)


def encdec_step(params, tables, src, tgt_in, tgt_out, batch, seq, d_model, heads, ffn, layers, vocab, lr=1e-3, update=True,
                clip_norm=1.0, steps=None):
    """One step of the ENCDEC session graph on the oracle: `layers` encoder
    blocks over the source, `layers` decoder blocks (pre-LN masked
    self-attention scaled by 1/sqrt(head_dim), cross-attention to the raw
    encoder output as MultiHeadAttention::cross_forward does it -- masked,
    scaled by 1/sqrt(d_model), Engine/transformer.cu:662-675 -- and a GELU
    FFN), projection, softmax cross-entropy."""
    B, S, D, H = batch, seq, d_model, heads
    rows = B * S
    enc_shapes, dec_shapes = [], []
    for _ in range(layers):
        enc_shapes += [(D, D), (D,)] * 4 + [(D, ffn), (ffn,), (ffn, D), (D,)]
    for _ in range(layers):
        dec_shapes += [(D, D), (D,)] * 8 + [(D, ffn), (ffn,), (ffn, D), (D,)]
    shapes = enc_shapes + dec_shapes + [(D, vocab), (vocab,)]
    P = [p.reshape(s) for p, s in zip(params, shapes)]
    G = [np.zeros_like(p) for p in P]
    tape = _Tape()

    def embed(tokens, table):
        emb = o.embedding_gather(tokens.ravel(), table.reshape(vocab, D))
        return o.matpe(emb, B, S, D).reshape(rows, D)

    e = embed(src, tables[0])
    de = np.zeros_like(e)
    for layer in range(layers):
        base = layer * 12
        h, dh = _layernorm_tokens(tape, e, de, rows, D)
        a, da = _attention(tape, h, dh, h, dh, P[base:base + 8], G[base:base + 8], B, S, S, D, H,
                           1.0 / math.sqrt(D // H), False)
        e1, de1 = _add(tape, e, de, a, da)
        h2, dh2 = _layernorm_tokens(tape, e1, de1, rows, D)
        f, df = _ffn(tape, h2, dh2, P[base + 8], P[base + 9], P[base + 10], P[base + 11], G[base + 8:base + 12])
        e, de = _add(tape, e1, de1, f, df)
    x = embed(tgt_in, tables[1])
    dx = np.zeros_like(x)
    off = 12 * layers
    for layer in range(layers):
        base = off + layer * 20
        h, dh = _layernorm_tokens(tape, x, dx, rows, D)
        a, da = _attention(tape, h, dh, h, dh, P[base:base + 8], G[base:base + 8], B, S, S, D, H,
                           1.0 / math.sqrt(D // H), True)
        x1, dx1 = _add(tape, x, dx, a, da)
        h2, dh2 = _layernorm_tokens(tape, x1, dx1, rows, D)
        c, dc = _attention(tape, h2, dh2, e, de, P[base + 8:base + 16], G[base + 8:base + 16], B, S, S, D, H,
                           1.0 / math.sqrt(D), True)
        x2, dx2 = _add(tape, x1, dx1, c, dc)
        h3, dh3 = _layernorm_tokens(tape, x2, dx2, rows, D)
        f, df = _ffn(tape, h3, dh3, P[base + 16], P[base + 17], P[base + 18], P[base + 19],
                     G[base + 16:base + 20])
        x, dx = _add(tape, x2, dx2, f, df)
    logits, dlogits = _linear(tape, x, dx, P[-2], P[-1], G[-2], G[-1])
    target = o.one_hot(tgt_out.ravel(), vocab)
    probs, loss = o.smce_fwd(logits, target, rows, vocab)
    dlogits[:] = o.smce_bwd(probs, target, float(B)).reshape(rows, vocab)
    tape.backward()
    grads = [g.ravel().copy() for g in G]
    if not update:
        return dict(loss=loss, grads=grads)
    raw = [g.copy() for g in grads]
    steps = steps or [1] * len(grads)
    clip, new_p, m, v = clip_and_update([p.ravel() for p in P], grads, steps, lr, clip_norm)
    return dict(loss=loss, grads=raw, clipped=grads, clip=clip, params=new_p, m=m, v=v)


# ================================================================== U-Net
def _conv(tape, x, dx, W, b, gW, gb, pad, stride):
    y = o.conv2d_fwd(x, W, b, pad, stride)
    dy = np.zeros_like(y)
    N = x.shape[0]

    def bwd():
        gW[...] = o.conv2d_bwd_k(x, dy, W.shape, pad, stride)          # assigned, as GV2D
        o.channel_bias_bwd(dy, None, gb.reshape(-1), N, W.shape[0], y.shape[2] * y.shape[3])
        if dx is not None:
            o.conv2d_bwd_x(dy, W, dx, pad, stride)

    tape.add(bwd)
    return y, dy


def _convT(tape, x, dx, W, b, gW, gb, pad, stride):
    y = o.convT2d_fwd(x, W, b, pad, stride)
    dy = np.zeros_like(y)
    N = x.shape[0]

    def bwd():
        gW[...] = o.convT2d_bwd_w(x, dy, W.shape, pad, stride)         # assigned, as GVT2D
        o.channel_bias_bwd(dy, None, gb.reshape(-1), N, W.shape[0], y.shape[2] * y.shape[3])
        dx[...] = o.convT2d_bwd_x(dy, W, x.shape, pad, stride)         # assigned, as CVT2D_GradInput

    tape.add(bwd)
    return y, dy


def _groupnorm(tape, x, dx, groups=8):
    N, C, Hh, Ww = x.shape
    y, _, sq = o.groupnorm_fwd(x, N, C, groups, Hh, Ww)
    y = y.reshape(x.shape)
    dy = np.zeros_like(y)

    def bwd():
        o.groupnorm_bwd(y, dy, sq, dx, N, C, groups, Hh, Ww)

    tape.add(bwd)
    return y, dy


def _silu(tape, x, dx):
    y = o.act_fwd(2, x).reshape(x.shape)
    dy = np.zeros_like(y)

    def bwd():
        o.act_bwd(2, x, dy, dx)

    tape.add(bwd)
    return y, dy


def _broadcast_channel(tape, a, da, tv, dtv):
    """Broadcast_Channel: y = a + tv[c]; the B gradient is reduced for the
    first min(width, channels) channels only, as the reference's
    Channel_Squeeze1D<<<width, ...>>> launch does (Engine/engine.cu:1435)."""
    N, C, Hh, Ww = a.shape
    y = o.channel_bias_fwd(a, tv.reshape(-1), N, C, Hh * Ww).reshape(a.shape)
    dy = np.zeros_like(y)

    def bwd():
        np.add(da, dy, out=da)
        red = min(Ww, C)
        part = np.zeros(red, np.float32)
        o.channel_bias_bwd(np.ascontiguousarray(dy[:, :red]), None, part, N, red, Hh * Ww)
        dtv.reshape(-1)[:red] += part

    tape.add(bwd)
    return y, dy


def _residual_block(tape, x, dx, t, dt, prm, grd, cin, cout, stride):
    """ResidualBlock::forward (Engine/diffusion.cu:129-137); prm/grd hold
    conv1 (W, b), conv2 (W, b), time Linear (W, b) and, when the shape
    changes, the 1x1 skip convolution (W, b)."""
    c1, dc1 = _conv(tape, x, dx, prm[0], prm[1], grd[0], grd[1], 1, stride)
    g1, dg1 = _groupnorm(tape, c1, dc1)
    s1, ds1 = _silu(tape, g1, dg1)
    tv, dtv = _linear(tape, t, dt, prm[4], prm[5], grd[4], grd[5])
    h, dh = _broadcast_channel(tape, s1, ds1, tv, dtv)
    c2, dc2 = _conv(tape, h, dh, prm[2], prm[3], grd[2], grd[3], 1, 1)
    g2, dg2 = _groupnorm(tape, c2, dc2)
    if cin != cout or stride != 1:
        skip, dskip = _conv(tape, x, dx, prm[6], prm[7], grd[6], grd[7], 0, stride)
    else:
        skip, dskip = x, dx
    a, da = _add(tape, g2, dg2, skip, dskip)
    return _silu(tape, a.reshape(g2.shape), da.reshape(g2.shape))


def unet_step(params, x_t, noise, batch, channels, image_size, base_width, t_embed, timestep, lr=1e-3,
              clip_norm=1.0, steps=None, update=True):
    """One step of the UNET session graph on the oracle (U_NET::build_train,
    Engine/diffusion.cu:271-294, with three levels)."""
    N, C, S, w = batch, channels, image_size, base_width
    th = t_embed // 2
    shapes = [(t_embed, th), (th,), (th, th), (th,)]

    def block_shapes(cin, cout, stride):
        s = [(cout, cin, 3, 3), (cout,), (cout, cout, 3, 3), (cout,), (th, cout), (cout,)]
        if cin != cout or stride != 1:
            s += [(cout, cin, 1, 1), (cout,)]
        return s

    layout = [("Enc1", C, w, 1), ("Enc2", w, 2 * w, 2), ("Enc3", 2 * w, 4 * w, 2), ("B0", 4 * w, 4 * w, 1),
              ("B1", 4 * w, 4 * w, 1)]
    for _, ci, co, st in layout:
        shapes += block_shapes(ci, co, st)
    shapes += [(4 * w, 4 * w, 2, 2), (4 * w,)] + block_shapes(6 * w, 2 * w, 1)
    shapes += [(2 * w, 2 * w, 2, 2), (2 * w,)] + block_shapes(3 * w, w, 1)
    shapes += [(C, w, 1, 1), (C,)]
    P = [p.reshape(s) for p, s in zip(params, shapes)]
    G = [np.zeros_like(p) for p in P]
    tape = _Tape()
    temb = o.timestep_pe(timestep, t_embed).reshape(1, t_embed)
    t0, dt0 = _linear(tape, temb, None, P[0], P[1], G[0], G[1])
    a0, da0 = _silu(tape, t0, dt0)
    t, dt = _linear(tape, a0, da0, P[2], P[3], G[2], G[3])
    x = x_t.reshape(N, C, S, S).astype(np.float32)
    dx = np.zeros_like(x)
    k = 4
    outs = []
    cur, dcur = x, dx
    for _, ci, co, st in layout:
        n = 8 if (ci != co or st != 1) else 6
        cur, dcur = _residual_block(tape, cur, dcur, t, dt, P[k:k + n], G[k:k + n], ci, co, st)
        outs.append((cur, dcur))
        k += n
    e1, e2 = outs[0], outs[1]

    def up_level(cur, dcur, skip, cin, cout, k):
        u, du = _convT(tape, cur, dcur, P[k], P[k + 1], G[k], G[k + 1], 0, 2)
        Nn, c1, Hh, Ww = u.shape
        c2 = skip[0].shape[1]
        cat = o.channel_concat(u, skip[0], Nn, c1, c2, Hh * Ww).reshape(Nn, c1 + c2, Hh, Ww)
        dcat = np.zeros_like(cat)

        def bwd():
            o.channel_split(du, skip[1], dcat, Nn, c1, c2, Hh * Ww)

        tape.add(bwd)
        n = 8
        y, dy = _residual_block(tape, cat, dcat, t, dt, P[k + 2:k + 2 + n], G[k + 2:k + 2 + n], cin, cout, 1)
        return y, dy, k + 2 + n

    cur, dcur, k = up_level(cur, dcur, e2, 6 * w, 2 * w, k)
    cur, dcur, k = up_level(cur, dcur, e1, 3 * w, w, k)
    y, dy = _conv(tape, cur, dcur, P[k], P[k + 1], G[k], G[k + 1], 0, 1)
    target = noise.reshape(y.shape).astype(np.float32)
    loss = o.mse_fwd(y, target)
    o.mse_bwd(y, target, dy)
    tape.backward()
    grads = [g.ravel().copy() for g in G]
    if not update:
        return dict(loss=loss, grads=grads)
    raw = [g.copy() for g in grads]
    steps = steps or [1] * len(grads)
    clip, new_p, m, v = clip_and_update([p.ravel() for p in P], grads, steps, lr, clip_norm)
    return dict(loss=loss, grads=raw, clipped=grads, clip=clip, params=new_p, m=m, v=v)
