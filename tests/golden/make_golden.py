"""Generates tests/golden/ref_*.npz from the reference's OWN CUDA kernels.

Runs on a CUDA machine with oracle/_ref/libmle_ref.so built (the reference's
Engine/kernels.cu compiled from source plus oracle/ref_harness.cu).  Every
fixture stores seeded inputs and the reference kernels' outputs; the CPU test
tests/test_golden.py replays the inputs through the C oracle and compares.

    python tests/golden/make_golden.py [outdir]
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import ref  # noqa: E402

DEV = torch.device("cuda:0")


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def H(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bcmm_cases(rng):
    out = {}
    cases = [(0, 2, 3, 5, 7, 9, 0, 3, 3, 3), (1, 2, 3, 5, 7, 9, 1, 3, 0, 3), (2, 4, 1, 6, 11, 5, 1, 3, 3, 0),
             (3, 2, 2, 8, 6, 8, 1, 3, 3, 3), (0, 3, 2, 4, 5, 6, 1, 0, 0, 0), (2, 2, 3, 7, 4, 3, 1, 1, 3, 2)]
    for i, (v, b, c, m, n, p, bw, ac, bc, cc) in enumerate(cases):
        def size(flag, inner):
            return (b if flag & 1 else 1) * (c if flag & 2 else 1) * inner
        A = rng.standard_normal(size(ac, m * n)).astype(np.float32)
        B = rng.standard_normal(size(bc, n * p)).astype(np.float32)
        C = rng.standard_normal(size(cc, m * p)).astype(np.float32)
        tc = T(C.copy() if bw else np.zeros_like(C))
        ref.call("ref_bcmm", v, ref.ptr(T(A)), ref.ptr(T(B)), ref.ptr(tc), b, c, m, n, p, bw, ac, bc, cc, 0.5)
        out[f"c{i}_args"] = np.array([v, b, c, m, n, p, bw, ac, bc, cc], np.int64)
        out[f"c{i}_A"], out[f"c{i}_B"], out[f"c{i}_C0"], out[f"c{i}_C"] = A, B, C if bw else np.zeros_like(C), H(tc)
    return out


def act_cases(rng):
    n = 777
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    g = rng.standard_normal(n).astype(np.float32)
    gx0 = rng.standard_normal(n).astype(np.float32)
    out = {"x": x, "g": g, "gx_init": gx0}
    for k in range(6):
        y = torch.empty(n, device=DEV)
        ref.call("ref_act_fwd", k, ref.ptr(T(x)), ref.ptr(y), n)
        gx = T(gx0)
        ref.call("ref_act_bwd", k, ref.ptr(T(x)), ref.ptr(T(g)), ref.ptr(gx), n)
        out[f"y{k}"], out[f"gx{k}"] = H(y), H(gx)
    return out


def norm_cases(rng):
    out = {}
    a, b, c, d = 6, 1, 1, 64
    n = a * b * c * d
    x = (rng.standard_normal(n) * 2 + 1).astype(np.float32)
    gy = rng.standard_normal(n).astype(np.float32)
    gx0 = rng.standard_normal(n).astype(np.float32)
    y, mean, sd = torch.empty(n, device=DEV), torch.empty(a, device=DEV), torch.empty(a, device=DEV)
    ref.call("ref_layernorm_fwd", ref.ptr(T(x)), ref.ptr(y), ref.ptr(mean), ref.ptr(sd), a, b, c, d)
    gx = T(gx0)
    s1, s2 = torch.empty(n, device=DEV), torch.empty(n, device=DEV)
    m1, m2 = torch.empty(a, device=DEV), torch.empty(a, device=DEV)
    ref.call("ref_layernorm_bwd", ref.ptr(gx), ref.ptr(y), ref.ptr(T(gy)), ref.ptr(sd), ref.ptr(s1), ref.ptr(s2),
             ref.ptr(m1), ref.ptr(m2), a, b, c, d)
    out.update(ln_x=x, ln_gy=gy, ln_gx0=gx0, ln_y=H(y), ln_sq=H(sd), ln_gx=H(gx))
    # GroupNorm [2, 16, 4, 4], 4 groups
    a, b, c, d, g = 2, 16, 4, 4, 4
    n = a * b * c * d
    x = (rng.standard_normal(n) * 2 + 1).astype(np.float32)
    gy = rng.standard_normal(n).astype(np.float32)
    gx0 = rng.standard_normal(n).astype(np.float32)
    y, mean, sd = torch.empty(n, device=DEV), torch.empty(a * g, device=DEV), torch.empty(a * g, device=DEV)
    ref.call("ref_groupnorm_fwd", ref.ptr(T(x)), ref.ptr(y), ref.ptr(mean), ref.ptr(sd), a, b, c, d, g)
    gx = T(gx0)
    s1, s2 = torch.empty(n, device=DEV), torch.empty(n, device=DEV)
    m1, m2 = torch.empty(a * g, device=DEV), torch.empty(a * g, device=DEV)
    ref.call("ref_groupnorm_bwd", ref.ptr(gx), ref.ptr(y), ref.ptr(T(gy)), ref.ptr(sd), ref.ptr(s1), ref.ptr(s2),
             ref.ptr(m1), ref.ptr(m2), a, b, c, d, g)
    out.update(gn_x=x, gn_gy=gy, gn_gx0=gx0, gn_y=H(y), gn_sq=H(sd), gn_gx=H(gx))
    return out


def softmax_cases(rng):
    out = {}
    a, b, c, d = 2, 3, 9, 13
    n = a * b * c * d
    x = (rng.standard_normal(n) * 2).astype(np.float32)
    gy = rng.standard_normal(n).astype(np.float32)
    gx0 = rng.standard_normal(n).astype(np.float32)
    out.update(x=x, gy=gy, gx0=gx0)
    for typ in (0, 1):
        for mask in (0, 1):
            lines = a * b * (c if typ == 0 else d)
            arr, mx = torch.empty(lines, device=DEV), torch.empty(lines, device=DEV)
            y = torch.empty(n, device=DEV)
            ref.call("ref_softmax_fwd", ref.ptr(T(x)), ref.ptr(arr), ref.ptr(y), ref.ptr(mx), a, b, c, d, typ, mask)
            gx = T(gx0)
            ref.call("ref_softmax_bwd", ref.ptr(y), ref.ptr(T(gy)), ref.ptr(gx), a, b, c, d, typ)
            out[f"y_{typ}{mask}"], out[f"gx_{typ}{mask}"] = H(y), H(gx)
    return out


def loss_cases(rng):
    rows, cols, batch = 12, 10, 4
    logits = (rng.standard_normal((rows, cols)) * 2).astype(np.float32)
    target = np.zeros((rows, cols), np.float32)
    target[np.arange(rows), rng.integers(0, cols, rows)] = 1.0
    soft = torch.empty(rows * cols, device=DEV)
    arr, mx = torch.empty(rows, device=DEV), torch.empty(rows, device=DEV)
    loss = torch.zeros(1, device=DEV)
    ref.call("ref_smce_fwd", ref.ptr(T(logits)), ref.ptr(T(target)), ref.ptr(soft), ref.ptr(arr), ref.ptr(mx),
             ref.ptr(loss), batch, 1, rows // batch, cols)
    grad = torch.empty(rows * cols, device=DEV)
    ref.call("ref_smce_bwd", ref.ptr(soft), ref.ptr(T(target)), ref.ptr(grad), rows * cols, batch)
    x = rng.standard_normal(300).astype(np.float32)
    t = rng.standard_normal(300).astype(np.float32)
    mloss = torch.zeros(1, device=DEV)
    ref.call("ref_mse_fwd", ref.ptr(T(x)), ref.ptr(T(t)), ref.ptr(mloss), 300)
    mgx0 = rng.standard_normal(300).astype(np.float32)
    mgx = T(mgx0)
    ref.call("ref_mse_bwd", ref.ptr(T(x)), ref.ptr(T(t)), ref.ptr(torch.zeros(1, device=DEV)), ref.ptr(mgx), 300)
    return dict(logits=logits, target=target, probs=H(soft), loss=H(loss), grad=H(grad), batch=np.array([batch]),
                mse_x=x, mse_t=t, mse_loss=H(mloss), mse_gx0=mgx0, mse_gx=H(mgx))


def optim_cases(rng):
    out = {}
    sizes = [1000, 37, 513]
    ws = torch.zeros(1, dtype=torch.float64, device=DEV)
    gs = []
    for i, n in enumerate(sizes):
        g = (rng.standard_normal(n) * 0.3).astype(np.float32)
        out[f"g{i}"] = g
        tg = T(g)
        gs.append(tg)
        ref.call("ref_sumsq", ref.ptr(ws), ref.ptr(tg), n)
    ref.call("ref_clip_finalize", ref.ptr(ws))
    out["clip"] = H(ws)
    for i, n in enumerate(sizes):
        ref.call("ref_clip_apply", ref.ptr(gs[i]), ref.ptr(ws), n)
        out[f"gc{i}"] = H(gs[i])
    for adamw in (0, 1):
        for t in (1, 5):
            n = 999
            w = (rng.standard_normal(n) * 0.02).astype(np.float32)
            g = (rng.standard_normal(n) * 0.1).astype(np.float32)
            m = (rng.standard_normal(n) * 0.01).astype(np.float32)
            v = np.abs(rng.standard_normal(n) * 1e-3).astype(np.float32)
            tw, tm, tv = T(w), T(m), T(v)
            ref.call("ref_adam", ref.ptr(tw), ref.ptr(T(g)), n, t, ref.ptr(tm), ref.ptr(tv), 0.9, 0.999, 1e-8, 0.01,
                     1e-3, adamw)
            k = f"a{adamw}{t}"
            out.update({k + "_w0": w, k + "_g": g, k + "_m0": m, k + "_v0": v, k + "_w": H(tw), k + "_m": H(tm),
                        k + "_v": H(tv)})
    return out


def glue_cases(rng):
    B, Hh, S, D = 2, 3, 4, 5
    n = B * Hh * S * D
    inp = rng.standard_normal(n).astype(np.float32)
    out0 = rng.standard_normal(n).astype(np.float32)
    out = {"inp": inp, "out0": out0}
    for flag in range(4):
        o = T(out0)
        ref.call("ref_headify", ref.ptr(T(inp)), ref.ptr(o), B, Hh, S, D, flag)
        out[f"h{flag}"] = H(o)
    x = rng.standard_normal(2 * 7 * 12).astype(np.float32)
    y = torch.empty(x.size, device=DEV)
    ref.call("ref_matpe", ref.ptr(T(x)), ref.ptr(y), 2, 7, 12, 2)
    out.update(pe_x=x, pe_y=H(y))
    g = rng.standard_normal((9, 11)).astype(np.float32)
    db0 = rng.standard_normal(11).astype(np.float32)
    db = T(db0)
    ref.call("ref_bcompress", ref.ptr(T(g)), ref.ptr(db), 3, 1, 3, 11)
    out.update(bc_g=g, bc_db0=db0, bc_db=H(db))
    acc0 = rng.standard_normal(50).astype(np.float32)
    acc = T(acc0)
    xs = rng.standard_normal(50).astype(np.float32)
    ref.call("ref_accumulate", ref.ptr(T(xs)), ref.ptr(acc), 50, 0.17677669529663687)
    out.update(acc_x=xs, acc_y0=acc0, acc_y=H(acc))
    return out


def linear_cases(rng):
    batch, ch, m, n, p = 3, 1, 4, 20, 12
    X = rng.random((batch * m, n)).astype(np.float32)
    W = (rng.standard_normal((n, p)) * 0.3).astype(np.float32)
    b = (rng.standard_normal(p) * 0.1).astype(np.float32)
    Y = torch.empty(batch * m * p, device=DEV)
    ref.call("ref_linear_fwd", ref.ptr(T(X)), ref.ptr(T(W)), ref.ptr(T(b)), ref.ptr(Y), batch, ch, m, n, p, 1)
    dY = rng.standard_normal((batch * m, p)).astype(np.float32)
    dX = torch.zeros(batch * m * n, device=DEV)
    dW, dB = torch.zeros(n * p, device=DEV), torch.zeros(p, device=DEV)
    ref.call("ref_linear_bwd", ref.ptr(T(X)), ref.ptr(T(W)), ref.ptr(T(dY)), ref.ptr(dX), ref.ptr(dW), ref.ptr(dB),
             batch, ch, m, n, p, 1)
    return dict(X=X, W=W, b=b, Y=H(Y), dY=dY, dX=H(dX), dW=H(dW), dB=H(dB),
                dims=np.array([batch, ch, m, n, p], np.int64))


def conv_cases(rng):
    """CV2D / GV2D / CV2D_GradInput and CVT2D / GVT2D / CVT2D_GradInput with
    the reference lambdas' launch shapes, small enough for the CPU oracle."""
    out = {}
    convs = [(2, 3, 9, 7, 4, 3, 1, 1), (2, 4, 9, 10, 3, 3, 1, 2), (1, 5, 6, 6, 2, 1, 0, 1)]
    for i, (N, Cin, Hh, W, Cout, K, pad, s) in enumerate(convs):
        OH, OW = (2 * pad + Hh - K) // s + 1, (2 * pad + W - K) // s + 1
        x = rng.standard_normal((N, Cin, Hh, W)).astype(np.float32)
        w = rng.standard_normal((Cout, Cin, K, K)).astype(np.float32)
        b = rng.standard_normal(Cout).astype(np.float32)
        dy = rng.standard_normal((N, Cout, OH, OW)).astype(np.float32)
        dx0 = rng.standard_normal(x.shape).astype(np.float32)
        y, dk, dx = torch.empty(N, Cout, OH, OW, device=DEV), torch.empty(w.shape, device=DEV), T(dx0)
        ref.call("ref_conv2d_fwd", ref.ptr(T(x)), ref.ptr(T(w)), ref.ptr(T(b)), ref.ptr(y), N, Cout, Cin, Hh, W, K, K,
                 pad, s)
        ref.call("ref_conv2d_bwd_k", ref.ptr(T(x)), ref.ptr(T(dy)), ref.ptr(dk), N, Cout, Cin, Hh, W, K, K, pad, s)
        ref.call("ref_conv2d_bwd_x", ref.ptr(T(dy)), ref.ptr(T(w)), ref.ptr(dx), N, Cout, Cin, Hh, W, K, K, pad, s)
        out.update({f"c{i}_args": np.array([N, Cin, Hh, W, Cout, K, pad, s], np.int64), f"c{i}_x": x, f"c{i}_w": w,
                    f"c{i}_b": b, f"c{i}_dy": dy, f"c{i}_dx0": dx0, f"c{i}_y": H(y), f"c{i}_dk": H(dk),
                    f"c{i}_dx": H(dx)})
    convts = [(2, 4, 4, 5, 3, 2, 0, 2), (1, 3, 5, 4, 2, 3, 1, 2), (2, 2, 6, 6, 3, 3, 1, 1)]
    for i, (N, Cin, Hh, W, Cout, K, pad, s) in enumerate(convts):
        OH, OW = (Hh - 1) * s - 2 * pad + K, (W - 1) * s - 2 * pad + K
        x = rng.standard_normal((N, Cin, Hh, W)).astype(np.float32)
        w = rng.standard_normal((Cout, Cin, K, K)).astype(np.float32)
        b = rng.standard_normal(Cout).astype(np.float32)
        dy = rng.standard_normal((N, Cout, OH, OW)).astype(np.float32)
        y, gw, gx = torch.empty(N, Cout, OH, OW, device=DEV), torch.empty(w.shape, device=DEV), torch.empty(x.shape,
                                                                                                          device=DEV)
        ref.call("ref_convT2d_fwd", ref.ptr(T(x)), ref.ptr(T(w)), ref.ptr(T(b)), ref.ptr(y), N, Cout, Cin, Hh, W, K,
                 K, pad, s)
        ref.call("ref_convT2d_bwd_w", ref.ptr(T(x)), ref.ptr(T(dy)), ref.ptr(gw), N, Cout, Cin, Hh, W, K, K, pad, s)
        ref.call("ref_convT2d_bwd_x", ref.ptr(T(dy)), ref.ptr(T(w)), ref.ptr(gx), N, Cout, Cin, Hh, W, K, K, pad, s)
        out.update({f"t{i}_args": np.array([N, Cin, Hh, W, Cout, K, pad, s], np.int64), f"t{i}_x": x, f"t{i}_w": w,
                    f"t{i}_b": b, f"t{i}_dy": dy, f"t{i}_y": H(y), f"t{i}_gw": H(gw), f"t{i}_gx": H(gx)})
    return out


def main(outdir: Path):
    outdir.mkdir(parents=True, exist_ok=True)
    rng = np.random.default_rng(20261201)
    for name, fn in [("bcmm", bcmm_cases), ("act", act_cases), ("norm", norm_cases), ("softmax", softmax_cases),
                     ("loss", loss_cases), ("optim", optim_cases), ("glue", glue_cases), ("linear", linear_cases),
                     ("conv", conv_cases)]:
        data = fn(rng)
        np.savez_compressed(outdir / f"ref_{name}.npz", **data)
        print("wrote", outdir / f"ref_{name}.npz")


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent)
