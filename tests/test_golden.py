"""Pins the CPU oracle to the reference: replays the inputs stored in
tests/golden/ref_*.npz (outputs of the reference's own CUDA kernels, produced
by tests/golden/make_golden.py) through oracle/mle_oracle.c and compares.
CPU only; tolerance 1e-5 relative per tensor (the reference sums in float,
the oracle in double)."""
from pathlib import Path

import numpy as np
import pytest

from conftest import RTOL_EXACT, rel_err
from oracle import ops as orc

GOLD = Path(__file__).resolve().parent / "golden"


def load(name):
    p = GOLD / f"ref_{name}.npz"
    if not p.exists():
        pytest.skip(f"{p.name} not generated yet (tests/golden/make_golden.py on a GPU)")
    return np.load(p)


def test_golden_bcmm():
    d = load("bcmm")
    i = 0
    while f"c{i}_args" in d:
        v, b, c, m, n, p, bw, ac, bc, cc = (int(x) for x in d[f"c{i}_args"])
        C = d[f"c{i}_C0"].copy()
        orc.bcmm(v, d[f"c{i}_A"], d[f"c{i}_B"], C, b, c, m, n, p, bw, ac, bc, cc, 0.5)
        assert rel_err(C, d[f"c{i}_C"]) <= RTOL_EXACT, i
        i += 1
    assert i >= 6


def test_golden_activations():
    d = load("act")
    for k in range(6):
        assert rel_err(orc.act_fwd(k, d["x"]), d[f"y{k}"]) <= RTOL_EXACT, k
        assert rel_err(orc.act_bwd(k, d["x"], d["g"], d["gx_init"].copy()), d[f"gx{k}"]) <= RTOL_EXACT, k


def test_golden_layernorm_groupnorm():
    d = load("norm")
    y, _, sq = orc.layernorm_fwd(d["ln_x"], 6, 1, 1, 64)
    assert rel_err(y, d["ln_y"]) <= RTOL_EXACT
    assert rel_err(sq, d["ln_sq"]) <= RTOL_EXACT
    gx = orc.layernorm_bwd(d["ln_y"], d["ln_gy"], d["ln_sq"], d["ln_gx0"].copy(), 6, 1, 1, 64)
    assert rel_err(gx, d["ln_gx"]) <= RTOL_EXACT
    y, _, sq = orc.groupnorm_fwd(d["gn_x"], 2, 16, 4, 4, 4)
    assert rel_err(y, d["gn_y"]) <= RTOL_EXACT
    gx = orc.groupnorm_bwd(d["gn_y"], d["gn_gy"], d["gn_sq"], d["gn_gx0"].copy(), 2, 16, 4, 4, 4)
    assert rel_err(gx, d["gn_gx"]) <= RTOL_EXACT


def test_golden_softmax():
    d = load("softmax")
    a, b, c, dd = 2, 3, 9, 13
    for typ in (0, 1):
        for mask in (0, 1):
            y = orc.softmax_fwd(d["x"], a * b, c, dd, typ, mask)
            assert rel_err(y, d[f"y_{typ}{mask}"]) <= RTOL_EXACT
            gx = orc.softmax_bwd(d[f"y_{typ}{mask}"], d["gy"], d["gx0"].copy(), a * b, c, dd, typ)
            assert rel_err(gx, d[f"gx_{typ}{mask}"]) <= RTOL_EXACT


def test_golden_losses():
    d = load("loss")
    rows, cols = d["logits"].shape
    probs, loss = orc.smce_fwd(d["logits"], d["target"], rows, cols)
    assert rel_err(probs, d["probs"].reshape(rows, cols)) <= RTOL_EXACT
    assert abs(loss - float(d["loss"][0])) <= RTOL_EXACT * abs(loss)
    grad = orc.smce_bwd(d["probs"], d["target"].ravel(), float(d["batch"][0]))
    assert rel_err(grad, d["grad"]) <= RTOL_EXACT
    assert abs(orc.mse_fwd(d["mse_x"], d["mse_t"]) - float(d["mse_loss"][0])) <= RTOL_EXACT * float(d["mse_loss"][0])
    assert rel_err(orc.mse_bwd(d["mse_x"], d["mse_t"], d["mse_gx0"].copy()), d["mse_gx"]) <= RTOL_EXACT


def test_golden_clip_and_adam():
    d = load("optim")
    acc = np.zeros(1, np.float64)
    for i in range(3):
        orc.sumsq(acc, d[f"g{i}"])
    orc.clip_finalize(acc)
    assert abs(acc[0] - d["clip"][0]) <= 1e-12 * acc[0]
    for i in range(3):
        assert rel_err(orc.clip_apply(d[f"g{i}"].copy(), acc), d[f"gc{i}"]) <= RTOL_EXACT
    for adamw in (0, 1):
        for t in (1, 5):
            k = f"a{adamw}{t}"
            w, m, v = d[k + "_w0"].copy(), d[k + "_m0"].copy(), d[k + "_v0"].copy()
            orc.adam(w, d[k + "_g"], m, v, t, 1e-3, bool(adamw))
            assert rel_err(m, d[k + "_m"]) <= RTOL_EXACT
            assert rel_err(v, d[k + "_v"]) <= RTOL_EXACT
            assert rel_err(w, d[k + "_w"]) <= RTOL_EXACT


def test_golden_glue():
    d = load("glue")
    for flag in range(4):
        out = orc.headify(d["inp"], d["out0"].copy(), 2, 3, 4, 5, flag)
        assert np.array_equal(out, d[f"h{flag}"]), flag
    assert rel_err(orc.matpe(d["pe_x"], 2, 7, 12, 2), d["pe_y"]) <= RTOL_EXACT
    assert rel_err(orc.bias_grad(d["bc_g"], d["bc_db0"].copy()), d["bc_db"]) <= RTOL_EXACT
    assert rel_err(orc.accumulate(d["acc_x"], d["acc_y0"].copy(), 0.17677669529663687), d["acc_y"]) <= 1e-7


def test_golden_linear():
    d = load("linear")
    batch, ch, m, n, p = (int(x) for x in d["dims"])
    rows = batch * ch * m
    y = np.zeros((rows, p), np.float32)
    orc.gemm(d["X"], d["W"], y, rows, p, n)
    assert rel_err(orc.bias_add(y, d["b"]), d["Y"].reshape(rows, p)) <= RTOL_EXACT
    dx = np.zeros((rows, n), np.float32)
    orc.gemm(d["dY"], d["W"], dx, rows, n, p, 0, 1)
    assert rel_err(dx, d["dX"].reshape(rows, n)) <= RTOL_EXACT
    dw = np.zeros((n, p), np.float32)
    orc.gemm(d["X"], d["dY"], dw, n, p, rows, 1, 0)
    assert rel_err(dw, d["dW"].reshape(n, p)) <= RTOL_EXACT
    assert rel_err(orc.bias_grad(d["dY"], np.zeros(p, np.float32)), d["dB"]) <= RTOL_EXACT


def test_golden_conv():
    d = load("conv")
    for i in range(3):
        N, Cin, Hh, W, Cout, K, pad, s = (int(v) for v in d[f"c{i}_args"])
        x, w, b, dy = d[f"c{i}_x"], d[f"c{i}_w"], d[f"c{i}_b"], d[f"c{i}_dy"]
        assert rel_err(orc.conv2d_fwd(x, w, b, pad, s), d[f"c{i}_y"]) <= RTOL_EXACT
        assert rel_err(orc.conv2d_bwd_k(x, dy, w.shape, pad, s), d[f"c{i}_dk"]) <= RTOL_EXACT
        assert rel_err(orc.conv2d_bwd_x(dy, w, d[f"c{i}_dx0"].copy(), pad, s), d[f"c{i}_dx"]) <= RTOL_EXACT
    for i in range(3):
        N, Cin, Hh, W, Cout, K, pad, s = (int(v) for v in d[f"t{i}_args"])
        x, w, b, dy = d[f"t{i}_x"], d[f"t{i}_w"], d[f"t{i}_b"], d[f"t{i}_dy"]
        assert rel_err(orc.convT2d_fwd(x, w, b, pad, s), d[f"t{i}_y"]) <= RTOL_EXACT
        assert rel_err(orc.convT2d_bwd_w(x, dy, w.shape, pad, s), d[f"t{i}_gw"]) <= RTOL_EXACT
        assert rel_err(orc.convT2d_bwd_x(dy, w, x.shape, pad, s), d[f"t{i}_gx"]) <= RTOL_EXACT


def test_oracle_key_update_is_a_scatter_add():
    """The oracle's KeyUpdate restatement against numpy's unbuffered
    scatter-add (np.add.at), repeated and masked keys included."""
    from oracle import ops as orc
    rng = np.random.default_rng(5)
    batch, clen, max_clen, dim, vocab, lr = 3, 40, 48, 16, 25, 1e-2
    keys = np.full((batch, max_clen), -1, np.int32)
    keys[:, :clen] = rng.integers(-1, vocab, (batch, clen))
    grad = rng.standard_normal((batch * clen, dim)).astype(np.float32)
    table = rng.standard_normal((vocab, dim)).astype(np.float32)
    got = orc.key_update(table.copy(), grad, keys, clen, max_clen, lr)
    want = table.astype(np.float64).copy()
    k = keys[:, :clen].ravel()
    np.add.at(want, k[k >= 0], -lr * grad[k >= 0].astype(np.float64))
    assert np.max(np.abs(got - want)) <= 1e-6 * np.max(np.abs(want))


def test_oracle_gemm_one_thread_wide_product():
    """The oracle's GEMM on one OpenMP thread (what a launcher that pins
    OMP_NUM_THREADS to 1 gives the CPU arms) over a product whose rows of
    double accumulators would not fit a thread's stack many times over:
    finite and equal to numpy, and the thread count restored after."""
    from oracle import ops as orc
    rng = np.random.default_rng(3)
    M, N, K = 3072, 4096, 3
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    C = np.zeros((M, N), np.float32)
    old = orc.set_threads(0)
    try:
        assert orc.set_threads(1) == 1
        orc.gemm(A, B, C, M, N, K)
    finally:
        assert orc.set_threads(old) == old
    ref = A.astype(np.float64) @ B.astype(np.float64)
    assert np.all(np.isfinite(C))
    assert np.max(np.abs(C - ref)) <= 1e-6 * np.max(np.abs(ref))
