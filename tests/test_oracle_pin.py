"""Reference kernels vs. oracle vs. the sm_100a kernels, on the GPU.

oracle/_ref/libmle_ref.so is the reference's own Engine/kernels.cu compiled
from source; these tests (1) pin the C oracle to it at sizes beyond the
committed fixtures and (2) show where the new kernels reproduce the reference
bit for bit (elementwise, column softmax, AdamW) or within the stated
tolerance (TF32 GEMMs).
"""
import numpy as np
import pytest

from conftest import RTOL_EXACT, RTOL_TC, rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ref():
    from oracle import ref as r
    if not r.available():
        pytest.skip("oracle/_ref not built")
    return r


@pytest.fixture(scope="module")
def ops():
    from ml_engine_b200 import ops as o
    return o


@pytest.fixture(scope="module")
def orc():
    from oracle import ops as o
    return o


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def H(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("kind", range(6))
def test_activation_bitwise(cuda, ref, ops, orc, rng, kind):
    n = 1 << 16
    x = (rng.standard_normal(n) * 4).astype(np.float32)
    g = rng.standard_normal(n).astype(np.float32)
    gx0 = rng.standard_normal(n).astype(np.float32)
    yr, ym = torch.empty(n, device=cuda), torch.empty(n, device=cuda)
    ref.call("ref_act_fwd", kind, ref.ptr(T(x, cuda)), ref.ptr(yr), n)
    ops.act_fwd(kind, T(x, cuda), ym)
    assert np.array_equal(H(yr), H(ym))
    assert rel_err(H(yr), orc.act_fwd(kind, x)) <= RTOL_EXACT
    gr, gm = T(gx0, cuda), T(gx0, cuda)
    ref.call("ref_act_bwd", kind, ref.ptr(T(x, cuda)), ref.ptr(T(g, cuda)), ref.ptr(gr), n)
    ops.act_bwd(kind, T(x, cuda), T(g, cuda), gm)
    assert np.array_equal(H(gr), H(gm))
    assert rel_err(H(gr), orc.act_bwd(kind, x, g, gx0.copy())) <= RTOL_EXACT


@pytest.mark.parametrize("mask", [0, 1])
def test_column_softmax_bitwise(cuda, ref, ops, orc, rng, mask):
    a, b, c, d = 4, 8, 128, 128
    n = a * b * c * d
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    arr, mx, yr = torch.empty(a * b * d, device=cuda), torch.empty(a * b * d, device=cuda), torch.empty(n, device=cuda)
    ref.call("ref_softmax_fwd", ref.ptr(T(x, cuda)), ref.ptr(arr), ref.ptr(yr), ref.ptr(mx), a, b, c, d, 1, mask)
    ym = torch.empty(n, device=cuda)
    ops.softmax_fwd(T(x, cuda), ym, a * b, c, d, 1, mask)
    assert np.array_equal(H(yr), H(ym))
    assert rel_err(H(yr), orc.softmax_fwd(x, a * b, c, d, 1, mask)) <= RTOL_EXACT
    gy = rng.standard_normal(n).astype(np.float32)
    gr, gm = torch.zeros(n, device=cuda), torch.zeros(n, device=cuda)
    ref.call("ref_softmax_bwd", ref.ptr(yr), ref.ptr(T(gy, cuda)), ref.ptr(gr), a, b, c, d, 1)
    ops.softmax_bwd(yr, T(gy, cuda), gm, a * b, c, d, 1)
    assert np.array_equal(H(gr), H(gm))


@pytest.mark.parametrize("adamw", [0, 1])
@pytest.mark.parametrize("t", [1, 2, 10, 1000])
def test_adam_bitwise(cuda, ref, ops, orc, rng, adamw, t):
    n = 100003
    w = (rng.standard_normal(n) * 0.02).astype(np.float32)
    g = (rng.standard_normal(n) * 0.1).astype(np.float32)
    m = (rng.standard_normal(n) * 0.01).astype(np.float32)
    v = np.abs(rng.standard_normal(n) * 1e-3).astype(np.float32)
    rw, rm, rv = T(w, cuda), T(m, cuda), T(v, cuda)
    ref.call("ref_adam", ref.ptr(rw), ref.ptr(T(g, cuda)), n, t, ref.ptr(rm), ref.ptr(rv), 0.9, 0.999, 1e-8, 0.01,
             1e-3, adamw)
    p = dict(w=T(w, cuda), g=T(g, cuda), m=T(m, cuda), v=T(v, cuda), t=torch.tensor([t], dtype=torch.int32,
                                                                                    device=cuda))
    ops.adam_update([p], lr=1e-3, adamw=bool(adamw))
    for a, b in ((rw, p["w"]), (rm, p["m"]), (rv, p["v"])):
        assert np.array_equal(H(a), H(b))
    ow, om, ov = w.copy(), m.copy(), v.copy()
    orc.adam(ow, g, om, ov, t, 1e-3, bool(adamw))
    assert rel_err(H(rw), ow) <= RTOL_EXACT


def test_clip_matches_reference(cuda, ref, ops, rng):
    sizes = [200000, 513, 7]
    gs = [(rng.standard_normal(n) * 0.2).astype(np.float32) for n in sizes]
    ws_r = torch.zeros(1, dtype=torch.float64, device=cuda)
    tr = [T(g, cuda) for g in gs]
    for t_, n in zip(tr, sizes):
        ref.call("ref_sumsq", ref.ptr(ws_r), ref.ptr(t_), n)
    ref.call("ref_clip_finalize", ref.ptr(ws_r))
    for t_, n in zip(tr, sizes):
        ref.call("ref_clip_apply", ref.ptr(t_), ref.ptr(ws_r), n)
    ps = [dict(w=torch.zeros(n, device=cuda), g=T(g, cuda), m=torch.zeros(n, device=cuda),
               v=torch.zeros(n, device=cuda), t=torch.ones(1, dtype=torch.int32, device=cuda))
          for g, n in zip(gs, sizes)]
    ws = torch.zeros(1, dtype=torch.float64, device=cuda)
    ops.grad_sumsq(ps, ws)
    ops.clip_finalize(ws)
    assert abs(H(ws)[0] - H(ws_r)[0]) <= 1e-12 * H(ws_r)[0]
    ops.clip_apply(ps, ws)
    for a, p in zip(tr, ps):
        assert rel_err(H(p["g"]), H(a)) <= 1e-7


@pytest.mark.parametrize("variant", range(4))
def test_bcmm_reference(cuda, ref, ops, orc, rng, variant):
    b, c, m, n, p = 2, 4, 128, 64, 96
    A = rng.standard_normal(b * c * m * n).astype(np.float32)
    B = rng.standard_normal(b * c * n * p).astype(np.float32)
    C0 = rng.standard_normal(b * c * m * p).astype(np.float32)
    cr, cm = T(C0, cuda), T(C0, cuda)
    ref.call("ref_bcmm", variant, ref.ptr(T(A, cuda)), ref.ptr(T(B, cuda)), ref.ptr(cr), b, c, m, n, p, 1, 3, 3, 3,
             0.5)
    ops.bcmm(variant, T(A, cuda), T(B, cuda), cm, b, c, m, n, p, 1, 3, 3, 3, 0.5)
    ro = orc.bcmm(variant, A, B, C0.copy(), b, c, m, n, p, 1, 3, 3, 3, 0.5)
    assert rel_err(H(cr) - C0, ro - C0) <= RTOL_EXACT
    assert np.max(np.abs(H(cm) - H(cr))) / np.max(np.abs(H(cr) - C0)) <= RTOL_TC


def test_layernorm_reference(cuda, ref, ops, orc, rng):
    a, d = 4096, 256
    n = a * d
    x = (rng.standard_normal(n) * 2 + 1).astype(np.float32)
    gy = rng.standard_normal(n).astype(np.float32)
    y, mean, sd = torch.empty(n, device=cuda), torch.empty(a, device=cuda), torch.empty(a, device=cuda)
    ref.call("ref_layernorm_fwd", ref.ptr(T(x, cuda)), ref.ptr(y), ref.ptr(mean), ref.ptr(sd), a, 1, 1, d)
    gx = torch.zeros(n, device=cuda)
    s1, s2, m1, m2 = (torch.empty(k, device=cuda) for k in (n, n, a, a))
    ref.call("ref_layernorm_bwd", ref.ptr(gx), ref.ptr(y), ref.ptr(T(gy, cuda)), ref.ptr(sd), ref.ptr(s1),
             ref.ptr(s2), ref.ptr(m1), ref.ptr(m2), a, 1, 1, d)
    ym, mm, sm = torch.empty(n, device=cuda), torch.empty(a, device=cuda), torch.empty(a, device=cuda)
    ops.layernorm_fwd(T(x, cuda), ym, mm, sm, a, 1, 1, d)
    gm = torch.zeros(n, device=cuda)
    ops.layernorm_bwd(ym, T(gy, cuda), sm, gm, a, 1, 1, d)
    assert rel_err(H(ym), H(y)) <= RTOL_EXACT
    assert rel_err(H(gm), H(gx)) <= RTOL_EXACT
    ry, _, rsq = orc.layernorm_fwd(x, a, 1, 1, d)
    assert rel_err(H(y), ry) <= RTOL_EXACT


def test_smce_reference(cuda, ref, ops, orc, rng):
    batch, S, V = 8, 16, 4096
    rows = batch * S
    logits = (rng.standard_normal((rows, V)) * 2).astype(np.float32)
    target = np.zeros((rows, V), np.float32)
    target[np.arange(rows), rng.integers(0, V, rows)] = 1
    soft, arr, mx = torch.empty(rows * V, device=cuda), torch.empty(rows, device=cuda), torch.empty(rows, device=cuda)
    loss = torch.zeros(1, device=cuda)
    ref.call("ref_smce_fwd", ref.ptr(T(logits, cuda)), ref.ptr(T(target, cuda)), ref.ptr(soft), ref.ptr(arr),
             ref.ptr(mx), ref.ptr(loss), batch, 1, S, V)
    grad = torch.empty(rows * V, device=cuda)
    ref.call("ref_smce_bwd", ref.ptr(soft), ref.ptr(T(target, cuda)), ref.ptr(grad), rows * V, batch)
    gm, lm = torch.empty(rows * V, device=cuda), torch.empty(1, device=cuda)
    ops.softmax_ce_fwd(T(logits, cuda), T(target, cuda), None, lm, gm, float(batch), rows, V)
    assert abs(H(lm)[0] - H(loss)[0]) <= RTOL_EXACT * abs(H(loss)[0])
    assert rel_err(H(gm), H(grad)) <= RTOL_EXACT
    _, oloss = orc.smce_fwd(logits, target, rows, V)
    assert abs(oloss - H(loss)[0]) <= RTOL_EXACT * abs(oloss)


@pytest.mark.parametrize("mask", [0, 1])
def test_fused_attention_bitwise_vs_reference_chain(cuda, ref, ops, rng, mask):
    """The fused attention kernels against the reference's own kernel chain
    (bcmmABT, Scale_Write, SoftMax/SoftMask type 1, bcmm; then bcmmABT,
    bcmmATB, deriv_softmax, Accumulate, bcmm, bcmmT) run through oracle/_ref:
    P, O, dQ, dK (reference key gradient) and dV are bitwise equal."""
    B, Hh, S, D = 2, 4, 128, 32
    bh, n_s = B * Hh, B * Hh * S * S
    old_path = ops.set_attention_path(ops.ATTN_PATH_FUSED)
    Q, K, V, dO = (rng.standard_normal((bh, S, D)).astype(np.float32) for _ in range(4))
    scale = float(np.float32(1.0 / np.sqrt(D)))  # GraphOperations::Scale holds a float
    tQ, tK, tV, tdO = (T(a, cuda) for a in (Q, K, V, dO))
    # reference forward
    scores, scaled, rP = (torch.zeros(n_s, device=cuda) for _ in range(3))
    ref.call("ref_bcmm", 1, ref.ptr(tQ), ref.ptr(tK), ref.ptr(scores), B, Hh, S, D, S, 0, 3, 3, 3, 1.0)
    ref.call("ref_scale_write", ref.ptr(scores), ref.ptr(scaled), n_s, scale)
    arr, mx = torch.empty(bh * S, device=cuda), torch.empty(bh * S, device=cuda)
    ref.call("ref_softmax_fwd", ref.ptr(scaled), ref.ptr(arr), ref.ptr(rP), ref.ptr(mx), B, Hh, S, S, 1, mask)
    rO = torch.zeros(bh * S * D, device=cuda)
    ref.call("ref_bcmm", 0, ref.ptr(rP), ref.ptr(tV), ref.ptr(rO), B, Hh, S, S, D, 0, 3, 3, 3, 1.0)
    # fused forward (head-major)
    P, O = torch.zeros(n_s, device=cuda), torch.zeros(bh * S * D, device=cuda)
    ops.attention_fwd(tQ, tK, tV, P, O, B, Hh, S, S, D, scale, mask, 1, 0)
    assert np.array_equal(H(P), H(rP))
    assert np.array_equal(H(O), H(rO))
    # reference backward
    rdP, rdSc, rdS = (torch.zeros(n_s, device=cuda) for _ in range(3))
    rdQ, rdK, rdV = (torch.zeros(bh * S * D, device=cuda) for _ in range(3))
    ref.call("ref_bcmm", 1, ref.ptr(tdO), ref.ptr(tV), ref.ptr(rdP), B, Hh, S, D, S, 1, 3, 3, 3, 1.0)
    ref.call("ref_bcmm", 2, ref.ptr(rP), ref.ptr(tdO), ref.ptr(rdV), B, Hh, S, S, D, 1, 3, 3, 3, 1.0)
    ref.call("ref_softmax_bwd", ref.ptr(rP), ref.ptr(rdP), ref.ptr(rdSc), B, Hh, S, S, 1)
    ref.call("ref_accumulate", ref.ptr(rdSc), ref.ptr(rdS), n_s, scale)
    ref.call("ref_bcmm", 0, ref.ptr(rdS), ref.ptr(tK), ref.ptr(rdQ), B, Hh, S, S, D, 1, 3, 3, 3, 1.0)
    ref.call("ref_bcmm", 3, ref.ptr(tQ), ref.ptr(rdS), ref.ptr(rdK), B, Hh, D, S, S, 1, 3, 3, 3, 1.0)
    dQ, dK, dV = (torch.zeros(bh * S * D, device=cuda) for _ in range(3))
    dP, dS = torch.zeros(n_s, device=cuda), torch.zeros(n_s, device=cuda)
    ops.attention_bwd(tQ, tK, tV, P, tdO, dQ, dK, dV, dP, dS, B, Hh, S, S, D, scale, mask, 1, 0, 0)
    ops.set_attention_path(old_path)
    for mine, theirs in ((dP, rdP), (dS, rdSc), (dV, rdV), (dQ, rdQ), (dK, rdK)):
        assert np.array_equal(H(mine), H(theirs))
