"""Parity of every sm_100a kernel (C ABI, include/mle_kernels.h) with the CPU
oracle on seeded inputs, including ragged, unaligned and edge sizes.

Tolerances (see conftest): 1e-5 for elementwise / reduction / Adam paths,
2e-3 per tensor for the TF32 tensor-core GEMMs.
"""
import ctypes

import numpy as np
import pytest

from conftest import RTOL_EXACT, RTOL_TC, norm_err, rel_err

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def H(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


@pytest.fixture(scope="module")
def ops():
    from ml_engine_b200 import ops as o
    return o


@pytest.fixture(scope="module")
def orc():
    from oracle import ops as o
    return o


# ---------------------------------------------------------------- elementwise
@pytest.mark.parametrize("n", [1, 7, 1024, 4099, 1 << 20])
def test_glue_ops(cuda, ops, orc, rng, n):
    x = rng.standard_normal(n).astype(np.float32)
    y = rng.standard_normal(n).astype(np.float32)
    gx, gy = T(x, cuda), T(y, cuda)
    out = torch.empty_like(gx)
    ops.fill(out, 3.5)
    assert np.all(H(out) == 3.5)
    ops.copy(gx, out)
    assert np.array_equal(H(out), x)
    acc = gy.clone()
    ops.accumulate(gx, acc, 0.125)
    assert rel_err(H(acc), orc.accumulate(x, y.copy(), 0.125)) <= 1e-7
    ops.scale_write(gx, out, 0.3)
    assert np.array_equal(H(out), orc.scale_write(x, 0.3))
    ops.scale_add(gx, gy, out, -1.0)
    assert np.array_equal(H(out), orc.scale_add(x, y, -1.0))
    a, b = gy.clone(), gx.clone()
    ops.add_bwd(gx, a, b)
    assert np.array_equal(H(a), y + x) and np.array_equal(H(b), x + x)


def test_unaligned_pointers(cuda, ops, orc, rng):
    """Views starting one element in take the scalar path."""
    x = rng.standard_normal(1001).astype(np.float32)
    base = T(x, cuda)
    v = base[1:]
    out = torch.zeros(1000, device=cuda)[0:]
    out2 = torch.zeros(1001, device=cuda)[1:]
    ops.act_fwd(ops.GELU, v, out2)
    assert rel_err(H(out2), orc.act_fwd(4, x[1:])) <= RTOL_EXACT
    ops.copy(v, out)
    assert np.array_equal(H(out), x[1:])


@pytest.mark.parametrize("kind", range(6))
def test_activation_fwd_bwd(cuda, ops, orc, rng, kind):
    n = 3 * 1024 + 5
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    g = rng.standard_normal(n).astype(np.float32)
    gx0 = rng.standard_normal(n).astype(np.float32)
    y = torch.empty(n, device=cuda)
    ops.act_fwd(kind, T(x, cuda), y)
    assert rel_err(H(y), orc.act_fwd(kind, x)) <= RTOL_EXACT
    gx = T(gx0, cuda)
    ops.act_bwd(kind, T(x, cuda), T(g, cuda), gx)
    assert rel_err(H(gx), orc.act_bwd(kind, x, g, gx0.copy())) <= RTOL_EXACT


@pytest.mark.parametrize("rows,cols", [(64, 256), (4096, 1024), (33, 10), (5, 1027)])
def test_activation_bwd_fused_bias(cuda, ops, orc, rng, rows, cols):
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    g = rng.standard_normal((rows, cols)).astype(np.float32)
    gx0 = np.zeros((rows, cols), np.float32)
    db0 = rng.standard_normal(cols).astype(np.float32)
    gx, db = T(gx0, cuda), T(db0, cuda)
    ops.act_bwd(ops.GELU, T(x, cuda), T(g, cuda), gx, bias_grad=db)
    ref_gx = orc.act_bwd(4, x, g, gx0.copy())
    ref_db = orc.bias_grad(ref_gx, db0.copy())
    assert rel_err(H(gx), ref_gx) <= RTOL_EXACT
    assert rel_err(H(db), ref_db) <= 1e-4  # column sums over up to 4096 rows, reordered


@pytest.mark.parametrize("rows,cols", [(64, 256), (33, 10), (5, 1027)])
@pytest.mark.parametrize("fused", [False, True])
def test_activation_bwd_assign(cuda, ops, rng, rows, cols, fused):
    """mle_act_bwd_assign never reads gx and leaves bit for bit what
    mle_act_bwd leaves in a cleared gx (bias column sums included)."""
    from ml_engine_b200._lib import kernels
    k = kernels()
    x = T((rng.standard_normal((rows, cols)) * 3).astype(np.float32), cuda)
    g = T(rng.standard_normal((rows, cols)).astype(np.float32), cuda)
    n = rows * cols
    for kind in range(6):
        want = torch.zeros(rows, cols, device=cuda)
        got = torch.full((rows, cols), float("nan"), device=cuda)
        db_w, db_g = torch.zeros(cols, device=cuda), torch.zeros(cols, device=cuda)
        st = torch.cuda.current_stream().cuda_stream
        k.call("mle_act_bwd", kind, x.data_ptr(), g.data_ptr(), want.data_ptr(), n,
               db_w.data_ptr() if fused else None, rows if fused else 0, cols if fused else 0, st)
        k.call("mle_act_bwd_assign", kind, x.data_ptr(), g.data_ptr(), got.data_ptr(), n,
               db_g.data_ptr() if fused else None, rows if fused else 0, cols if fused else 0, st)
        assert torch.equal(got, want), kind
        if fused:
            assert rel_err(H(db_g), H(db_w)) <= 1e-6, kind  # column-sum atomics in any order


@pytest.mark.parametrize("rows,cols", [(64, 256), (1000, 10), (7, 4096)])
def test_bias_add_and_grad(cuda, ops, orc, rng, rows, cols):
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    b = rng.standard_normal(cols).astype(np.float32)
    y = torch.empty(rows, cols, device=cuda)
    ops.bias_add_fwd(T(x, cuda), T(b, cuda), y)
    assert np.array_equal(H(y), orc.bias_add(x, b))
    db0 = rng.standard_normal(cols).astype(np.float32)
    db = T(db0, cuda)
    ops.bias_grad(T(x, cuda), db)
    assert rel_err(H(db), orc.bias_grad(x, db0.copy())) <= 1e-5 * max(1, rows / 64)


@pytest.mark.parametrize("S", [35, 64])
def test_channel_bias(cuda, ops, orc, rng, S):
    B, C = 4, 6
    x = rng.standard_normal(B * C * S).astype(np.float32)
    b = rng.standard_normal(C).astype(np.float32)
    y = torch.empty(B * C * S, device=cuda)
    ops.channel_bias_fwd(T(x, cuda), T(b, cuda), y, B, C, S)
    assert np.array_equal(H(y), orc.channel_bias_fwd(x, b, B, C, S))
    gx0 = rng.standard_normal(B * C * S).astype(np.float32)
    gb0 = rng.standard_normal(C).astype(np.float32)
    gx, gb = T(gx0, cuda), T(gb0, cuda)
    ops.channel_bias_bwd(T(x, cuda), gx, gb, B, C, S)
    rgx, rgb = gx0.copy(), gb0.copy()
    orc.channel_bias_bwd(x, rgx, rgb, B, C, S)
    assert np.array_equal(H(gx), rgx)
    assert rel_err(H(gb), rgb) <= RTOL_EXACT


def test_channel_bias_first(cuda, ops, orc, rng):
    """Broadcast_Channel's reduction of the first min(dim[3], C) channels."""
    B, C, first, S = 5, 12, 7, 16
    g = rng.standard_normal(B * C * S).astype(np.float32)
    gb0 = rng.standard_normal(C).astype(np.float32)
    gb = T(gb0, cuda)
    ops.channel_bias_bwd_first(T(g, cuda), gb, B, C, first, S)
    want = gb0.copy()
    want[:first] += g.reshape(B, C, S)[:, :first].sum(axis=(0, 2), dtype=np.float64).astype(np.float32)
    got = H(gb)
    assert np.array_equal(got[first:], gb0[first:])
    assert rel_err(got, want) <= RTOL_EXACT


@pytest.mark.parametrize("S", [35, 64])
def test_channel_concat_split(cuda, ops, orc, rng, S):
    """CopyCrop's channel concatenation and its gradient split."""
    B, c1, c2 = 3, 5, 7
    a = rng.standard_normal(B * c1 * S).astype(np.float32)
    b = rng.standard_normal(B * c2 * S).astype(np.float32)
    c = torch.empty(B * (c1 + c2) * S, device=cuda)
    ops.channel_concat(T(a, cuda), T(b, cuda), c, B, c1, c2, S)
    assert np.array_equal(H(c), orc.channel_concat(a, b, B, c1, c2, S))
    gc = rng.standard_normal(B * (c1 + c2) * S).astype(np.float32)
    ga0 = rng.standard_normal(B * c1 * S).astype(np.float32)
    gb0 = rng.standard_normal(B * c2 * S).astype(np.float32)
    ga, gb = T(ga0, cuda), T(gb0, cuda)
    ops.channel_split(ga, gb, T(gc, cuda), B, c1, c2, S)
    ra, rb = ga0.copy(), gb0.copy()
    orc.channel_split(ra, rb, gc, B, c1, c2, S)
    assert np.array_equal(H(ga), ra) and np.array_equal(H(gb), rb)


@pytest.mark.parametrize("flag", [0, 1, 2, 3])
def test_headify(cuda, ops, orc, rng, flag):
    B, Hh, S, D = 3, 4, 5, 8
    n = B * Hh * S * D
    inp = rng.standard_normal(n).astype(np.float32)
    out0 = rng.standard_normal(n).astype(np.float32)
    out = T(out0, cuda)
    ops.headify(T(inp, cuda), out, B, Hh, S, D, flag)
    assert np.array_equal(H(out), orc.headify(inp, out0.copy(), B, Hh, S, D, flag))


def test_matpe(cuda, ops, orc, rng):
    B, S, D = 2, 17, 24
    x = rng.standard_normal(B * S * D).astype(np.float32)
    y = torch.empty(B * S * D, device=cuda)
    ops.matpe_fwd(T(x, cuda), y, B, S, D, 3)
    assert rel_err(H(y), orc.matpe(x, B, S, D, 3)) <= RTOL_EXACT


# -------------------------------------------------------------- normalisation
# segment lengths for every path: warp (<= 1024), one CTA (2048, 4096), clusters of
# 2 and 8 CTAs (8192, 60000 with a partial last CTA), streamed block (70000
# and the unaligned 4099)
@pytest.mark.parametrize("batch,channels,row,col", [(64, 1, 1, 256), (33, 1, 1, 1000), (7, 1, 4, 1024),
                                                    (6, 1, 1, 2048), (5, 1, 1, 8192), (3, 1, 1, 60000),
                                                    (2, 1, 1, 70000),
                                                    (3, 1, 1, 4099), (4, 3, 5, 8)])
def test_layernorm(cuda, ops, orc, rng, batch, channels, row, col):
    n = batch * channels * row * col
    x = (rng.standard_normal(n) * 2 + 0.5).astype(np.float32)
    gy = rng.standard_normal(n).astype(np.float32)
    y, mean, sq = torch.empty(n, device=cuda), torch.empty(batch, device=cuda), torch.empty(batch, device=cuda)
    ops.layernorm_fwd(T(x, cuda), y, mean, sq, batch, channels, row, col)
    ry, rmean, rsq = orc.layernorm_fwd(x, batch, channels, row, col)
    assert rel_err(H(y), ry) <= RTOL_EXACT
    assert rel_err(H(sq), rsq) <= RTOL_EXACT
    gx0 = rng.standard_normal(n).astype(np.float32)
    gx = T(gx0, cuda)
    ops.layernorm_bwd(y, T(gy, cuda), sq, gx, batch, channels, row, col)
    assert rel_err(H(gx), orc.layernorm_bwd(ry, gy, rsq, gx0.copy(), batch, channels, row, col)) <= RTOL_EXACT


@pytest.mark.parametrize("batch,channels,row,col", [(4096, 1, 1, 256), (8192, 1, 1, 512), (33, 1, 1, 1000),
                                                    (7, 1, 4, 32), (5, 1, 1, 100), (3, 1, 1, 2048)])
def test_add_layernorm_matches_two_launches(cuda, ops, rng, batch, channels, row, col):
    """The residual Add and its LayerNorm in one pass against mle_scale_add
    followed by mle_layernorm_fwd: the sum, the normalised output and the
    statistics bit for bit; segments the one-pass kernel does not take
    (over 1024 elements) are refused with nothing written."""
    from ml_engine_b200 import MLEError
    n = batch * channels * row * col
    x = T((rng.standard_normal(n) * 2 + 0.5).astype(np.float32), cuda)
    r = T(rng.standard_normal(n).astype(np.float32), cuda)
    xr, y = torch.full((n,), 7.0, device=cuda), torch.full((n,), 7.0, device=cuda)
    mean, sq = torch.zeros(batch, device=cuda), torch.zeros(batch, device=cuda)
    seg = channels * row * col
    if seg > 1024:
        with pytest.raises(MLEError):
            ops.add_layernorm_fwd(x, r, xr, y, mean, sq, batch, channels, row, col)
        assert torch.all(xr == 7.0) and torch.all(y == 7.0)
        return
    ops.add_layernorm_fwd(x, r, xr, y, mean, sq, batch, channels, row, col)
    rxr, ry = torch.empty(n, device=cuda), torch.empty(n, device=cuda)
    rmean, rsq = torch.zeros(batch, device=cuda), torch.zeros(batch, device=cuda)
    ops.scale_add(x, r, rxr, 1.0)
    ops.layernorm_fwd(rxr, ry, rmean, rsq, batch, channels, row, col)
    assert torch.equal(xr, rxr) and torch.equal(y, ry)
    assert torch.equal(mean, rmean) and torch.equal(sq, rsq)


@pytest.mark.parametrize("batch,channels,groups,row,col", [(4, 64, 8, 16, 16), (2, 24, 8, 3, 5), (2, 64, 8, 64, 64),
                                                           (3, 128, 8, 32, 32)])
def test_groupnorm(cuda, ops, orc, rng, batch, channels, groups, row, col):
    n = batch * channels * row * col
    x = (rng.standard_normal(n) * 2 + 0.5).astype(np.float32)
    gy = rng.standard_normal(n).astype(np.float32)
    y = torch.empty(n, device=cuda)
    mean, sq = torch.empty(batch * groups, device=cuda), torch.empty(batch * groups, device=cuda)
    ops.groupnorm_fwd(T(x, cuda), y, mean, sq, batch, channels, groups, row, col)
    ry, _, rsq = orc.groupnorm_fwd(x, batch, channels, groups, row, col)
    assert rel_err(H(y), ry) <= RTOL_EXACT
    gx0 = rng.standard_normal(n).astype(np.float32)
    gx = T(gx0, cuda)
    ops.groupnorm_bwd(y, T(gy, cuda), sq, gx, batch, channels, groups, row, col)
    assert rel_err(H(gx), orc.groupnorm_bwd(ry, gy, rsq, gx0.copy(), batch, channels, groups, row, col)) <= RTOL_EXACT


# --------------------------------------------------------- softmax and losses
@pytest.mark.parametrize("axis,causal", [(0, 0), (1, 0), (1, 1), (0, 1)])
@pytest.mark.parametrize("bc,rows,cols", [(6, 128, 128), (3, 17, 33), (2, 5, 4096)])
def test_softmax(cuda, ops, orc, rng, axis, causal, bc, rows, cols):
    n = bc * rows * cols
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    y = torch.empty(n, device=cuda)
    ops.softmax_fwd(T(x, cuda), y, bc, rows, cols, axis, causal)
    ry = orc.softmax_fwd(x, bc, rows, cols, axis, causal)
    assert rel_err(H(y), ry) <= RTOL_EXACT
    gy = rng.standard_normal(n).astype(np.float32)
    gx0 = rng.standard_normal(n).astype(np.float32)
    gx = T(gx0, cuda)
    ops.softmax_bwd(y, T(gy, cuda), gx, bc, rows, cols, axis)
    assert rel_err(H(gx), orc.softmax_bwd(ry, gy, gx0.copy(), bc, rows, cols, axis)) <= RTOL_EXACT


@pytest.mark.parametrize("rows,cols", [(64, 10), (256, 4096), (3, 8192 + 4), (9, 1001), (40, 8192)])
def test_softmax_cross_entropy(cuda, ops, orc, rng, rows, cols):
    logits = (rng.standard_normal((rows, cols)) * 2).astype(np.float32)
    labels = rng.integers(0, cols, rows)
    target = np.zeros((rows, cols), np.float32)
    target[np.arange(rows), labels] = 1.0
    probs = torch.empty(rows, cols, device=cuda)
    grad = torch.empty(rows, cols, device=cuda)
    loss = torch.empty(1, device=cuda)
    batch = 4.0
    ops.softmax_ce_fwd(T(logits, cuda), T(target, cuda), probs, loss, grad, batch, rows, cols)
    rp, rloss = orc.smce_fwd(logits, target, rows, cols)
    assert rel_err(H(probs), rp) <= RTOL_EXACT
    assert abs(float(H(loss)[0]) - rloss) <= RTOL_EXACT * abs(rloss)
    assert rel_err(H(grad), orc.smce_bwd(rp, target, batch)) <= RTOL_EXACT
    g2 = torch.empty(rows, cols, device=cuda)
    ops.softmax_ce_bwd(probs, T(target, cuda), g2, batch)
    assert rel_err(H(g2), orc.smce_bwd(rp, target, batch)) <= RTOL_EXACT


@pytest.mark.parametrize("rows,cols", [(64, 12), (256, 1024), (33, 4096), (40, 8192)])
def test_softmax_cross_entropy_index_labels(cuda, ops, rng, rows, cols):
    """The index-label entry points against the dense ones on the one-hot
    target of the same labels: probs and gradients bit for bit, the loss up
    to the order of its atomics (labels -1 and cols are rows of zeros)."""
    logits = (rng.standard_normal((rows, cols)) * 2).astype(np.float32)
    labels = rng.integers(0, cols, rows).astype(np.int32)
    labels[0], labels[-1] = -1, cols
    target = np.zeros((rows, cols), np.float32)
    ok = (labels >= 0) & (labels < cols)
    target[np.arange(rows)[ok], labels[ok]] = 1.0
    tl, tt = T(logits, cuda), T(target, cuda)
    out = {}
    for kind in ("dense", "index"):
        probs, grad = torch.empty(rows, cols, device=cuda), torch.empty(rows, cols, device=cuda)
        loss, g2 = torch.empty(1, device=cuda), torch.empty(rows, cols, device=cuda)
        up = torch.full((1,), 0.75, device=cuda)
        if kind == "dense":
            ops.softmax_ce_fwd(tl, tt, probs, loss, grad, 4.0, rows, cols)
            ops.softmax_ce_bwd(probs, tt, g2, 4.0, upstream=up)
        else:
            lab = T(labels, cuda)
            ops.softmax_ce_index_fwd(tl, lab, probs, loss, grad, 4.0, rows, cols)
            ops.softmax_ce_index_bwd(probs, lab, g2, 4.0, rows, cols, upstream=up)
        out[kind] = [H(t) for t in (probs, grad, g2, loss)]
    for a, b in zip(out["dense"][:3], out["index"][:3]):
        assert np.array_equal(a, b)
    # the loss sums per-row terms with float atomics in either kernel
    la, lb = float(out["dense"][3][0]), float(out["index"][3][0])
    assert abs(la - lb) <= 1e-6 * abs(la)


def test_mse(cuda, ops, orc, rng):
    n = 32 * 3 * 64 * 64
    x = rng.standard_normal(n).astype(np.float32)
    t = rng.standard_normal(n).astype(np.float32)
    loss = torch.empty(1, device=cuda)
    ops.mse_fwd(T(x, cuda), T(t, cuda), loss)
    assert abs(float(H(loss)[0]) - orc.mse_fwd(x, t)) <= 1e-5 * orc.mse_fwd(x, t)
    gx0 = rng.standard_normal(n).astype(np.float32)
    gx = T(gx0, cuda)
    ops.mse_bwd(T(x, cuda), T(t, cuda), gx)
    assert rel_err(H(gx), orc.mse_bwd(x, t, gx0.copy())) <= RTOL_EXACT


# ----------------------------------------------------------------------- GEMM
GEMM_SHAPES = [(128, 128, 32), (256, 512, 384), (200, 130, 70), (64, 256, 784), (784, 256, 64), (1000, 96, 8),
               (4096, 256, 256), (256, 256, 4096), (33, 1024, 129),
               (1, 128, 256), (3, 64, 1000),  # at most 8 rows: one warp per output
               (512, 256, 480),               # 15 k-blocks: a stage of two k-blocks holds only the last one
               (256, 256, 2080)]              # split-K ranges of an odd number of k-blocks


@pytest.fixture(params=[2, 1], ids=["kpl2", "kpl1"])
def stage_kblocks(request):
    """Two k-blocks per GEMM stage where both operands have split views
    (the default), or one everywhere."""
    from ml_engine_b200._lib import kernels
    k = kernels()
    old = k.mle_get_gemm_stage_kblocks()
    k.call("mle_set_gemm_stage_kblocks", request.param)
    yield request.param
    k.call("mle_set_gemm_stage_kblocks", old)


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("beta", [0.0, 1.0])
def test_gemm_tf32(cuda, ops, orc, rng, stage_kblocks, M, N, K, ta, tb, beta):
    from ml_engine_b200._lib import kernels
    A = rng.standard_normal((K, M) if ta else (M, K)).astype(np.float32)
    B = rng.standard_normal((N, K) if tb else (K, N)).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    C = T(C0, cuda)
    ops.gemm(T(A, cuda), T(B, cuda), C, M, N, K, ta, tb, alpha=0.5, beta=beta)
    kpl = kernels().mle_gemm_last_stage_kblocks()
    if kpl:  # a tensor-core product: two k-blocks per stage iff both operands split
        split = (M % 32 == 0 if ta else K % 32 == 0) and (K % 32 == 0 if tb else N % 32 == 0)
        assert kpl == (2 if split and stage_kblocks == 2 else 1)
    if (M, N, K) == (4096, 256, 256):
        assert kpl == stage_kblocks
    ref = C0.copy() if beta else np.zeros_like(C0)
    prod = np.zeros((M, N), np.float32)
    orc.gemm(A, B, prod, M, N, K, ta, tb)
    ref = ref + 0.5 * prod
    # relative to the product's scale: C0 can dominate the sum
    err = np.max(np.abs(H(C) - ref)) / max(np.max(np.abs(0.5 * prod)), 1e-30)
    assert err <= RTOL_TC, err


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("beta", [0.0, 1.0])
@pytest.mark.parametrize("M,N,K,mode", [(4000, 2000, 520, 1), (1000, 100, 300, 2), (700, 200, 96, 2),
                                        (1024, 512, 544, 2), (512, 192, 96, 2)])
def test_gemm_cta_pairs(cuda, ops, rng, stage_kblocks, ta, tb, beta, M, N, K, mode):
    """Products on CTA pairs (cta_group::2 MMAs, 256-row tiles) with ragged
    edges in M, N and K, against float64 products: chosen by the tile model
    for the large one, forced (mode 2) for 64- and 128-wide pair tiles."""
    from ml_engine_b200._lib import kernels
    A = rng.standard_normal((K, M) if ta else (M, K)).astype(np.float32)
    B = rng.standard_normal((N, K) if tb else (K, N)).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    C = T(C0, cuda)
    k = kernels()
    old = k.mle_get_gemm_pairs()
    k.mle_set_gemm_pairs(mode)
    try:
        ops.gemm(T(A, cuda), T(B, cuda), C, M, N, K, ta, tb, alpha=0.5, beta=beta)
        got = H(C)
        choice = (ctypes.c_int * 3)()
        k.call("mle_gemm_last_choice", choice)
    finally:
        k.mle_set_gemm_pairs(old)
    assert choice[2] == 1, list(choice)  # the product ran on CTA pairs
    a64 = (A.T if ta else A).astype(np.float64)
    b64 = (B.T if tb else B).astype(np.float64)
    prod = a64 @ b64
    ref = (C0.astype(np.float64) if beta else 0.0) + 0.5 * prod
    err = np.max(np.abs(got - ref)) / np.max(np.abs(0.5 * prod))
    assert err <= RTOL_TC, err


def _tf32(x, mode):
    """fp32 -> TF32 (low 13 mantissa bits cleared): 'trunc' or nearest-even."""
    b = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    if mode == "rne":
        b = b + 0xFFF + ((b >> 13) & 1)
    return (b & 0xFFFFE000).astype(np.uint32).view(np.float32)


@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 1)])
@pytest.mark.parametrize("mode,emul", [(0, "trunc"), (1, "rne")])
def test_gemm_operand_rounding(cuda, ops, rng, ta, tb, mode, emul):
    """Operand loads of fp32 type leave the tensor core to drop the low 13
    mantissa bits; TF32-typed tensor maps round to nearest, ties to even
    (row 0 of A holds exact ties).  The product then equals the float64
    product of the converted operands up to fp32 accumulation."""
    from ml_engine_b200._lib import kernels
    M, N, K = 256, 256, 512
    A = rng.standard_normal((M, K)).astype(np.float32)
    A[0, :64] = (A[0, :64].view(np.uint32) & np.uint32(0xFFFFE000) | np.uint32(0x1000)).view(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    C = torch.zeros(M, N, device=cuda)
    k = kernels()
    old = k.mle_get_gemm_operand_rounding()
    k.call("mle_set_gemm_operand_rounding", mode)
    try:
        ops.gemm(T(np.ascontiguousarray(A.T) if ta else A, cuda), T(np.ascontiguousarray(B.T) if tb else B, cuda),
                 C, M, N, K, ta, tb)
        got = H(C).astype(np.float64)
    finally:
        k.call("mle_set_gemm_operand_rounding", old)
    ref = _tf32(A, emul).astype(np.float64) @ _tf32(B, emul).astype(np.float64)
    assert np.max(np.abs(got - ref)) / np.max(np.abs(ref)) <= 2e-5
    assert np.max(np.abs(got[0] - ref[0])) / np.max(np.abs(ref[0])) <= 2e-5


@pytest.mark.parametrize("bn,splits,pair", [(64, 1, 0), (128, 2, 0), (256, 4, 1), (64, 3, 1)])
def test_gemm_forced_tiles(cuda, ops, rng, bn, splits, pair):
    """mle_set_gemm_tiles overrides the tile model (the product reports the
    forced width, split count and pairing) and the result stays within the
    TF32 tolerance; width 0 hands the choice back to the model."""
    from ml_engine_b200._lib import kernels
    k = kernels()
    M, N, K = 1000, 384, 800
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    C = T(C0, cuda)
    k.call("mle_set_gemm_tiles", bn, splits, pair)
    try:
        ops.gemm(T(A, cuda), T(B, cuda), C, M, N, K, 0, 0, alpha=1.0, beta=1.0)
        got = H(C)
        choice = (ctypes.c_int * 3)()
        k.call("mle_gemm_last_choice", choice)
    finally:
        k.call("mle_set_gemm_tiles", 0, 0, 0)
    assert list(choice) == [bn, splits, pair]
    prod = A.astype(np.float64) @ B.astype(np.float64)
    assert np.max(np.abs(got - C0 - prod)) / np.max(np.abs(prod)) <= RTOL_TC


def test_gemm_fallback_exact(cuda, ops, orc, rng):
    """N = 10 (MNIST logits) has a 40-byte row stride: CUDA-core path, fp32."""
    M, N, K = 64, 10, 256
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    C = torch.empty(M, N, device=cuda)
    ops.gemm(T(A, cuda), T(B, cuda), C, M, N, K)
    prod = np.zeros((M, N), np.float32)
    orc.gemm(A, B, prod, M, N, K)
    assert rel_err(H(C), prod) <= RTOL_EXACT


def test_gemm_bias_and_batch(cuda, ops, orc, rng):
    batch, M, N, K = 3, 130, 96, 40
    A = rng.standard_normal((batch, M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)  # broadcast over batch
    bias = rng.standard_normal(N).astype(np.float32)
    C = torch.empty(batch, M, N, device=cuda)
    ops.gemm(T(A, cuda), T(B, cuda), C, M, N, K, bias=T(bias, cuda), batch=batch, stride_a=M * K, stride_b=0,
             stride_c=M * N)
    for b in range(batch):
        prod = np.zeros((M, N), np.float32)
        orc.gemm(A[b].copy(), B, prod, M, N, K)
        assert rel_err(H(C)[b], prod + bias) <= RTOL_TC


BCMM_CASES = [
    # variant, batch, channels, m, n, p, backward, A_case, B_case, C_case
    (0, 4, 1, 128, 64, 96, 0, 3, 0, 3),    # Linear forward (W broadcast)
    (1, 4, 1, 128, 96, 64, 1, 3, 0, 3),    # Linear dX
    (2, 4, 1, 64, 128, 96, 1, 3, 3, 0),    # Linear dW (batch reduction folded into K)
    (1, 2, 8, 128, 32, 128, 0, 3, 3, 3),   # attention scores Q K^T
    (0, 2, 8, 128, 128, 32, 0, 3, 3, 3),   # P V
    (3, 2, 8, 32, 128, 128, 1, 3, 3, 3),   # bcmmT (BMMABT dK)
    (2, 2, 3, 40, 50, 60, 1, 1, 3, 2),     # mixed broadcast with C reduction over batch
    (0, 3, 2, 20, 30, 10, 1, 0, 0, 0),     # everything broadcast: product counted batch*channels times
]


@pytest.mark.parametrize("case", BCMM_CASES)
def test_bcmm_broadcast_semantics(cuda, ops, orc, rng, case):
    variant, batch, ch, m, n, p, bwd, ac, bc, cc = case

    def size(flag, inner):
        return (batch if flag & 1 else 1) * (ch if flag & 2 else 1) * inner

    A = rng.standard_normal(size(ac, m * n)).astype(np.float32)
    B = rng.standard_normal(size(bc, n * p)).astype(np.float32)
    C0 = rng.standard_normal(size(cc, m * p)).astype(np.float32) if bwd else np.zeros(size(cc, m * p), np.float32)
    C = T(C0, cuda)
    ops.bcmm(variant, T(A, cuda), T(B, cuda), C, batch, ch, m, n, p, bwd, ac, bc, cc, 0.75)
    ref = orc.bcmm(variant, A, B, C0.copy(), batch, ch, m, n, p, bwd, ac, bc, cc, 0.75)
    delta = ref - C0 if bwd else ref
    err = np.max(np.abs(H(C) - ref)) / max(np.max(np.abs(delta)), 1e-30)
    assert err <= RTOL_TC, err


@pytest.mark.parametrize("rows,fin,fout", [(64, 784, 256), (4096, 256, 1024), (4096, 1024, 256), (100, 40, 72)])
def test_linear_fwd_bwd(cuda, ops, orc, rng, rows, fin, fout):
    X = rng.random((rows, fin)).astype(np.float32)
    W = (rng.standard_normal((fin, fout)) * np.sqrt(2.0 / fin)).astype(np.float32)
    b = rng.standard_normal(fout).astype(np.float32) * 0.1
    Y = torch.empty(rows, fout, device=cuda)
    ops.linear_fwd(T(X, cuda), T(W, cuda), T(b, cuda), Y, rows, fin, fout)
    ry = np.zeros((rows, fout), np.float32)
    orc.gemm(X, W, ry, rows, fout, fin)
    ry = orc.bias_add(ry, b)
    assert rel_err(H(Y), ry) <= RTOL_TC
    dY = rng.standard_normal((rows, fout)).astype(np.float32)
    dX0 = rng.standard_normal((rows, fin)).astype(np.float32)
    dX, dW, dB = T(dX0, cuda), torch.zeros(fin, fout, device=cuda), torch.zeros(fout, device=cuda)
    ops.linear_bwd(T(X, cuda), T(W, cuda), T(dY, cuda), dX, dW, dB, rows, fin, fout)
    rdx = dX0.copy()
    orc.gemm(dY, W, rdx, rows, fin, fout, 0, 1, accumulate=True)
    rdw = np.zeros((fin, fout), np.float32)
    orc.gemm(X, dY, rdw, fin, fout, rows, 1, 0)
    rdb = orc.bias_grad(dY, np.zeros(fout, np.float32))
    assert np.max(np.abs(H(dX) - rdx)) / np.max(np.abs(rdx - dX0)) <= RTOL_TC
    assert rel_err(H(dW), rdw) <= RTOL_TC
    # the bias gradient is summed from the dW product's (TF32-rounded) dY tiles
    assert rel_err(H(dB), rdb) <= RTOL_TC


def _tf32_rne(x):
    """fp32 -> the nearest TF32 value (10 mantissa bits, ties to even), as
    the tensor maps of TF32 element type round operands on their way to
    shared memory (finite inputs)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0xFFF + ((u >> 13) & 1)) & ~np.uint64(0x1FFF)
    return u.astype(np.uint32).view(np.float32)


@pytest.mark.parametrize("rows,fin,fout,pairs", [(4096, 256, 256, 0), (4096, 256, 1024, 0), (4096, 1024, 256, 0),
                                                 (8192, 256, 64, 0), (1000, 40, 72, 0), (4133, 300, 100, 0),
                                                 (8192, 512, 2048, 2)])
@pytest.mark.parametrize("rounding", [1, 0])
def test_linear_bwd_bias_from_weight_product(cuda, ops, orc, rng, stage_kblocks, rows, fin, fout, pairs, rounding):
    """The bias gradient taken by the weight-gradient product's epilogue
    warps from dY's tiles in shared memory (the column sums of each tile's
    k-range, added atomically) against the oracle's column sums, added onto
    a non-zero dB: many row-tiles (only the first sums), split reductions,
    ragged rows and columns, one and two k-blocks per stage, and CTA pairs
    forced (each CTA of a pair sums the columns it staged).  The tiles hold
    the operand values the product uses: dY rounded to TF32 under operand
    rounding 1, dY itself under 0; the oracle sums the same values, so the
    bound is the fp32 summation-order one."""
    from ml_engine_b200._lib import kernels
    k = kernels()
    old_pairs, old_round = k.mle_get_gemm_pairs(), k.mle_get_gemm_operand_rounding()
    k.mle_set_gemm_pairs(pairs)
    k.call("mle_set_gemm_operand_rounding", rounding)
    try:
        X = rng.standard_normal((rows, fin)).astype(np.float32)
        W = (rng.standard_normal((fin, fout)) * 0.05).astype(np.float32)
        dY = rng.standard_normal((rows, fout)).astype(np.float32)
        dB0 = rng.standard_normal(fout).astype(np.float32)
        dW, dB = torch.zeros(fin, fout, device=cuda), T(dB0, cuda)
        ops.linear_bwd(T(X, cuda), T(W, cuda), T(dY, cuda), None, dW, dB, rows, fin, fout)
        rdw = np.zeros((fin, fout), np.float32)
        orc.gemm(X, dY, rdw, fin, fout, rows, 1, 0)
        ch = (ctypes.c_int * 3)()
        k.mle_gemm_last_choice(ch)
        fused = k.mle_gemm_last_column_sums() == 1  # summed by the product's epilogue warps
        rdb = orc.bias_grad(_tf32_rne(dY) if fused and rounding else dY, dB0.copy())
        assert rel_err(H(dW), rdw) <= RTOL_TC
        assert rel_err(H(dB), rdb) <= 1e-5
    finally:
        k.mle_set_gemm_pairs(old_pairs)
        k.call("mle_set_gemm_operand_rounding", old_round)


# ------------------------------------------------------------------ attention
ATTN_CASES = [  # B, H, Sq, Sk, hd, axis, causal
    (2, 8, 128, 128, 32, 1, 0),   # configs[1] shape per head
    (2, 4, 64, 64, 64, 1, 1),     # masked (SoftMask)
    (1, 2, 256, 256, 64, 1, 1),   # configs[2] head shape
    (1, 2, 40, 72, 16, 1, 0),     # Sq != Sk: the reference key gradient needs the composed path
    (2, 3, 37, 37, 32, 1, 1),     # ragged row and key blocks, masked: CUDA-core kernels only
    (1, 2, 40, 72, 16, 0, 0),     # row-wise softmax: composed (tensor cores)
    (1, 2, 272, 64, 32, 1, 1),    # tensor path: single-pass column softmax of 512-thread blocks, ragged rows
    (1, 1, 544, 64, 16, 1, 0),    # tensor path: columns over 512 rows take the multi-pass kernels
]


@pytest.fixture(params=["fused", "tensor"])
def attn_path(request, ops):
    """Runs each attention case with the CUDA-core kernels in the reference's
    order (exact) and with the tensor-core path (TF32 tolerance) forced."""
    old = ops.set_attention_path(ops.ATTN_PATH_FUSED if request.param == "fused" else ops.ATTN_PATH_TENSOR)
    yield request.param
    ops.set_attention_path(old)


def _attn_tol(ops, path, Sq, Sk, D, axis, key_mode, backward):
    """(tolerance, runs token-major) for the path the entry points take."""
    fused = ops.attention_fused_supported(Sq, Sk, D, axis, key_mode if backward else 1)
    if path == "tensor" and ops.attention_tensor_supported(Sq, Sk, D, axis, key_mode, backward):
        return RTOL_TC, True
    return (1e-5 if fused else RTOL_TC), fused


def _attn_inputs(rng, B, Hh, Sq, Sk, D):
    bh = B * Hh
    return [rng.standard_normal((bh, s, D)).astype(np.float32) for s in (Sq, Sk, Sk, Sq)]


def _to_token_major(x, B, Hh):
    bh, S, D = x.shape
    return np.ascontiguousarray(x.reshape(B, Hh, S, D).transpose(0, 2, 1, 3).reshape(B, S, Hh * D))


def _from_token_major(x, B, Hh, D):
    S = x.shape[1]
    return np.ascontiguousarray(x.reshape(B, S, Hh, D).transpose(0, 2, 1, 3).reshape(B * Hh, S, D))


@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("case", ATTN_CASES)
def test_attention_fwd(cuda, ops, orc, rng, case, layout, attn_path):
    B, Hh, Sq, Sk, D, axis, causal = case
    tol, token_major_ok = _attn_tol(ops, attn_path, Sq, Sk, D, axis, 1, False)
    if layout == 1 and not token_major_ok:
        pytest.skip("token-major layout needs the fused or the tensor-core path")
    Q, K, V, _ = _attn_inputs(rng, B, Hh, Sq, Sk, D)
    scale = float(1.0 / np.sqrt(D))
    conv = (lambda x: _to_token_major(x, B, Hh)) if layout else (lambda x: x)
    P = torch.zeros(B * Hh, Sq, Sk, device=cuda)
    O = torch.zeros(*conv(np.zeros((B * Hh, Sq, D), np.float32)).shape, device=cuda)
    ops.attention_fwd(T(conv(Q), cuda), T(conv(K), cuda), T(conv(V), cuda), P, O, B, Hh, Sq, Sk, D, scale, causal,
                      axis, layout)
    S = orc.bcmm(1, Q, K, np.zeros((B * Hh, Sq, Sk), np.float32), B, Hh, Sq, D, Sk, 0, 3, 3, 3)
    rP = orc.softmax_fwd(orc.scale_write(S, scale), B * Hh, Sq, Sk, axis, causal)
    rO = orc.bcmm(0, rP, V, np.zeros((B * Hh, Sq, D), np.float32), B, Hh, Sq, Sk, D, 0, 3, 3, 3)
    o = H(O)
    if layout:
        o = _from_token_major(o, B, Hh, D)
    assert rel_err(H(P), rP) <= tol
    assert rel_err(o, rO) <= tol


@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("key_mode", [0, 1])
@pytest.mark.parametrize("case", ATTN_CASES)
def test_attention_bwd(cuda, ops, orc, rng, case, key_mode, layout, attn_path):
    B, Hh, Sq, Sk, D, axis, causal = case
    tol, token_major_ok = _attn_tol(ops, attn_path, Sq, Sk, D, axis, key_mode, True)
    if layout == 1 and not token_major_ok:
        pytest.skip("token-major layout needs the fused or the tensor-core path")
    bh = B * Hh
    Q, K, V, dO = _attn_inputs(rng, B, Hh, Sq, Sk, D)
    scale = float(1.0 / np.sqrt(D))
    S = orc.bcmm(1, Q, K, np.zeros((bh, Sq, Sk), np.float32), B, Hh, Sq, D, Sk, 0, 3, 3, 3)
    P = orc.softmax_fwd(orc.scale_write(S, scale), bh, Sq, Sk, axis, causal)
    conv = (lambda x: _to_token_major(x, B, Hh)) if layout else (lambda x: x)
    back = (lambda x: _from_token_major(x, B, Hh, D)) if layout else (lambda x: x)
    dQ0, dK0, dV0 = (rng.standard_normal((bh, s, D)).astype(np.float32) for s in (Sq, Sk, Sk))
    dQ, dK, dV = T(conv(dQ0), cuda), T(conv(dK0), cuda), T(conv(dV0), cuda)
    dP, dS = torch.zeros(bh, Sq, Sk, device=cuda), torch.zeros(bh, Sq, Sk, device=cuda)
    ops.attention_bwd(T(conv(Q), cuda), T(conv(K), cuda), T(conv(V), cuda), T(P, cuda), T(conv(dO), cuda), dQ, dK,
                      dV, dP, dS, B, Hh, Sq, Sk, D, scale, causal, axis, key_mode, layout)
    # reference chain (Engine/engine.cu:2246-2253, 2450-2455, 2540-2546, 2302-2309)
    rdP = orc.bcmm(1, dO, V, np.zeros((bh, Sq, Sk), np.float32), B, Hh, Sq, D, Sk, 1, 3, 3, 3)
    rdV = orc.bcmm(2, P, dO, np.zeros((bh, Sk, D), np.float32), B, Hh, Sk, Sq, D, 1, 3, 3, 3)
    rdSc = orc.softmax_bwd(P, rdP, np.zeros_like(P), bh, Sq, Sk, axis)
    rdS = orc.accumulate(rdSc, np.zeros_like(P), scale)
    rdQ = orc.bcmm(0, rdS, K, np.zeros((bh, Sq, D), np.float32), B, Hh, Sq, Sk, D, 1, 3, 3, 3)
    if key_mode == 0:  # bcmmT(Q, dScores, K.grad, hd, Sq, Sk): the reference's own call
        rdK = orc.bcmm(3, Q, rdS, np.zeros((bh, Sk, D), np.float32), B, Hh, D, Sq, Sk, 1, 3, 3, 3)
    else:              # the mathematical gradient dS^T Q
        rdK = orc.bcmm(2, rdS, Q, np.zeros((bh, Sk, D), np.float32), B, Hh, Sk, Sq, D, 1, 3, 3, 3)
    assert rel_err(H(dP), rdP) <= tol
    assert rel_err(H(dS), rdSc) <= tol
    assert rel_err(back(H(dV)) - dV0, rdV) <= tol
    assert rel_err(back(H(dQ)) - dQ0, rdQ) <= tol
    assert rel_err(back(H(dK)) - dK0, rdK) <= tol


@pytest.mark.parametrize("case", [(2, 8, 128, 128, 32, 1, 0), (2, 4, 64, 64, 64, 1, 1)])
@pytest.mark.parametrize("mask", [1, 2, 4, 7])
def test_attention_bwd_assign(cuda, ops, rng, attn_path, case, mask):
    """mle_attention_bwd_assign writes the gradients of its mask over
    whatever they held and accumulates the others: the same results as
    mle_attention_bwd into cleared buffers (the tensor-core products may
    tile the beta = 0 form differently, hence the 1e-6)."""
    from ml_engine_b200._lib import kernels
    B, Hh, Sq, Sk, D, axis, causal = case
    bh = B * Hh
    Q, K, V, dO = (T(_to_token_major(x, B, Hh), cuda) for x in _attn_inputs(rng, B, Hh, Sq, Sk, D))
    scale = float(1.0 / np.sqrt(D))
    P = torch.empty(bh, Sq, Sk, device=cuda)
    O = torch.empty_like(Q)
    ops.attention_fwd(Q, K, V, P, O, B, Hh, Sq, Sk, D, scale, causal, axis, 1)
    old = [T(rng.standard_normal(t.numel()).astype(np.float32).reshape(t.shape), cuda) for t in (Q, K, K)]
    want = [torch.zeros_like(t) if mask >> i & 1 else t.clone() for i, t in enumerate(old)]
    ws = torch.empty(bh * Sq * Sk, device=cuda)
    st = torch.cuda.current_stream().cuda_stream
    k = kernels()
    p = [x.data_ptr() for x in (Q, K, V, P, dO)]
    k.call("mle_attention_bwd", *p, *[t.data_ptr() for t in want], None, None, ws.data_ptr(), B, Hh, Sq, Sk, D,
           ctypes.c_float(scale), causal, axis, 0, 1, st)
    got = [t.clone() for t in old]
    k.call("mle_attention_bwd_assign", *p, *[t.data_ptr() for t in got], None, None, ws.data_ptr(), B, Hh, Sq, Sk, D,
           ctypes.c_float(scale), causal, axis, 0, 1, mask, st)
    for i in range(3):
        assert rel_err(H(got[i]), H(want[i])) <= 1e-6, i


@pytest.mark.parametrize("mask", [0, 1, 2, 3])
def test_add_bwd_assign(cuda, ops, rng, mask):
    """Add backward with assigned outputs: bit for bit the accumulation
    into cleared buffers; the others still accumulate."""
    from ml_engine_b200._lib import kernels
    for n in (4099, 1 << 16):
        g = T(rng.standard_normal(n).astype(np.float32), cuda)
        a0, b0 = (T(rng.standard_normal(n).astype(np.float32), cuda) for _ in range(2))
        wa = torch.zeros_like(a0) if mask & 1 else a0.clone()
        wb = torch.zeros_like(b0) if mask & 2 else b0.clone()
        ops.add_bwd(g, wa, wb)
        ga, gb = a0.clone(), b0.clone()
        kernels().call("mle_add_bwd_assign", g.data_ptr(), ga.data_ptr(), gb.data_ptr(), n, mask,
                       torch.cuda.current_stream().cuda_stream)
        assert torch.equal(ga, wa) and torch.equal(gb, wb)


def test_matpe_table_matches_direct(cuda, ops, rng):
    B, S, D = 3, 50, 64
    x = rng.standard_normal(B * S * D).astype(np.float32)
    y1, y2 = torch.empty(B * S * D, device=cuda), torch.empty(B * S * D, device=cuda)
    table = torch.empty(S * D, device=cuda)
    ops.matpe_fwd(T(x, cuda), y1, B, S, D, 2)
    ops.matpe_table(table, S, D, 2)
    ops.rows_add_table(T(x, cuda), table, y2, B)
    assert np.array_equal(H(y1), H(y2))


# ------------------------------------------------------------------ optimizer
def _make_params(rng, sizes, dev):
    ps, host = [], []
    for n in sizes:
        w = (rng.standard_normal(n) * 0.02).astype(np.float32)
        g = (rng.standard_normal(n) * 0.5).astype(np.float32)
        m = (rng.standard_normal(n) * 0.01).astype(np.float32)
        v = np.abs(rng.standard_normal(n) * 0.001).astype(np.float32)
        host.append(dict(w=w, g=g, m=m, v=v))
        ps.append(dict(w=T(w, dev), g=T(g, dev), m=T(m, dev), v=T(v, dev),
                       t=torch.tensor([3], dtype=torch.int32, device=dev)))
    return ps, host


@pytest.mark.parametrize("adamw", [True, False])
@pytest.mark.parametrize("clip", [True, False])
def test_clip_adam_multi_tensor(cuda, ops, orc, rng, adamw, clip):
    sizes = [784 * 256, 256, 2560, 10, 1, 5000, 4096 * 3 + 1]
    ps, host = _make_params(rng, sizes, cuda)
    ws = torch.zeros(1, dtype=torch.float64, device=cuda)
    if clip:
        ops.grad_sumsq(ps, ws)
        ops.clip_finalize(ws)
    ops.adam_update(ps, lr=1e-3, adamw=adamw, clip_ws=ws if clip else None)
    acc = np.zeros(1, np.float64)
    if clip:
        for h in host:
            orc.sumsq(acc, h["g"])
        orc.clip_finalize(acc)
        assert abs(H(ws)[0] - acc[0]) <= 1e-12 * acc[0]
    for p, h in zip(ps, host):
        g = h["g"].copy()
        if clip:
            orc.clip_apply(g, acc)
        w, m, v = h["w"].copy(), h["m"].copy(), h["v"].copy()
        orc.adam(w, g, m, v, 3, 1e-3, adamw)
        assert rel_err(H(p["m"]), m) <= RTOL_EXACT
        assert rel_err(H(p["v"]), v) <= RTOL_EXACT
        assert rel_err(H(p["w"]), w) <= RTOL_EXACT
        if clip:
            assert rel_err(H(p["g"]), g) <= RTOL_EXACT
        assert int(H(p["t"])[0]) == 4


def _clone_params(ps):
    return [{k: x.clone() for k, x in p.items()} for p in ps]


@pytest.mark.parametrize("adamw", [True, False])
@pytest.mark.parametrize("clip", [True, False])
@pytest.mark.parametrize("pre_scale", [1.0, 0.25])
def test_fused_clip_adam_matches_separate_launches(cuda, ops, orc, rng, adamw, clip, pre_scale):
    """The one-launch norm + clip + update (cooperative kernel, table in
    device memory) against the sum-of-squares, finalize and update launches
    over 130 tensors (more than one launch table of the separate path), two
    steps through the same workspace.  Without a clip the arithmetic is the
    same element by element: bit-identical.  With one, the norm's partial
    sums are added in another order, so the coefficient agrees to rounding,
    and the first step is also checked against the oracle."""
    sizes = [784 * 256, 256, 2560, 10, 1, 5000, 4096 * 3 + 1] + [int(x) for x in rng.integers(1, 3000, 123)]
    if clip:
        sizes[0] = 1 << 20  # a norm well above max_norm
    ps, host = _make_params(rng, sizes, cuda)
    ref = _clone_params(ps)
    ws = ops.clip_adam_workspace(ops.param_views(ps))
    max_norm = 1.0 if clip else 0.0
    for step in range(2):
        ops.clip_adam(ws, lr=1e-3, max_norm=max_norm, pre_scale=pre_scale, adamw=adamw)
        cw = torch.zeros(1, dtype=torch.float64, device=cuda)
        if clip:
            ops.grad_sumsq(ref, cw, scale=pre_scale)
            ops.clip_finalize(cw, max_norm)
        ops.adam_update(ref, lr=1e-3, adamw=adamw, clip_ws=cw if clip else None, pre_scale=pre_scale)
        if step == 0 and clip:
            acc = np.zeros(1, np.float64)
            for h in host:
                orc.sumsq(acc, (h["g"] * np.float32(pre_scale)).astype(np.float32))
            orc.clip_finalize(acc)
            for p, h in list(zip(ps, host))[:9]:
                g = (h["g"] * np.float32(pre_scale)).astype(np.float32)
                orc.clip_apply(g, acc)
                w, m, v = h["w"].copy(), h["m"].copy(), h["v"].copy()
                orc.adam(w, g, m, v, 3, 1e-3, adamw)
                for k, want in (("g", g), ("w", w), ("m", m), ("v", v)):
                    assert rel_err(H(p[k]), want) <= RTOL_EXACT, k
    assert ops.clip_adam_status(ws) == 0
    for p, r in zip(ps, ref):
        assert int(H(p["t"])[0]) == 5 and int(H(r["t"])[0]) == 5
        for k in ("w", "m", "v", "g"):
            if not clip:
                assert torch.equal(p[k], r[k]), k
            else:
                assert rel_err(H(p[k]), H(r[k])) <= RTOL_EXACT, k


def test_fused_clip_adam_nan_norm_and_errors(cuda, ops, rng):
    """A NaN in one gradient makes the coefficient NaN and every tensor's
    weights NaN, as with the separate launches; a short workspace and a
    null one are refused."""
    from ml_engine_b200 import MLEError
    ps, _ = _make_params(rng, [1000, 33, 4097], cuda)
    ps[1]["g"][5] = float("nan")
    ws = ops.clip_adam_workspace(ps)
    ops.clip_adam(ws, lr=1e-3, max_norm=1.0)
    assert ops.clip_adam_status(ws) == 0
    for p in ps:
        assert torch.isnan(p["w"]).all()
    views = ops.param_views(ps)
    st = torch.cuda.current_stream().cuda_stream
    with pytest.raises(MLEError):
        ops.kernels().call("mle_clip_adam_prepare", ctypes.cast(views, ctypes.c_void_p), 3, ws.data_ptr(), 64, st)
    with pytest.raises(MLEError):
        ops.kernels().call("mle_clip_adam_run", None, 1.0, 1.0, 1e-3, 1, 1, st)


def test_clip_apply_and_nan(cuda, ops, orc, rng):
    ps, host = _make_params(rng, [1000, 33], cuda)
    ws = torch.zeros(1, dtype=torch.float64, device=cuda)
    ops.grad_sumsq(ps, ws)
    ops.clip_finalize(ws)
    ops.clip_apply(ps, ws)
    acc = np.zeros(1, np.float64)
    for h in host:
        orc.sumsq(acc, h["g"])
    orc.clip_finalize(acc)
    for p, h in zip(ps, host):
        assert rel_err(H(p["g"]), orc.clip_apply(h["g"].copy(), acc)) <= RTOL_EXACT
    nan_ws = torch.tensor([float("nan")], dtype=torch.float64, device=cuda)
    ops.clip_finalize(nan_ws)
    assert np.isnan(H(nan_ws)[0])


def test_small_norm_is_not_scaled(cuda, ops, rng):
    ps, _ = _make_params(rng, [10], cuda)
    ps[0]["g"].mul_(1e-3)
    ws = torch.zeros(1, dtype=torch.float64, device=cuda)
    ops.grad_sumsq(ps, ws)
    ops.clip_finalize(ws)
    assert H(ws)[0] == 1.0


def test_argument_errors(cuda, ops):
    from ml_engine_b200 import MLEError
    x = torch.zeros(4, device=cuda)
    with pytest.raises(MLEError):
        ops.act_fwd(17, x, x)
    with pytest.raises(MLEError):
        ops.gemm(x, x, x, 2, 2, 2, beta=0.5)


def test_watchdog_clear(cuda, ops):
    assert ops.watchdog() == 0


@pytest.mark.parametrize("n,rows,pairs,outs", [(1, 1024, 0, None), (2, 1024, 0, None), (3, 1024, 0, None),
                                                (3, 8192, 1, None), (3, 8192, 1, (512, 512, 512)),
                                                (2, 1024, 0, (256, 96))])
def test_linear_group_matches_separate_linears(cuda, ops, rng, n, rows, pairs, outs):
    """mle_linear_group_fwd/_bwd against n separate mle_linear_fwd/_bwd
    calls (TF32 products; dX is one product over the concatenated
    reduction when every out_features is a multiple of 64, else the n
    products reduce-added); the 8192-row cases are large enough for the
    group to run on CTA pairs (512 x 3: the query/key/value projections of
    configs[2])."""
    from ml_engine_b200._lib import kernels
    old_pairs = kernels().mle_get_gemm_pairs()
    kernels().mle_set_gemm_pairs(pairs)
    try:
        _linear_group_case(cuda, ops, rng, n, rows, outs)
    finally:
        kernels().mle_set_gemm_pairs(old_pairs)


def _linear_group_case(cuda, ops, rng, n, rows, outs=None):
    from ml_engine_b200._lib import kernels
    din = 256
    outs = list(outs) if outs else [256, 128, 512][:n]
    X = T(rng.standard_normal((rows, din)).astype(np.float32), cuda)
    Ws = [T((rng.standard_normal((din, o)) * 0.05).astype(np.float32), cuda) for o in outs]
    Bs = [T(rng.standard_normal(o).astype(np.float32), cuda) for o in outs]
    dYs = [T(rng.standard_normal((rows, o)).astype(np.float32), cuda) for o in outs]
    dX0 = rng.standard_normal((rows, din)).astype(np.float32)
    arr = lambda ts: (ctypes.c_void_p * n)(*[t.data_ptr() for t in ts])
    Ys = [torch.empty(rows, o, device=cuda) for o in outs]
    out_arr = (ctypes.c_int * n)(*outs)
    st = torch.cuda.current_stream().cuda_stream
    kernels().call("mle_linear_group_fwd", X.data_ptr(), arr(Ws), arr(Bs), arr(Ys), n, rows, din, out_arr, st)
    dX = T(dX0, cuda)
    dWs = [torch.zeros(din, o, device=cuda) for o in outs]
    dBs = [torch.zeros(o, device=cuda) for o in outs]
    kernels().call("mle_linear_group_bwd", X.data_ptr(), arr(Ws), arr(dYs), dX.data_ptr(), arr(dWs), arr(dBs), n,
                   rows, din, out_arr, st)
    rX = T(dX0, cuda)
    for i, o in enumerate(outs):
        y = torch.empty(rows, o, device=cuda)
        ops.linear_fwd(X, Ws[i], Bs[i], y, rows, din, o)
        assert norm_err(H(Ys[i]), H(y)) <= RTOL_TC
        dw, db = torch.zeros(din, o, device=cuda), torch.zeros(o, device=cuda)
        ops.linear_bwd(X, Ws[i], dYs[i], rX, dw, db, rows, din, o)
        assert norm_err(H(dWs[i]), H(dw)) <= RTOL_TC
        # the bias gradients come from the dW products' TF32-rounded dY tiles,
        # or from a separate fp32 column sum where a launch has more tiles than CTAs
        assert norm_err(H(dBs[i]), H(db)) <= 1e-3
    assert norm_err(H(dX) - dX0, H(rX) - dX0) <= RTOL_TC


KEYS_CASES = [  # B, H, Sq, Sk, hd, causal: shapes the keys-on-lanes kernels take
    (2, 8, 128, 128, 32, 0),   # configs[1] heads
    (1, 4, 256, 256, 64, 1),   # configs[2] masked self-attention heads
    (1, 4, 256, 256, 64, 0),   # configs[2] cross-attention heads (unmasked here)
    (2, 3, 200, 136, 64, 1),   # ragged: queries below the 256-wide tile, a partial second key block
    (1, 2, 96, 256, 128, 0),   # head_dim 128, queries below the 128-wide tile
]


@pytest.mark.parametrize("key_mode", [0, 1])
@pytest.mark.parametrize("case", KEYS_CASES)
def test_attention_keys_kernels(cuda, ops, orc, rng, case, key_mode):
    """The tensor-core path with the keys-on-lanes kernels (P and the score
    gradient computed with the scores / dP kept in TMEM, no dP or dS
    output requested) against the C oracle's reference chain (TF32 bound)
    and against the same path with the products written to HBM and
    softmaxed in place (summation order only)."""
    from ml_engine_b200._lib import kernels
    B, Hh, Sq, Sk, D, causal = case
    if key_mode == 0 and Sq != Sk:
        pytest.skip("the reference key gradient is defined for Sq == Sk")
    bh = B * Hh
    Q, K, V, dO = _attn_inputs(rng, B, Hh, Sq, Sk, D)
    scale = float(1.0 / np.sqrt(D))
    tm = lambda x: T(_to_token_major(x, B, Hh), cuda)   # noqa: E731
    back = lambda x: _from_token_major(H(x), B, Hh, D)   # noqa: E731
    k = kernels()
    old_path = ops.set_attention_path(ops.ATTN_PATH_TENSOR)
    runs = {}
    try:
        for keys in (1, 0):
            k.call("mle_set_attention_keys_kernel", keys)
            P = torch.zeros(bh, Sq, Sk, device=cuda)
            O = torch.zeros(B, Sq, Hh * D, device=cuda)
            ops.attention_fwd(tm(Q), tm(K), tm(V), P, O, B, Hh, Sq, Sk, D, scale, causal, 1, 1)
            dQ, dK, dV = (torch.zeros(B, s, Hh * D, device=cuda) for s in (Sq, Sk, Sk))
            ops.attention_bwd(tm(Q), tm(K), tm(V), P, tm(dO), dQ, dK, dV, None, None, B, Hh, Sq, Sk, D, scale,
                              causal, 1, key_mode, 1)
            torch.cuda.synchronize()
            runs[keys] = (H(P), back(O), back(dQ), back(dK), back(dV))
    finally:
        k.call("mle_set_attention_keys_kernel", 1)
        ops.set_attention_path(old_path)
    S = orc.bcmm(1, Q, K, np.zeros((bh, Sq, Sk), np.float32), B, Hh, Sq, D, Sk, 0, 3, 3, 3)
    rP = orc.softmax_fwd(orc.scale_write(S, scale), bh, Sq, Sk, 1, causal)
    rO = orc.bcmm(0, rP, V, np.zeros((bh, Sq, D), np.float32), B, Hh, Sq, Sk, D, 0, 3, 3, 3)
    rdP = orc.bcmm(1, dO, V, np.zeros((bh, Sq, Sk), np.float32), B, Hh, Sq, D, Sk, 1, 3, 3, 3)
    rdV = orc.bcmm(2, rP, dO, np.zeros((bh, Sk, D), np.float32), B, Hh, Sk, Sq, D, 1, 3, 3, 3)
    rdS = orc.accumulate(orc.softmax_bwd(rP, rdP, np.zeros_like(rP), bh, Sq, Sk, 1), np.zeros_like(rP), scale)
    rdQ = orc.bcmm(0, rdS, K, np.zeros((bh, Sq, D), np.float32), B, Hh, Sq, Sk, D, 1, 3, 3, 3)
    if key_mode == 0:
        rdK = orc.bcmm(3, Q, rdS, np.zeros((bh, Sk, D), np.float32), B, Hh, D, Sq, Sk, 1, 3, 3, 3)
    else:
        rdK = orc.bcmm(2, rdS, Q, np.zeros((bh, Sk, D), np.float32), B, Hh, Sk, Sq, D, 1, 3, 3, 3)
    for name, got, want in zip("P O dQ dK dV".split(), runs[1], (rP, rO, rdQ, rdK, rdV)):
        assert rel_err(got, want) <= RTOL_TC, (name, rel_err(got, want))
    # the two paths differ in summation order only (the column sums, the
    # dP product's tiling); the score gradient's cancellation p (dP - d)
    # magnifies that in dQ and dK
    for name, a, b in zip("P O dQ dK dV".split(), runs[1], runs[0]):
        assert rel_err(a, b) <= 1e-3, (name, rel_err(a, b))


FLASH_CASES = [  # B, H, Sq, Sk, hd, causal
    (2, 8, 128, 128, 32, 0),   # configs[1] heads
    (2, 8, 128, 128, 32, 1),
    (1, 4, 256, 256, 64, 1),   # configs[2] masked self-attention heads
    (1, 4, 256, 256, 64, 0),   # configs[2] cross-attention heads (unmasked)
    (3, 2, 192, 192, 64, 1),   # a partial second block of queries and keys
    (2, 3, 200, 136, 64, 1),   # ragged: Sq, Sk no multiple of the 64-wide chunk
    (1, 2, 96, 448, 64, 0),    # queries below one block, seven key chunks
    (12, 8, 256, 256, 64, 1),  # 192 units: persistent CTAs walk more than one
    (40, 8, 128, 128, 32, 0),  # 320 units of configs[1]'s shape: up to three per CTA
]


def _flash_reference(orc, Q, K, V, dO, B, Hh, Sq, Sk, D, scale, causal, key_mode):
    """The reference's chain on the C oracle: P, O, the column statistics,
    dQ, dK (either key gradient), dV."""
    bh = B * Hh
    S = orc.scale_write(orc.bcmm(1, Q, K, np.zeros((bh, Sq, Sk), np.float32), B, Hh, Sq, D, Sk, 0, 3, 3, 3), scale)
    rP = orc.softmax_fwd(S, bh, Sq, Sk, 1, causal)
    rO = orc.bcmm(0, rP, V, np.zeros((bh, Sq, D), np.float32), B, Hh, Sq, Sk, D, 0, 3, 3, 3)
    rdP = orc.bcmm(1, dO, V, np.zeros((bh, Sq, Sk), np.float32), B, Hh, Sq, D, Sk, 1, 3, 3, 3)
    rdV = orc.bcmm(2, rP, dO, np.zeros((bh, Sk, D), np.float32), B, Hh, Sk, Sq, D, 1, 3, 3, 3)
    rdS = orc.accumulate(orc.softmax_bwd(rP, rdP, np.zeros_like(rP), bh, Sq, Sk, 1), np.zeros_like(rP), scale)
    rdQ = orc.bcmm(0, rdS, K, np.zeros((bh, Sq, D), np.float32), B, Hh, Sq, Sk, D, 1, 3, 3, 3)
    if key_mode == 0:
        rdK = orc.bcmm(3, Q, rdS, np.zeros((bh, Sk, D), np.float32), B, Hh, D, Sq, Sk, 1, 3, 3, 3)
    else:
        rdK = orc.bcmm(2, rdS, Q, np.zeros((bh, Sk, D), np.float32), B, Hh, Sk, Sq, D, 1, 3, 3, 3)
    S3 = S.reshape(bh, Sq, Sk).astype(np.float64)
    m = S3.max(axis=1)                                  # every query, masked ones included
    e = np.exp(S3 - m[:, None, :])
    if causal:
        e = e * (np.arange(Sk)[None, None, :] <= np.arange(Sq)[None, :, None])
    l = e.sum(axis=1)
    return rO, rdQ, rdK, rdV, m, 1.0 / np.where(l < 1e-45, 1.0, l)


@pytest.mark.parametrize("key_mode", [0, 1])
@pytest.mark.parametrize("case", FLASH_CASES)
def test_attention_flash(cuda, ops, orc, rng, case, key_mode):
    """The flash entry points (scores, probabilities and score gradients
    never in HBM; the backward recomputes P from the forward's column max
    and inverse sum) against the C oracle's reference chain at the TF32
    bound, in the token-major layout the graph nodes use, with dQ, dK, dV
    accumulated onto existing values; the statistics against float64."""
    B, Hh, Sq, Sk, D, causal = case
    if key_mode == 0 and not (Sq == Sk and Sk % D == 0):
        pytest.skip("the reference key gradient is defined for Sq == Sk, Sk % hd == 0")
    assert ops.attention_flash_supported(Sq, Sk, D, 1, key_mode)
    bh = B * Hh
    Q, K, V, dO = _attn_inputs(rng, B, Hh, Sq, Sk, D)
    scale = float(1.0 / np.sqrt(D))
    tm = lambda x: T(_to_token_major(x, B, Hh), cuda)   # noqa: E731
    back = lambda x: _from_token_major(H(x), B, Hh, D)   # noqa: E731
    O = torch.full((B, Sq, Hh * D), float("nan"), device=cuda)
    stats = torch.zeros(2 * bh * Sk, device=cuda)
    ops.attention_flash_fwd(tm(Q), tm(K), tm(V), O, stats, B, Hh, Sq, Sk, D, scale, causal, 1)
    pre = [rng.standard_normal((bh, s, D)).astype(np.float32) for s in (Sq, Sk, Sk)]
    dQ, dK, dV = (tm(x) for x in pre)
    ops.attention_flash_bwd(tm(Q), tm(K), tm(V), tm(dO), stats, dQ, dK, dV, B, Hh, Sq, Sk, D, scale, causal,
                            key_mode, 1, 0)
    rO, rdQ, rdK, rdV, rm, rinv = _flash_reference(orc, Q, K, V, dO, B, Hh, Sq, Sk, D, scale, causal, key_mode)
    st = H(stats).reshape(2, bh, Sk)
    assert rel_err(st[0], rm) <= RTOL_TC
    assert rel_err(st[1], rinv) <= RTOL_TC
    got = (back(O), back(dQ) - pre[0], back(dK) - pre[1], back(dV) - pre[2])
    for name, a, r in zip("O dQ dK dV".split(), got, (rO, rdQ, rdK, rdV)):
        assert np.isfinite(a).all(), name
        assert norm_err(a, r) <= RTOL_TC, (name, norm_err(a, r))
        assert rel_err(a, r) <= 2 * RTOL_TC, (name, rel_err(a, r))


@pytest.mark.parametrize("case", [(2, 8, 128, 128, 32, 1), (1, 4, 256, 256, 64, 1)])
def test_attention_flash_assign_and_layouts(cuda, ops, rng, case):
    """assign_mask writes dQ, dK, dV instead of adding (the buffers' NaN
    contents must vanish); the head-major layout gives the token-major
    results; the flash path and the keys-on-lanes tensor-core path agree to
    summation order."""
    B, Hh, Sq, Sk, D, causal = case
    bh = B * Hh
    Q, K, V, dO = _attn_inputs(rng, B, Hh, Sq, Sk, D)
    scale = float(1.0 / np.sqrt(D))
    tm = lambda x: T(_to_token_major(x, B, Hh), cuda)   # noqa: E731
    back = lambda x: _from_token_major(H(x), B, Hh, D)   # noqa: E731
    outs = {}
    for layout in (1, 0):
        cv = tm if layout == 1 else (lambda x: T(x, cuda))                           # noqa: E731
        bk = back if layout == 1 else H
        O = torch.empty((B, Sq, Hh * D), device=cuda)
        stats = torch.empty(2 * bh * Sk, device=cuda)
        ops.attention_flash_fwd(cv(Q), cv(K), cv(V), O, stats, B, Hh, Sq, Sk, D, scale, causal, layout)
        dQ, dK, dV = (torch.full((B, s, Hh * D), float("nan"), device=cuda) for s in (Sq, Sk, Sk))
        ops.attention_flash_bwd(cv(Q), cv(K), cv(V), cv(dO), stats, dQ, dK, dV, B, Hh, Sq, Sk, D, scale, causal,
                                0, layout, 7)
        outs[layout] = [bk(x).reshape(bh, -1, D) for x in (O, dQ, dK, dV)]
    for name, a, b in zip("O dQ dK dV".split(), outs[1], outs[0]):
        assert np.isfinite(a).all(), name
        assert np.array_equal(a, b), name
    old_path = ops.set_attention_path(ops.ATTN_PATH_TENSOR)
    try:
        P = torch.zeros(bh, Sq, Sk, device=cuda)
        O = torch.zeros(B, Sq, Hh * D, device=cuda)
        ops.attention_fwd(tm(Q), tm(K), tm(V), P, O, B, Hh, Sq, Sk, D, scale, causal, 1, 1)
        dQ, dK, dV = (torch.zeros(B, s, Hh * D, device=cuda) for s in (Sq, Sk, Sk))
        ops.attention_bwd(tm(Q), tm(K), tm(V), P, tm(dO), dQ, dK, dV, None, None, B, Hh, Sq, Sk, D, scale,
                          causal, 1, 0, 1)
        ref = [back(x) for x in (O, dQ, dK, dV)]
    finally:
        ops.set_attention_path(old_path)
    for name, a, b in zip("O dQ dK dV".split(), outs[1], ref):
        assert rel_err(a, b) <= 1e-3, (name, rel_err(a, b))


@pytest.mark.parametrize("gemm_mode", [0, 1], ids=["tf32", "fp32"])
def test_linear_bwd_long_reduction(cuda, ops, gemm_mode):
    """configs[2]'s weight gradient on one GPU reduces over K = 65536 tokens
    (dW = X^T dY, 512 x 512): against a float64 product of the same fp32
    inputs (torch on the GPU; the C oracle would take minutes at this
    size), per-tensor normwise within the TF32 bound and max-relative within
    it too; fp32 mode (FMA chains of 65536 terms) within 1e-4."""
    from ml_engine_b200._lib import kernels
    rows, fin, fout = 65536, 512, 512
    g = torch.Generator(device=cuda).manual_seed(3)
    X = torch.randn(rows, fin, device=cuda, generator=g)
    W = torch.randn(fin, fout, device=cuda, generator=g) * 0.02
    dY = torch.randn(rows, fout, device=cuda, generator=g) * 1e-3
    dX, dW = torch.zeros(rows, fin, device=cuda), torch.zeros(fin, fout, device=cuda)
    k = kernels()
    old = k.mle_get_gemm_mode()
    try:
        k.call("mle_set_gemm_mode", gemm_mode)
        ops.linear_bwd(X, W, dY, dX, dW, None, rows, fin, fout)
        torch.cuda.synchronize()
    finally:
        k.call("mle_set_gemm_mode", old)
    rdW = (X.double().t() @ dY.double()).cpu().numpy()
    rdX = (dY.double() @ W.double().t()).cpu().numpy()
    for got, want in ((H(dW), rdW), (H(dX), rdX)):
        if gemm_mode == 0:
            assert norm_err(got, want) <= RTOL_TC and rel_err(got, want) <= RTOL_TC
        else:   # fp32 FMA chains 65536 long
            assert rel_err(got, want) <= 1e-4
