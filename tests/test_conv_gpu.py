"""Convolute2D / Convolute2DT on the tensor-core GEMM against the CPU
oracle's restatement of CV2D, GV2D, CV2D_GradInput, CVT2D, GVT2D and
CVT2D_GradInput (and, where oracle/_ref is built, the reference kernels
themselves).  TF32 products: <= 2e-3 normwise per tensor; fp32 GEMM mode:
<= 1e-5 normwise."""
import numpy as np
import pytest

from conftest import RTOL_EXACT, RTOL_TC, norm_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

CONV = [  # N, Cin, H, W, Cout, K, pad, stride
    (2, 3, 16, 16, 8, 3, 1, 1),      # first layer of a U-Net: 3 channels, two rows per 32-pixel block
    (4, 16, 32, 32, 32, 3, 1, 1),    # 3x3 implicit GEMM, one row per block
    (2, 32, 17, 13, 16, 3, 1, 2),    # stride-2 downsampling, odd sizes (im2col)
    (2, 16, 64, 64, 32, 3, 1, 2),    # U-Net downsampling: the stride-1 implicit GEMM over the 4 phase images
    (2, 32, 16, 16, 64, 1, 0, 2),    # strided 1x1 skip projection: one phase image, read in place
    (2, 8, 15, 15, 16, 3, 1, 2),     # odd input, phases of 8 x 8
    (1, 8, 32, 32, 32, 4, 1, 2),     # 4x4 taps: a 3x3 kernel per phase
    (2, 64, 8, 8, 32, 1, 0, 1),      # 1x1 skip projection read in place
    (2, 64, 64, 64, 64, 3, 1, 1),    # U-Net top level: 32 pixel tiles per image, half-height M tile
    (2, 192, 16, 16, 160, 3, 1, 1),  # two M tiles, six channel blocks per tap
    (2, 40, 12, 12, 24, 3, 1, 1),    # width 12: pixel blocks straddle rows
    (2, 8, 10, 10, 8, 3, 1, 1),      # width 10: rows not 16-byte aligned, im2col
    (3, 24, 8, 8, 3, 1, 0, 1),       # 3 output channels (the U-Net's output projection)
    (2, 16, 4, 4, 16, 3, 1, 1),      # 16-pixel images: blocks run past the image
    (2, 8, 32, 32, 16, 5, 2, 1),     # 5x5 taps
]
CONVT = [  # N, Cin, H, W, Cout, K, pad, stride
    (2, 32, 8, 8, 16, 2, 0, 2),      # 2x2 stride-2 upsampling
    (2, 16, 7, 9, 8, 3, 1, 2),
    (2, 8, 10, 10, 8, 3, 1, 1),
]


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def H(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.fixture(params=[(0, 1), (0, 2), (1, 1)], ids=["tf32", "tf32-pairs", "fp32"])
def gemm_mode(request):
    """GEMM mode and CTA-pair setting: the tile model's choice, or every
    tensor-core product forced onto CTA pairs (256-row tiles)."""
    from ml_engine_b200._lib import kernels
    k = kernels()
    old, old_pairs = k.mle_get_gemm_mode(), k.mle_get_gemm_pairs()
    mode, pairs = request.param
    k.mle_set_gemm_mode(mode)
    k.mle_set_gemm_pairs(pairs)
    yield mode
    k.mle_set_gemm_mode(old)
    k.mle_set_gemm_pairs(old_pairs)


@pytest.mark.parametrize("case", [c for c in CONV if c[7] == 2])
def test_conv2d_stride2_phase_form_matches_im2col(cuda, rng, case):
    """The stride-2 phase form (stride-1 implicit GEMM over the polyphase
    sub-images) against im2col + GEMM + col2im on the same inputs, TF32
    mode: both products take the same TF32-rounded operand values, so y, dx
    and dW differ only by fp32 summation order (and a shape the phase form
    cannot take runs im2col both times).  Every case has at least 16 output
    channels: narrower im2col products run on the fp32 CUDA-core GEMM."""
    from ml_engine_b200 import ops
    from ml_engine_b200._lib import kernels
    k = kernels()
    old_mode, old_phase = k.mle_get_gemm_mode(), k.mle_get_conv_phase()
    N, Cin, Hh, W, Cout, K, pad, stride = case
    x = T(rng.standard_normal((N, Cin, Hh, W)).astype(np.float32), cuda)
    w = T((rng.standard_normal((Cout, Cin, K, K)) * 0.2).astype(np.float32), cuda)
    b = T(rng.standard_normal(Cout).astype(np.float32), cuda)
    OH, OW = ops.conv_out_size(Hh, K, pad, stride), ops.conv_out_size(W, K, pad, stride)
    dy = T(rng.standard_normal((N, Cout, OH, OW)).astype(np.float32), cuda)
    dx0 = T(rng.standard_normal((N, Cin, Hh, W)).astype(np.float32), cuda)
    out = {}
    try:
        k.mle_set_gemm_mode(0)
        for phase in (2, 0):  # forced for every stride-2 shape, then im2col
            k.call("mle_set_conv_phase", phase)
            y = torch.empty(N, Cout, OH, OW, device=cuda)
            ws = ops.conv2d_workspace(x, w, pad, stride)
            ops.conv2d_fwd(x, w, b, y, ws, pad, stride)
            dx, dw, db = dx0.clone(), torch.zeros(Cout, Cin, K, K, device=cuda), torch.zeros(Cout, device=cuda)
            ops.conv2d_bwd(x, w, dy, dx, dw, db, ws, pad, stride)
            out[phase] = (H(y), H(dx), H(dw))
    finally:
        k.mle_set_gemm_mode(old_mode)
        k.call("mle_set_conv_phase", old_phase)
    for a, r, name in zip(out[2], out[0], ("y", "dx", "dW")):
        assert norm_err(a, r) <= 1e-5, (name, norm_err(a, r))


@pytest.mark.parametrize("case", CONV)
def test_conv2d(cuda, rng, gemm_mode, case):
    from ml_engine_b200 import ops
    from oracle import ops as orc
    N, Cin, Hh, W, Cout, K, pad, stride = case
    x = rng.standard_normal((N, Cin, Hh, W)).astype(np.float32)
    w = (rng.standard_normal((Cout, Cin, K, K)) * 0.2).astype(np.float32)
    b = rng.standard_normal(Cout).astype(np.float32)
    OH, OW = ops.conv_out_size(Hh, K, pad, stride), ops.conv_out_size(W, K, pad, stride)
    dy = rng.standard_normal((N, Cout, OH, OW)).astype(np.float32)
    dx0 = rng.standard_normal(x.shape).astype(np.float32)
    db0 = rng.standard_normal(Cout).astype(np.float32)
    tx, tw, tb = T(x, cuda), T(w, cuda), T(b, cuda)
    y = torch.empty(N, Cout, OH, OW, device=cuda)
    ws = ops.conv2d_workspace(tx, tw, pad, stride)
    ops.conv2d_fwd(tx, tw, tb, y, ws, pad, stride)
    dx, dw, db = T(dx0, cuda), torch.full((Cout, Cin, K, K), 7.0, device=cuda), T(db0, cuda)
    ops.conv2d_bwd(tx, tw, T(dy, cuda), dx, dw, db, ws, pad, stride)
    tol = RTOL_TC if gemm_mode == 0 else 1e-5
    assert norm_err(H(y), orc.conv2d_fwd(x, w, b, pad, stride)) <= tol
    assert norm_err(H(dw), orc.conv2d_bwd_k(x, dy, w.shape, pad, stride)) <= tol      # assigned
    assert norm_err(H(dx) - dx0, orc.conv2d_bwd_x(dy, w, np.zeros_like(x), pad, stride)) <= tol
    rdb = db0.copy()
    orc.channel_bias_bwd(dy, None, rdb, N, Cout, OH * OW)
    assert norm_err(H(db), rdb) <= 1e-5


@pytest.mark.parametrize("case", [CONV[1], CONV[2], CONV[3]], ids=["implicit", "columns", "in-place"])
def test_conv2d_backward_parts_on_two_streams(cuda, rng, gemm_mode, case):
    """The input-gradient part and the weight/bias part of the backward as
    two calls on two concurrent streams (as the engine issues them) give
    the single call's results: their workspace regions are disjoint."""
    from ml_engine_b200 import ops
    N, Cin, Hh, W, Cout, K, pad, stride = case
    x = rng.standard_normal((N, Cin, Hh, W)).astype(np.float32)
    w = (rng.standard_normal((Cout, Cin, K, K)) * 0.2).astype(np.float32)
    OH, OW = ops.conv_out_size(Hh, K, pad, stride), ops.conv_out_size(W, K, pad, stride)
    dy = T(rng.standard_normal((N, Cout, OH, OW)).astype(np.float32), cuda)
    tx, tw = T(x, cuda), T(w, cuda)
    y = torch.empty(N, Cout, OH, OW, device=cuda)
    ws = ops.conv2d_workspace(tx, tw, pad, stride)
    ops.conv2d_fwd(tx, tw, T(np.zeros(Cout, np.float32), cuda), y, ws, pad, stride)
    dx1, dw1, db1 = torch.zeros_like(tx), torch.zeros_like(tw), torch.zeros(Cout, device=cuda)
    ops.conv2d_bwd(tx, tw, dy, dx1, dw1, db1, ws, pad, stride)
    torch.cuda.synchronize()
    dx2, dw2, db2 = torch.zeros_like(tx), torch.zeros_like(tw), torch.zeros(Cout, device=cuda)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    for _ in range(2):  # twice: the workspace stays valid for another backward
        dx2.zero_(), db2.zero_()
        torch.cuda.synchronize()
        with torch.cuda.stream(s1):
            ops.conv2d_bwd(tx, tw, dy, dx2, None, None, ws, pad, stride)
        with torch.cuda.stream(s2):
            ops.conv2d_bwd(tx, tw, dy, None, dw2, db2, ws, pad, stride)
        torch.cuda.synchronize()
        # split-K reduce-adds and bias atomics may sum in another order
        for got, want in ((dx2, dx1), (dw2, dw1), (db2, db1)):
            assert norm_err(H(got), H(want)) <= 1e-6


@pytest.mark.parametrize("case", [CONV[1], CONV[2], CONV[3], CONV[7]], ids=["implicit", "columns", "in-place",
                                                                            "width10"])
def test_conv2d_bwd_assign(cuda, rng, gemm_mode, case):
    """mle_conv2d_bwd_assign with assign_dx = 1 writes dx over whatever it
    held: the input gradient mle_conv2d_bwd accumulates into a cleared dx."""
    from ml_engine_b200 import ops
    from ml_engine_b200._lib import kernels
    N, Cin, Hh, W, Cout, K, pad, stride = case
    x = T(rng.standard_normal((N, Cin, Hh, W)).astype(np.float32), cuda)
    w = T((rng.standard_normal((Cout, Cin, K, K)) * 0.2).astype(np.float32), cuda)
    OH, OW = ops.conv_out_size(Hh, K, pad, stride), ops.conv_out_size(W, K, pad, stride)
    dy = T(rng.standard_normal((N, Cout, OH, OW)).astype(np.float32), cuda)
    y = torch.empty(N, Cout, OH, OW, device=cuda)
    ws = ops.conv2d_workspace(x, w, pad, stride)
    ops.conv2d_fwd(x, w, T(np.zeros(Cout, np.float32), cuda), y, ws, pad, stride)
    want = torch.zeros_like(x)
    ops.conv2d_bwd(x, w, dy, want, None, None, ws, pad, stride)
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        got = torch.full_like(x, float("nan"))
        kernels().call("mle_conv2d_bwd_assign", x.data_ptr(), w.data_ptr(), dy.data_ptr(), got.data_ptr(), None, None,
                       ws.data_ptr(), N, Cin, Hh, W, Cout, K, K, pad, stride, 1, st)
        assert norm_err(H(got), H(want)) <= 1e-6


@pytest.mark.parametrize("case", CONVT)
def test_convT2d(cuda, rng, gemm_mode, case):
    from ml_engine_b200 import ops
    from oracle import ops as orc
    N, Cin, Hh, W, Cout, K, pad, stride = case
    x = rng.standard_normal((N, Cin, Hh, W)).astype(np.float32)
    w = (rng.standard_normal((Cout, Cin, K, K)) * 0.2).astype(np.float32)
    b = rng.standard_normal(Cout).astype(np.float32)
    OH, OW = ops.convT_out_size(Hh, K, pad, stride), ops.convT_out_size(W, K, pad, stride)
    dy = rng.standard_normal((N, Cout, OH, OW)).astype(np.float32)
    tx, tw = T(x, cuda), T(w, cuda)
    y = torch.empty(N, Cout, OH, OW, device=cuda)
    ws = ops.convT2d_workspace(tx, tw, pad, stride)
    ops.convT2d_fwd(tx, tw, T(b, cuda), y, ws, pad, stride)
    dx = torch.full(x.shape, 3.0, device=cuda)
    dw = torch.full(w.shape, 5.0, device=cuda)
    db = torch.zeros(Cout, device=cuda)
    ops.convT2d_bwd(tx, tw, T(dy, cuda), dx, dw, db, ws, pad, stride)
    tol = RTOL_TC if gemm_mode == 0 else 1e-5
    assert norm_err(H(y), orc.convT2d_fwd(x, w, b, pad, stride)) <= tol
    assert norm_err(H(dw), orc.convT2d_bwd_w(x, dy, w.shape, pad, stride)) <= tol     # assigned
    assert norm_err(H(dx), orc.convT2d_bwd_x(dy, w, x.shape, pad, stride)) <= tol     # assigned
    rdb = np.zeros(Cout, np.float32)
    orc.channel_bias_bwd(dy, None, rdb, N, Cout, OH * OW)
    assert norm_err(H(db), rdb) <= 1e-5


@pytest.mark.parametrize("case", CONV[1:3])
def test_conv2d_reference_kernels(cuda, rng, case):
    """Oracle vs the reference's own CV2D / GV2D / CV2D_GradInput."""
    from oracle import ops as orc
    from oracle import ref
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    N, Cin, Hh, W, Cout, K, pad, stride = case
    x = rng.standard_normal((N, Cin, Hh, W)).astype(np.float32)
    w = (rng.standard_normal((Cout, Cin, K, K)) * 0.2).astype(np.float32)
    b = rng.standard_normal(Cout).astype(np.float32)
    OH, OW = (2 * pad + Hh - K) // stride + 1, (2 * pad + W - K) // stride + 1
    dy = rng.standard_normal((N, Cout, OH, OW)).astype(np.float32)
    y = torch.empty(N, Cout, OH, OW, device=cuda)
    ref.call("ref_conv2d_fwd", ref.ptr(T(x, cuda)), ref.ptr(T(w, cuda)), ref.ptr(T(b, cuda)), ref.ptr(y), N, Cout,
             Cin, Hh, W, K, K, pad, stride)
    dk = torch.empty(w.shape, device=cuda)
    ref.call("ref_conv2d_bwd_k", ref.ptr(T(x, cuda)), ref.ptr(T(dy, cuda)), ref.ptr(dk), N, Cout, Cin, Hh, W, K, K,
             pad, stride)
    dx = torch.zeros(x.shape, device=cuda)
    ref.call("ref_conv2d_bwd_x", ref.ptr(T(dy, cuda)), ref.ptr(T(w, cuda)), ref.ptr(dx), N, Cout, Cin, Hh, W, K, K,
             pad, stride)
    assert norm_err(H(y), orc.conv2d_fwd(x, w, b, pad, stride)) <= RTOL_EXACT
    assert norm_err(H(dk), orc.conv2d_bwd_k(x, dy, w.shape, pad, stride)) <= RTOL_EXACT
    assert norm_err(H(dx), orc.conv2d_bwd_x(dy, w, np.zeros_like(x), pad, stride)) <= RTOL_EXACT


@pytest.mark.parametrize("case", CONVT[:2])
def test_convT2d_reference_kernels(cuda, rng, case):
    """Oracle vs the reference's own CVT2D / GVT2D / CVT2D_GradInput."""
    from oracle import ops as orc
    from oracle import ref
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    N, Cin, Hh, W, Cout, K, pad, stride = case
    x = rng.standard_normal((N, Cin, Hh, W)).astype(np.float32)
    w = (rng.standard_normal((Cout, Cin, K, K)) * 0.2).astype(np.float32)
    b = rng.standard_normal(Cout).astype(np.float32)
    OH, OW = (Hh - 1) * stride - 2 * pad + K, (W - 1) * stride - 2 * pad + K
    dy = rng.standard_normal((N, Cout, OH, OW)).astype(np.float32)
    y = torch.empty(N, Cout, OH, OW, device=cuda)
    ref.call("ref_convT2d_fwd", ref.ptr(T(x, cuda)), ref.ptr(T(w, cuda)), ref.ptr(T(b, cuda)), ref.ptr(y), N, Cout,
             Cin, Hh, W, K, K, pad, stride)
    gw = torch.empty(w.shape, device=cuda)
    ref.call("ref_convT2d_bwd_w", ref.ptr(T(x, cuda)), ref.ptr(T(dy, cuda)), ref.ptr(gw), N, Cout, Cin, Hh, W, K, K,
             pad, stride)
    gx = torch.empty(x.shape, device=cuda)
    ref.call("ref_convT2d_bwd_x", ref.ptr(T(dy, cuda)), ref.ptr(T(w, cuda)), ref.ptr(gx), N, Cout, Cin, Hh, W, K, K,
             pad, stride)
    assert norm_err(H(y), orc.convT2d_fwd(x, w, b, pad, stride)) <= RTOL_EXACT
    assert norm_err(H(gw), orc.convT2d_bwd_w(x, dy, w.shape, pad, stride)) <= RTOL_EXACT
    assert norm_err(H(gx), orc.convT2d_bwd_x(dy, w, x.shape, pad, stride)) <= RTOL_EXACT
