"""Whole training steps of the native sessions (C++ runtime + sm_100a
kernels) against the same steps composed from the CPU oracle
(oracle/graphs.py), on identical seeded parameters and inputs.

Checked per step: loss, every parameter gradient, the Adam first moment and
the step counters.  Tolerances:
  * fp32 GEMM mode (the MLP default): 1e-4 max-relative per tensor -- the
    products are fp32 FMA chains in k order like the reference's, the
    oracle accumulates in double;
  * TF32 tensor cores (the transformer default): 2e-3 normwise per tensor.
    A tensor whose exact gradient is zero (the query bias: the reference's
    column-wise softmax is invariant to a shift shared by all queries) has
    no relative scale; it is bounded by 1e-4 of the global gradient norm.
Weights after AdamW are checked through the update size: with t = 1 the
update is lr * sign-like(g), so an element whose tiny gradient changes sign
under TF32 rounding moves by up to 2*lr; the test bounds that and the
fraction of such elements.
"""
import numpy as np
import pytest

from conftest import RTOL_TC, norm_err, rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _session(**kw):
    from ml_engine_b200.session import Session
    return Session(**kw)


def _check_step(s, ref, p0, lr, exact, rtol=RTOL_TC, rtol_names=None):
    """Per gradient tensor: max-relative <= 1e-4 (fp32 products) or
    normwise <= rtol (TF32; rtol_names maps a name fragment to its own
    bound).  A tensor whose exact gradient is zero (its oracle norm below
    1e-6 of the global one: the attention query bias under the column
    softmax, a convolution bias right before a GroupNorm of one channel per
    group) has no relative scale; it is bounded absolutely.  Every tensor is
    checked before the test fails, and the failure lists all of them."""
    n = len(s.param_names)
    gnorm = np.sqrt(sum(float(np.sum(np.asarray(g, np.float64) ** 2)) for g in ref["clipped"]))
    bad = []
    for i in range(n):
        name = s.param_names[i]
        g = s.read_param(i, 1)   # clipped gradient written back by the update
        r = ref["clipped"][i]
        zero = np.linalg.norm(r) <= 1e-6 * gnorm
        tol = rtol
        for key, t in (rtol_names or {}).items():
            if key in name:
                tol = t
        if zero:
            if np.linalg.norm(g - r) > 1e-5 * gnorm:
                bad.append((name, "zero-gradient tensor", np.linalg.norm(g - r) / gnorm))
        elif exact:
            if rel_err(g, r) > 1e-4:
                bad.append((name, "max-relative", rel_err(g, r)))
        elif norm_err(g, r) > tol:
            bad.append((name, f"normwise > {tol}", norm_err(g, r)))
        m = s.read_param(i, 2)
        if not zero and norm_err(m, ref["m"][i]) > (1e-4 if exact else tol):
            bad.append((name, "first moment", norm_err(m, ref["m"][i])))
        w = s.read_param(i, 0)
        diff = np.abs((w - p0[i]) - (ref["params"][i] - p0[i]))
        if np.max(diff) > 2.05 * lr:
            bad.append((name, "weight update", np.max(diff) / lr))
        # a tensor whose exact gradient vanishes moves by noise amplified to
        # ~lr by Adam's normalisation: only the bound above holds
        if not zero and np.mean(diff > 0.05 * lr) > (0.001 if exact else 0.02):
            bad.append((name, "weights moved differently", np.mean(diff > 0.05 * lr)))
        if s.param_step(i) != 2:
            bad.append((name, "step counter", s.param_step(i)))
    if bad:
        pytest.fail("\n".join(f"{n}: {what} {v:.3g}" for n, what, v in bad))


def _mlp_case(rng, **kw):
    from oracle import graphs
    lr = 1e-3
    s = _session(config=1, batch=64, in_features=784, hidden=256, classes=10, lr=lr, clip_norm=1.0, seed=3, **kw)
    p0 = [(rng.standard_normal(n) * 0.05).astype(np.float32) for n in s.param_sizes]
    for i, p in enumerate(p0):
        s.write_param(i, p)
    x = rng.random((64, 784), dtype=np.float32)
    labels = rng.integers(0, 10, 64).astype(np.int32)
    s.inputs["x"][:] = x.ravel()
    s.inputs["labels"][:] = labels
    loss = s.step()
    ref = graphs.mlp_step(p0, x, labels, lr=lr)
    return s, ref, p0, lr, loss


def test_mlp_step_matches_oracle_fp32(cuda, rng):
    s, ref, p0, lr, loss = _mlp_case(rng, gemm_mode=1)
    assert abs(loss - ref["loss"]) <= 1e-5 * abs(ref["loss"]), (loss, ref["loss"])
    assert abs(s.read_param(0, 1)[0] - ref["clipped"][0][0]) <= 1e-4 * np.max(np.abs(ref["clipped"][0]))
    _check_step(s, ref, p0, lr, exact=True)


def test_mlp_step_tf32_mask_sensitivity(cuda, rng):
    """On TF32 tensor cores the forward differs from fp32 by ~6e-4 relative;
    pre-activations within that distance of zero can take the other ReLU
    branch.  The loss and the last layer (no mask after it) stay within the
    TF32 bound; the first layer's gradient is only close in norm."""
    s, ref, p0, lr, loss = _mlp_case(rng, gemm_mode=0)
    assert abs(loss - ref["loss"]) <= 1e-3 * abs(ref["loss"])
    for i in (2, 3):
        assert norm_err(s.read_param(i, 1), ref["clipped"][i]) <= RTOL_TC
    for i in (0, 1):
        assert norm_err(s.read_param(i, 1), ref["clipped"][i]) <= 0.2


@pytest.mark.parametrize("fused", [1, 0])
def test_encoder_step_matches_oracle(cuda, rng, fused):
    from oracle import graphs
    cfg = dict(batch=2, seq=32, d_model=64, heads=4, ffn=128, layers=2, vocab=256)
    lr = 1e-3
    s = _session(config=2, batch=cfg["batch"], seq_len=cfg["seq"], d_model=cfg["d_model"], heads=cfg["heads"],
                 ffn=cfg["ffn"], layers=cfg["layers"], vocab=cfg["vocab"], lr=lr, clip_norm=1.0,
                 fused_attention=fused, seed=5)
    p0 = [(rng.standard_normal(n) * 0.05).astype(np.float32) for n in s.param_sizes]
    for i, p in enumerate(p0):
        s.write_param(i, p)
    table = (rng.standard_normal(cfg["vocab"] * cfg["d_model"]) * 0.5).astype(np.float32)
    s.write_embedding(0, table)
    tokens = rng.integers(0, cfg["vocab"], (cfg["batch"], cfg["seq"])).astype(np.int32)
    targets = rng.integers(0, cfg["vocab"], (cfg["batch"], cfg["seq"])).astype(np.int32)
    s.inputs["tokens"][:] = tokens.ravel()
    s.inputs["targets"][:] = targets.ravel()
    loss = s.step()
    ref = graphs.encoder_step(p0, table, tokens, targets, cfg["batch"], cfg["seq"], cfg["d_model"], cfg["heads"],
                              cfg["ffn"], cfg["layers"], cfg["vocab"], lr=lr)
    assert abs(loss - ref["loss"]) <= 1e-4 * abs(ref["loss"]), (loss, ref["loss"])
    _check_step(s, ref, p0, lr, exact=False)


@pytest.mark.parametrize("fused", [1, 0])
def test_encdec_step_matches_oracle(cuda, rng, fused):
    """configs[2] structure at a small size: encoder stack, decoder stack
    with masked self-attention and masked cross-attention to the encoder
    output (scale 1/sqrt(d_model)), projection, SMCE, clip, AdamW."""
    from oracle import graphs
    cfg = dict(batch=2, seq=32, d_model=64, heads=4, ffn=128, layers=2, vocab=256)
    lr = 1e-3
    s = _session(config=3, batch=cfg["batch"], seq_len=cfg["seq"], d_model=cfg["d_model"], heads=cfg["heads"],
                 ffn=cfg["ffn"], layers=cfg["layers"], vocab=cfg["vocab"], lr=lr, clip_norm=1.0,
                 fused_attention=fused, seed=7)
    p0 = [(rng.standard_normal(n) * 0.05).astype(np.float32) for n in s.param_sizes]
    for i, p in enumerate(p0):
        s.write_param(i, p)
    tables = [(rng.standard_normal(cfg["vocab"] * cfg["d_model"]) * 0.5).astype(np.float32) for _ in range(2)]
    s.write_embedding(0, tables[0])
    s.write_embedding(1, tables[1])
    shape = (cfg["batch"], cfg["seq"])
    src, tgt_in, tgt_out = (rng.integers(0, cfg["vocab"], shape).astype(np.int32) for _ in range(3))
    s.inputs["src"][:] = src.ravel()
    s.inputs["tgt_in"][:] = tgt_in.ravel()
    s.inputs["tgt_out"][:] = tgt_out.ravel()
    loss = s.step()
    ref = graphs.encdec_step(p0, tables, src, tgt_in, tgt_out, cfg["batch"], cfg["seq"], cfg["d_model"],
                             cfg["heads"], cfg["ffn"], cfg["layers"], cfg["vocab"], lr=lr)
    assert abs(loss - ref["loss"]) <= 1e-4 * abs(ref["loss"]), (loss, ref["loss"])
    _check_step(s, ref, p0, lr, exact=False)


@pytest.mark.parametrize("gemm_mode", [1, 0], ids=["fp32", "tf32"])
def test_unet_step_matches_oracle(cuda, rng, gemm_mode):
    """configs[3] structure at a small size: ResidualBlocks (Conv2D,
    GroupNorm(8), SiLU, time-MLP Broadcast_Channel, 1x1 skip), stride-2
    downsampling, Conv2DT upsampling with CopyCrop skips, MSE, clip, AdamW.
    fp32 GEMM mode: 1e-4 max-relative per tensor.  TF32: normwise per
    tensor 3e-3 (worst measured 2.5e-3, the weights of Enc3's stride-2 and
    skip convolutions, whose gradient has come back through nine TF32
    convolution + GroupNorm layers; the transformers hold 2e-3 at their
    benchmarked shapes), and 5e-3 for two kinds of tensor whose gradient is
    a sum whose terms largely cancel, so the convolutions' TF32 error
    reaches them enlarged by that cancellation: the time-MLP Linears (3.3e-3
    measured; their upstream is Broadcast_Channel's backward, a sum over the
    batch and every pixel of the convolution path's gradient; their own
    products are fp32 skinny GEMMs) and the convolution biases (up to
    3.1e-3 measured; a bias gradient is the per-channel sum over the batch
    and every pixel of the upstream gradient, and behind a GroupNorm, whose
    backward removes the gradient's mean over each group, those sums nearly
    cancel -- exactly, with one channel per group)."""
    from oracle import graphs
    cfg = dict(batch=2, channels=3, image_size=16, base_width=8, t_embed=32, timestep=500)
    lr = 1e-3
    s = _session(config=4, lr=lr, clip_norm=1.0, seed=9, gemm_mode=gemm_mode, **cfg)
    p0 = [(rng.standard_normal(n) * 0.1).astype(np.float32) for n in s.param_sizes]
    for i, p in enumerate(p0):
        s.write_param(i, p)
    n_img = cfg["batch"] * cfg["channels"] * cfg["image_size"] ** 2
    x_t = rng.standard_normal(n_img).astype(np.float32)
    noise = rng.standard_normal(n_img).astype(np.float32)
    s.inputs["x_t"][:] = x_t
    s.inputs["noise"][:] = noise
    loss = s.step()
    ref = graphs.unet_step(p0, x_t, noise, lr=lr, **cfg)
    assert abs(loss - ref["loss"]) <= 1e-4 * abs(ref["loss"]), (loss, ref["loss"])
    _check_step(s, ref, p0, lr, exact=gemm_mode == 1, rtol=3e-3, rtol_names={"Time MLP": 5e-3, "Bias": 5e-3})


def test_graph_replay_equals_eager(cuda, rng):
    """A captured CUDA graph of the step gives the same parameters as eager
    steps on the same inputs (device step counters advance in both).  The
    split-K and column-sum atomics make the last bits order-dependent."""
    kw = dict(config=2, batch=2, seq_len=32, d_model=64, heads=4, ffn=128, layers=1, vocab=128, seed=9)
    a, b = _session(**kw), _session(**kw)
    tokens = rng.integers(0, 128, 64).astype(np.int32)
    targets = rng.integers(0, 128, 64).astype(np.int32)
    for s in (a, b):
        s.inputs["tokens"][:] = tokens
        s.inputs["targets"][:] = targets
    for _ in range(3):
        a.step()
    b.step()
    b.capture()
    b.step()
    b.step()
    for i in range(len(a.param_names)):
        assert norm_err(b.read_param(i), a.read_param(i)) <= 1e-5, a.param_names[i]
        assert a.param_step(i) == b.param_step(i) == 4


def test_loss_decreases_on_fixed_batch(cuda, rng):
    s = _session(config=1, batch=64, in_features=784, hidden=256, classes=10, lr=1e-3, seed=11, gemm_mode=1)
    s.inputs["x"][:] = rng.random(64 * 784, dtype=np.float32)
    s.inputs["labels"][:] = rng.integers(0, 10, 64)
    first = s.step()
    for _ in range(30):
        last = s.step()
    assert last < 0.5 * first


def _read_reference_checkpoint(path):
    """Records of the reference's AdamParameter::save (Engine/engine.cu:
    139-188): u32 name length, name, i32 count, f32 weights, m, v."""
    import struct
    recs = []
    with open(path, "rb") as f:
        data = f.read()
    off = 0
    while off < len(data):
        (n,) = struct.unpack_from("<I", data, off)
        off += 4
        name = data[off:off + n].decode()
        off += n
        (total,) = struct.unpack_from("<i", data, off)
        off += 4
        arrs = []
        for _ in range(3):
            arrs.append(np.frombuffer(data, np.float32, total, off).copy())
            off += 4 * total
        recs.append((name, arrs))
    return recs


def test_checkpoint_roundtrip_and_resume(cuda, rng, tmp_path):
    """save() writes the reference's record format (checked field by field
    against the session's parameters) and a step sidecar; a session with
    other weights and moments that loads it holds the same state and
    continues like the original."""
    kw = dict(config=2, batch=2, seq_len=32, d_model=64, heads=4, ffn=128, layers=1, vocab=128, gemm_mode=1)
    a = _session(seed=9, **kw)
    tokens = rng.integers(0, 128, 64).astype(np.int32)
    targets = rng.integers(0, 128, 64).astype(np.int32)
    a.inputs["tokens"][:] = tokens
    a.inputs["targets"][:] = targets
    for _ in range(3):
        a.step()
    path = tmp_path / "ckpt.bin"
    a.save(path)
    recs = _read_reference_checkpoint(path)
    assert [r[0] for r in recs] == list(a.param_names)
    for i, (_, (w, m, v)) in enumerate(recs):
        assert np.array_equal(w, a.read_param(i, 0))
        assert np.array_equal(m, a.read_param(i, 2))
        assert np.array_equal(v, a.read_param(i, 3))
    steps = np.fromfile(str(path) + ".t", np.int32)
    assert steps[0] == len(recs) and np.all(steps[1:] == 4)

    # same seed for the (untrained, gather-only) embedding table; every
    # parameter and moment overwritten before the load
    b = _session(seed=9, **kw)
    b.inputs["tokens"][:] = tokens
    b.inputs["targets"][:] = targets
    for i in range(len(recs)):
        for which in (0, 2, 3):
            b.write_param(i, rng.standard_normal(b.param_sizes[i]).astype(np.float32), which)
    assert not np.array_equal(b.read_param(0), a.read_param(0))
    b.load(path)
    for i in range(len(recs)):
        assert np.array_equal(b.read_param(i, 0), a.read_param(i, 0))
        assert b.param_step(i) == 4
    # the next step: equal up to the order of the bias-gradient atomics
    la, lb = a.step(), b.step()
    assert abs(la - lb) <= 1e-6 * abs(la)
    for i in range(len(recs)):
        assert norm_err(b.read_param(i, 0), a.read_param(i, 0)) <= 1e-6, a.param_names[i]
        assert b.param_step(i) == 5


def test_checkpoint_mismatch_changes_nothing(cuda, rng, tmp_path):
    from ml_engine_b200._lib import MLEError
    a = _session(config=2, batch=2, seq_len=16, d_model=32, heads=2, ffn=64, layers=1, vocab=64, seed=1)
    path = tmp_path / "small.bin"
    a.save(path)
    b = _session(config=2, batch=2, seq_len=16, d_model=64, heads=2, ffn=64, layers=1, vocab=64, seed=2)
    before = [b.read_param(i) for i in range(len(b.param_names))]
    with pytest.raises(MLEError):
        b.load(path)
    for i, w in enumerate(before):
        assert np.array_equal(b.read_param(i), w)


def test_index_labels_match_dense_targets(cuda, rng):
    """The session's index-label loss (default) against the reference's dense
    one-hot target graph (dense_targets=1): same loss and parameters."""
    kw = dict(config=2, batch=2, seq_len=32, d_model=64, heads=4, ffn=128, layers=1, vocab=128, seed=9, gemm_mode=1)
    a, b = _session(dense_targets=1, **kw), _session(dense_targets=0, **kw)
    tokens = rng.integers(0, 128, 64).astype(np.int32)
    targets = rng.integers(0, 128, 64).astype(np.int32)
    for s in (a, b):
        s.inputs["tokens"][:] = tokens
        s.inputs["targets"][:] = targets
    for _ in range(2):
        la, lb = a.step(), b.step()
        assert abs(la - lb) <= 1e-6 * abs(la)
    for i in range(len(a.param_names)):
        assert norm_err(b.read_param(i), a.read_param(i)) <= 1e-6, a.param_names[i]


@pytest.mark.parametrize("gemm_mode", [0, 1], ids=["tf32", "fp32"])
def test_first_write_assign_unet(cuda, rng, gemm_mode):
    """First-writer assignment in the U-Net (convolutions write the
    gradients of the activations they read; Adds, activations and the loss
    as in the encoder) against every gradient cleared and accumulated: the
    same losses and gradients over an eager step and two graph replays at
    learning rate 0.  Each run is bitwise repeatable, but in TF32 mode an
    assigned convolution product may tile differently from an accumulated
    one, and the summation-order differences pass through thirteen
    GroupNorm layers, so TF32 gets the TF32 tolerance.  An uncleared
    gradient would be off by a whole step's gradient.  Tensors whose exact
    gradient is zero (a bias before a GroupNorm of one channel per group)
    are bounded absolutely."""
    from ml_engine_b200._lib import engine
    cfg = dict(config=4, batch=2, channels=3, image_size=16, base_width=8, t_embed=32, timestep=500, seed=9, lr=0.0,
               gemm_mode=gemm_mode)
    lib = engine()
    old = lib.mle_get_grad_first_write()
    n_img = 2 * 3 * 16 * 16
    x_t = rng.standard_normal(n_img).astype(np.float32)
    noise = rng.standard_normal(n_img).astype(np.float32)
    runs = {}
    try:
        for mode in (0, 1):
            lib.call("mle_set_grad_first_write", mode)
            s = _session(**cfg)
            s.inputs["x_t"][:] = x_t
            s.inputs["noise"][:] = noise
            losses = [s.step()]
            s.capture()
            losses += [s.step(), s.step()]
            runs[mode] = (s, losses, [s.read_param(i, 1) for i in range(len(s.param_names))])
    finally:
        lib.call("mle_set_grad_first_write", old)
    (a, la, ga), (b, lb, gb) = runs[0], runs[1]
    for x, y in zip(la + lb, la[:1] * 6):
        assert abs(x - y) <= 1e-5 * abs(y), (la, lb)
    gnorm = np.sqrt(sum(float(np.sum(np.asarray(g, np.float64) ** 2)) for g in ga))
    for i in range(len(a.param_names)):
        floor = np.linalg.norm(gb[i] - ga[i]) <= 1e-6 * gnorm
        tol = RTOL_TC if gemm_mode == 0 else 1e-4
        assert norm_err(gb[i], ga[i]) <= tol or floor, (a.param_names[i], norm_err(gb[i], ga[i]))


def test_first_write_assign_matches_cleared_gradients(cuda, rng):
    """First-writer assignment (gradients the first backward writer
    overwrites are not cleared; the loss, activations and large-input
    Linears assign) against every gradient cleared and accumulated, over an
    eager step and two graph replays: the same losses and gradients.  A
    gradient left uncleared but still accumulated would be off by a whole
    step's gradient.  The learning rate is 0, so every step sees the same
    weights: the gradients of both runs then differ only where split-K
    reduce-adds and column-sum atomics reorder sums (with a moving model,
    Adam amplifies that noise in near-degenerate tensors such as the query
    weights).  The FFN width makes the second Linear's input gradient large
    enough to be assigned."""
    from ml_engine_b200._lib import engine
    kw = dict(config=2, batch=16, seq_len=256, d_model=512, heads=8, ffn=2048, layers=1, vocab=512, seed=5, lr=0.0)
    lib = engine()
    old = lib.mle_get_grad_first_write()
    tokens = rng.integers(0, 512, 16 * 256).astype(np.int32)
    targets = rng.integers(0, 512, 16 * 256).astype(np.int32)
    runs = {}
    try:
        for mode in (0, 1):
            lib.call("mle_set_grad_first_write", mode)
            s = _session(**kw)
            s.inputs["tokens"][:] = tokens
            s.inputs["targets"][:] = targets
            losses = [s.step()]
            s.capture()
            losses += [s.step(), s.step()]
            runs[mode] = (s, losses, [s.read_param(i, 1) for i in range(len(s.param_names))])
    finally:
        lib.call("mle_set_grad_first_write", old)
    (a, la, ga), (b, lb, gb) = runs[0], runs[1]
    for x, y in zip(la + lb, la[:1] * 6):  # the same weights every step: the same loss
        assert abs(x - y) <= 1e-5 * abs(y), (la, lb)
    gnorm = np.sqrt(sum(float(np.sum(np.asarray(g, np.float64) ** 2)) for g in ga))
    for i in range(len(a.param_names)):
        # the query bias's exact gradient is zero (column softmax): no relative scale
        floor = np.linalg.norm(gb[i] - ga[i]) <= 1e-7 * gnorm
        assert norm_err(gb[i], ga[i]) <= 1e-4 or floor, (a.param_names[i], norm_err(gb[i], ga[i]))


def test_fused_optimizer_matches_separate_launches(cuda, rng):
    """The single cooperative norm + clip + AdamW launch that ParameterUpdate
    takes by default, against the sum-of-squares, finalize and update
    launches, over an eager step and two graph replays: the same losses,
    clipped gradients, moments and step counters, and fewer kernel nodes in
    the captured step.  The learning rate is 0 so both runs see the same
    weights; their gradients then differ only by the backward's reordered
    sums, and the clip coefficient by the norm's summation order."""
    import ctypes
    from ml_engine_b200._lib import engine
    kw = dict(config=2, batch=16, seq_len=256, d_model=512, heads=8, ffn=2048, layers=1, vocab=512, seed=5, lr=0.0)
    lib = engine()
    old = lib.mle_get_fused_optimizer()
    tokens = rng.integers(0, 512, 16 * 256).astype(np.int32)
    targets = rng.integers(0, 512, 16 * 256).astype(np.int32)
    runs = {}
    try:
        for mode in (0, 1):
            lib.call("mle_set_fused_optimizer", mode)
            s = _session(**kw)
            s.inputs["tokens"][:] = tokens
            s.inputs["targets"][:] = targets
            losses = [s.step()]
            s.capture()
            losses += [s.step(), s.step()]
            kk, mm, cc = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
            s._lib.call("mle_session_graph_counts", s._h, ctypes.addressof(kk), ctypes.addressof(mm),
                        ctypes.addressof(cc))
            state = [[s.read_param(i, w) for w in (1, 2, 3)] for i in range(len(s.param_names))]
            steps = [s.param_step(i) for i in range(len(s.param_names))]
            runs[mode] = (s, losses, state, steps, kk.value)
    finally:
        lib.call("mle_set_fused_optimizer", old)
    (a, la, sa, ta, ka), (b, lb, sb, tb, kb) = runs[0], runs[1]
    assert ta == tb
    assert kb < ka, (ka, kb)
    for x, y in zip(la + lb, la[:1] * 6):
        assert abs(x - y) <= 1e-5 * abs(y), (la, lb)
    for which in range(3):
        gnorm = np.sqrt(sum(float(np.sum(np.asarray(st[which], np.float64) ** 2)) for st in sa))
        for i in range(len(a.param_names)):
            x, y = sb[i][which], sa[i][which]
            floor = np.linalg.norm(x - y) <= 1e-7 * gnorm
            assert norm_err(x, y) <= 1e-4 or floor, (a.param_names[i], which, norm_err(x, y))


def test_add_norm_fusion_matches_separate_launches(cuda, rng):
    """The forward's residual Add + LayerNorm passes against the Add and the
    norm launched apart, on the pre-LN encoder: the same loss and gradients
    up to the step's own run-to-run spread (its loss and gradient sums use
    atomics, so even repeated steps of one run differ in the last bits; the
    pass itself is checked bit for bit against the two launches in the
    kernel tests), and fewer kernels in the captured step."""
    import ctypes
    from ml_engine_b200._lib import engine
    kw = dict(config=2, batch=16, seq_len=256, d_model=512, heads=8, ffn=2048, layers=1, vocab=512, seed=5, lr=0.0)
    lib = engine()
    old = lib.mle_get_add_norm_fusion()
    tokens = rng.integers(0, 512, 16 * 256).astype(np.int32)
    targets = rng.integers(0, 512, 16 * 256).astype(np.int32)
    runs = {}
    try:
        for mode in (0, 1):
            lib.call("mle_set_add_norm_fusion", mode)
            s = _session(**kw)
            s.inputs["tokens"][:] = tokens
            s.inputs["targets"][:] = targets
            losses = [s.step()]
            s.capture()
            losses += [s.step(), s.step()]
            kk, mm, cc = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
            s._lib.call("mle_session_graph_counts", s._h, ctypes.addressof(kk), ctypes.addressof(mm),
                        ctypes.addressof(cc))
            runs[mode] = (s, losses, [s.read_param(i, 1) for i in range(len(s.param_names))], kk.value)
    finally:
        lib.call("mle_set_add_norm_fusion", old)
    (a, la, ga, ka), (b, lb, gb, kb) = runs[0], runs[1]
    assert kb < ka, (ka, kb)
    for x, y in zip(la + lb, la[:1] * 6):
        assert abs(x - y) <= 1e-5 * abs(y), (la, lb)
    gnorm = np.sqrt(sum(float(np.sum(np.asarray(g, np.float64) ** 2)) for g in ga))
    for i in range(len(a.param_names)):
        floor = np.linalg.norm(gb[i] - ga[i]) <= 1e-7 * gnorm
        assert norm_err(gb[i], ga[i]) <= 1e-4 or floor, (a.param_names[i], norm_err(gb[i], ga[i]))
