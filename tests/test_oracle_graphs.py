"""CPU checks of the whole-step oracle (oracle/graphs.py): the MLP step's
gradients against central finite differences of its own loss, and the
encoder step's shapes, finiteness and loss scale."""
import numpy as np

from conftest import rel_err


def _mlp_params(rng):
    return [(rng.standard_normal(n) * 0.05).astype(np.float32) for n in (784 * 256, 256, 256 * 10, 10)]


def test_mlp_gradients_match_finite_differences(rng):
    from oracle import graphs
    p = _mlp_params(rng)
    x = rng.random((8, 784), dtype=np.float32)
    labels = rng.integers(0, 10, 8).astype(np.int32)
    out = graphs.mlp_step(p, x, labels, clip_norm=0.0)
    # The reference divides the CE gradient by the batch (dim 0) while the
    # loss is averaged over batch*classes, so d(loss)/dw = grad / classes.
    for pi, idx in [(2, 5), (2, 300), (3, 7), (0, 1234), (1, 17)]:
        eps = 1e-2
        pp = [q.astype(np.float64).copy() for q in p]
        pp[pi][idx] += eps
        lp = graphs.mlp_step([q.astype(np.float32) for q in pp], x, labels, clip_norm=0.0)["loss"]
        pp[pi][idx] -= 2 * eps
        lm = graphs.mlp_step([q.astype(np.float32) for q in pp], x, labels, clip_norm=0.0)["loss"]
        fd = (lp - lm) / (2 * eps)
        an = out["grads"][pi][idx] / 10.0
        assert abs(fd - an) <= 2e-3 * max(abs(an), 1e-4) + 2e-6, (pi, idx, fd, an)


def test_encoder_step_runs(rng):
    from oracle import graphs
    cfg = dict(batch=2, seq=8, d_model=16, heads=2, ffn=32, layers=2, vocab=32)
    sizes = []
    for _ in range(cfg["layers"]):
        sizes += [16 * 16, 16] * 4 + [16 * 32, 32, 32 * 16, 16]
    sizes += [16 * 32, 32]
    p = [(rng.standard_normal(n) * 0.05).astype(np.float32) for n in sizes]
    table = rng.standard_normal(32 * 16).astype(np.float32)
    tok = rng.integers(0, 32, (2, 8)).astype(np.int32)
    tgt = rng.integers(0, 32, (2, 8)).astype(np.int32)
    out = graphs.encoder_step(p, table, tok, tgt, **cfg)
    assert abs(out["loss"] - np.log(32) / 32) < 0.5 * np.log(32) / 32
    assert all(np.all(np.isfinite(g)) for g in out["grads"])
    assert all(g.size == q.size for g, q in zip(out["grads"], p))
    assert out["clip"] >= 1.0
