"""Data parallelism on two GPUs: two ranks, each with half of the global
batch and NCCL bucket reductions overlapped with the backward, take the same
steps as one GPU with the whole batch (eager step, then two replays of the
captured graph that contains the NCCL calls)."""
import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest

from conftest import norm_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
ROOT = Path(__file__).resolve().parents[1]
CFG = dict(config=2, seq_len=32, d_model=64, heads=4, ffn=128, layers=2, vocab=256, lr=1e-3, clip_norm=1.0,
           fused_attention=1, seed=5)
B = 8
STEPS = 3


def _problem():
    rng = np.random.default_rng(11)
    from ml_engine_b200.session import Session
    s = Session(batch=B, **CFG)
    sizes = list(s.param_sizes)
    s.close()
    params = [(rng.standard_normal(n) * 0.05).astype(np.float32) for n in sizes]
    table = (rng.standard_normal(CFG["vocab"] * CFG["d_model"]) * 0.5).astype(np.float32)
    toks = [rng.integers(0, CFG["vocab"], (B, CFG["seq_len"])).astype(np.int32) for _ in range(STEPS)]
    tgts = [rng.integers(0, CFG["vocab"], (B, CFG["seq_len"])).astype(np.int32) for _ in range(STEPS)]
    return params, table, toks, tgts


def _run(session, params, table, toks, tgts, rows, embed=False):
    for i, p in enumerate(params):
        session.write_param(i, p)
    session.write_embedding(0, table)
    losses = []
    for k in range(STEPS):
        session.inputs["tokens"][:] = toks[k][rows].ravel()
        session.inputs["targets"][:] = tgts[k][rows].ravel()
        losses.append(session.step())
        if k == 0:
            session.capture()
    n = len(params)
    w = [session.read_param(i, 0) for i in range(n)]
    if embed:   # the trained embedding table joins the compared tensors
        w.append(session.read_embedding(0))
    return losses, w, [session.read_param(i, 1) for i in range(n)]


def _worker(rank, world, port, q, embed_lr=0.0):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))   # carries the NCCL id only
    from ml_engine_b200.session import Session
    params, table, toks, tgts = _problem()
    s = Session(batch=B // world, embed_lr=embed_lr, **CFG)
    uid = [Session.dp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    s.enable_dp(uid[0], rank, world)
    losses, w, g = _run(s, params, table, toks, tgts, slice(rank * B // world, (rank + 1) * B // world),
                        embed=embed_lr > 0)
    q.put((rank, losses, w, g))
    dist.barrier()
    s.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("embed_lr", [0.0, 1e-3], ids=["frozen_table", "trained_table"])
def test_two_rank_dp_equals_one_gpu_global_batch(cuda, embed_lr):
    """With a trained table the ranks' embedding deltas are summed with the
    gradient buckets and averaged, so the table moves as one GPU's with the
    whole batch would (compared with the parameters below)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import socket as _s
    import torch.multiprocessing as mp
    with _s.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, embed_lr)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = {}
        for _ in procs:
            r, losses, w, g = q.get(timeout=300)
            res[r] = (losses, w, g)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.exitcode is None:
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    from ml_engine_b200.session import Session
    params, table, toks, tgts = _problem()
    s = Session(batch=B, embed_lr=embed_lr, **CFG)
    losses, w_one, g_one = _run(s, params, table, toks, tgts, slice(0, B), embed=embed_lr > 0)
    s.close()
    # both ranks hold identical parameters and clipped gradients after every step
    for a, b in zip(res[0][1] + res[0][2], res[1][1] + res[1][2]):
        assert np.array_equal(a, b)
    # the mean of the ranks' local losses is the global-batch loss
    for k in range(STEPS):
        dp_loss = 0.5 * (res[0][0][k] + res[1][0][k])
        assert abs(dp_loss - losses[k]) <= 1e-4 * abs(losses[k]), (k, dp_loss, losses[k])
    # last step's clipped gradients: TF32 tolerance per tensor; a tensor whose
    # exact gradient vanishes (the query bias under the column softmax) is
    # bounded against the global gradient norm instead
    gnorm = np.sqrt(sum(float(np.sum(np.asarray(g, np.float64) ** 2)) for g in g_one))
    for i, (a, b) in enumerate(zip(res[0][2], g_one)):
        assert norm_err(a, b) <= 2e-3 or np.linalg.norm(a - b) <= 1e-4 * gnorm, (i, norm_err(a, b))
    # parameters: each AdamW step moves an element by at most ~lr
    for i, (a, b) in enumerate(zip(res[0][1], w_one)):
        assert np.max(np.abs(a - b)) <= 2.05 * CFG["lr"] * STEPS, i
    if embed_lr > 0:   # the table's total update over the steps, TF32 tolerance
        moved_dp, moved_one = res[0][1][-1] - table, w_one[-1] - table
        assert np.linalg.norm(moved_one) > 0
        assert norm_err(moved_dp, moved_one) <= 2e-3, norm_err(moved_dp, moved_one)


_MISSING_RANK = r"""
import sys, time
sys.path.insert(0, sys.argv[1])
from ml_engine_b200.session import Session
from ml_engine_b200._lib import MLEError
s = Session(config=1, batch=8, in_features=16, hidden=8, classes=4, seed=1)
uid = Session.dp_unique_id()
t0 = time.time()
try:
    s.enable_dp(uid, 0, 2)          # rank 1 of 2 never joins
    print("JOINED")
except MLEError as e:
    print("ERROR", time.time() - t0, e)
s.step()                            # the session still trains on its own
print("STEP OK")
"""


def test_dp_missing_rank_times_out_on_host(cuda):
    """A communicator whose other rank never joins: the set-up gives up on
    the host after MLE_DP_TIMEOUT_S (non-blocking NCCL initialisation,
    ncclCommAbort) and returns MLE_ERR_TIMEOUT instead of waiting for good;
    nothing was launched on the GPU for the communicator, and the session
    stays usable.  One process on one GPU; NVLS off."""
    import subprocess
    env = dict(os.environ, MLE_DP_TIMEOUT_S="3", NCCL_NVLS_ENABLE="0", CUDA_VISIBLE_DEVICES="0")
    out = subprocess.run([sys.executable, "-c", _MISSING_RANK, str(ROOT)], capture_output=True, text=True,
                         timeout=120, env=env)
    assert out.returncode == 0, out.stderr[-3000:]
    lines = out.stdout.splitlines()
    err = [x for x in lines if x.startswith("ERROR")]
    assert err and "JOINED" not in lines, out.stdout + out.stderr[-2000:]
    waited = float(err[0].split()[1])
    assert 2.5 <= waited <= 60.0, waited
    assert "timed out" in err[0] or "TIMEOUT" in err[0].upper() or "wait" in err[0], err[0]
    assert "STEP OK" in lines
