"""Host side of data parallelism, on the CPU: the gradient-bucket plan
(mle_dp_plan_buckets, the planner mle_session_enable_dp uses) and bench.py's
multi-rank logic over a world-size-2 gloo process group."""
import ctypes
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def _plan(addrs, counts, bucket_mb, max_out=64, chunks=None):
    from ml_engine_b200._lib import engine
    lib = engine()
    n = len(addrs)
    a = (ctypes.c_uint64 * max(n, 1))(*addrs)
    c = (ctypes.c_int64 * max(n, 1))(*counts)
    ch = None if chunks is None else (ctypes.c_uint64 * max(n, 1))(*chunks)
    ob, oc, on = (ctypes.c_uint64 * max_out)(), (ctypes.c_int64 * max_out)(), ctypes.c_int()
    lib.call("mle_dp_plan_buckets", a, c, ch, n, bucket_mb, ob, oc, max_out, ctypes.byref(on))
    return [(ob[i], oc[i]) for i in range(on.value)]


def test_plan_never_spans_two_allocations():
    """Two arena chunks that happen to be adjacent in the address space are
    still two cudaMalloc ranges: one NCCL buffer may not cover both."""
    base = 1 << 32
    chunk = 1 << 20                      # bytes per (toy) chunk
    addrs = [base, base + chunk - 4096, base + chunk, base + chunk + 4096]
    counts = [1024, 1024, 1024, 1024]    # 4 KiB each: they touch across the boundary
    ids = [base, base, base + chunk, base + chunk]
    b = _plan(addrs, counts, bucket_mb=32, chunks=ids)
    assert len(b) == 3                   # [0] alone (gap), [1] alone (chunk end), [2]+[3] merged
    for start, cnt in b:
        end = start + 4 * cnt
        assert (start < base + chunk) == (end <= base + chunk)
    merged = _plan(addrs, counts, bucket_mb=32)          # no chunk ids: one allocation
    assert len(merged) == 2


def test_auto_bucket_size():
    from ml_engine_b200._lib import engine
    lib = engine()
    mib = (1 << 20) // 4
    assert lib.mle_dp_auto_bucket_mb(0) == 1
    assert lib.mle_dp_auto_bucket_mb(2_630_000) == 4        # configs[1]: 10.5 MB -> 3 buckets
    assert lib.mle_dp_auto_bucket_mb(48_200_000) == 32      # configs[2]: 193 MB -> 6 buckets
    for total in (1, mib, 7 * mib, 100 * mib, 10_000 * mib):
        mb = lib.mle_dp_auto_bucket_mb(total)
        assert mb in (1, 2, 4, 8, 16, 32)
        assert mb == 32 or total <= 4 * mb * mib             # at most four buckets below the cap
        assert mb == 1 or total > 4 * (mb // 2) * mib        # the smallest such power of two
    addrs, cur = [], 1 << 32
    for _ in range(40):
        addrs.append(cur)
        cur += 256 * 1024 * 4
    b = _plan(addrs, [256 * 1024] * 40, bucket_mb=0)        # 40 MiB -> 16 MiB buckets
    assert len(b) == 3


def test_plan_merges_contiguous_runs_within_cap():
    base = 1 << 32
    # tensors laid out as the arena does: 256-byte aligned, some pads between
    sizes = [1000, 64, 300000, 7, 100000, 1 << 20]
    addrs, cur = [], base
    for n in sizes:
        addrs.append(cur)
        cur += ((n * 4 + 255) // 256) * 256
    order = np.random.default_rng(0).permutation(len(sizes))   # planner sorts by address
    b = _plan([addrs[i] for i in order], [sizes[i] for i in order], bucket_mb=2)
    cap = 2 * (1 << 20) // 4
    covered = []
    for start, cnt in b:
        assert cnt <= cap or any(start == a and cnt == n for a, n in zip(addrs, sizes))
        covered.append((start, start + 4 * cnt))
    for a, n in zip(addrs, sizes):       # every tensor inside exactly one bucket
        assert sum(1 for s, e in covered if s <= a and a + 4 * n <= e) == 1
    assert all(covered[i][1] <= covered[i + 1][0] for i in range(len(covered) - 1))
    assert len(b) < len(sizes)           # contiguous small tensors were merged


def test_plan_splits_on_gaps_and_rejects_small_output():
    b = _plan([0x1000, 0x100000], [16, 16], bucket_mb=32)
    assert b == [(0x1000, 16), (0x100000, 16)]
    from ml_engine_b200._lib import MLEError
    with pytest.raises(MLEError):
        _plan([0x1000, 0x100000], [16, 16], bucket_mb=32, max_out=1)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _max_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    import bench
    import torch.distributed as dist
    w, r, _ = bench.init_ranks()
    got = bench.max_over_ranks(1.5 + r, w, "cpu")
    bench.barrier(w)
    q.put((r, dist.get_backend(), got))
    dist.destroy_process_group()


def test_bench_max_over_ranks_gloo():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_max_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[0] for r in res] == [0, 1]
    assert all(r[1] == "gloo" and r[2] == 2.5 for r in res)


def test_bench_reference_arm_prints_once_under_torchrun():
    if not (ROOT / "oracle" / "lib" / "libmle_oracle.so").exists():
        pytest.skip("oracle not built")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(ROOT / "bench.py"),
           "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0", "--config", "mlp"]
    # torchrun's own setting: one OpenMP thread per rank; the CPU arm must
    # still run the oracle on every host core
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [json.loads(x) for x in out.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    assert lines[0]["impl"] == "reference" and lines[0]["n_gpus"] == 2 and lines[0]["value"] > 0
    assert lines[0]["cpu_baseline"]["cores"] == (os.cpu_count() or 1)
