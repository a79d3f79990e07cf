#!/usr/bin/env python
"""Training-step benchmark of the ML_Engine hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

Workload: BASELINE configs[1] -- 2-layer pre-LN transformer encoder, batch 32
x seq 128, d_model 256, 8 heads, FFN 1024 (GELU), vocab 4096, next-token
softmax cross-entropy, AdamW with clipNorm 1.0 -- one step = zero_grad,
forward, backward, clip, AdamW over one local batch (4096 tokens).  Under
torchrun each rank runs one replica-parallel (data-parallel) session with its
own batch; gradients are summed with NCCL (weak scaling).

Legs (all on the session's stream, CUDA events, max over ranks):
  value  steps/s with the inputs resident in HBM (captured step replayed);
  e2e    the same through the public API with host buffers: every step fills
         the pinned host inputs with new token ids, uploads them, runs the
         step and reads the loss back to the host;
  roofline  the dominant kernel (the projection layer's backward GEMMs)
         timed alone against the measured tensor peak;
  cpu_baseline  the CPU oracle's step on a bounded sample (rank 0, N=1).
--impl reference times the reference's path on the host cores (the oracle
port: the reference has no CPU implementation and its own CUDA graph cannot
run its SoftMaxCrossEntropy node safely).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CFG = dict(batch=32, seq_len=128, d_model=256, heads=8, ffn=1024, layers=2, vocab=4096)
TOKENS_PER_STEP = CFG["batch"] * CFG["seq_len"]
METRIC = "train steps/s (fwd+bwd+AdamW) at 1/2/4/8 B200; bwd % of roofline"
WORKLOAD = "configs[1]: 2-layer pre-LN transformer encoder, batch 32 x seq 128, d256 h8 ffn1024 gelu, vocab 4096"


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while timing."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, dev_index):
        self.dev = str(dev_index)
        self.samples = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.dev, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            deadline = time.time() + 5.0   # wait for the first sample before timing
            while not self.samples and time.time() < deadline:
                time.sleep(0.05)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 8:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit())
        mx = max(float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[4 + i].strip() == "Active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(self.samples)}


# ------------------------------------------------------------ ranks
def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world, device):
    """Largest value of x over the ranks (every rank gets it)."""
    if world > 1:
        import torch
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return x


def init_ranks():
    """(world, rank, local_rank) from the torchrun environment; joins the
    process group (NCCL on GPUs, gloo without) with a short timeout."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch
        import torch.distributed as dist
        if torch.cuda.is_available():
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                    device_id=torch.device("cuda", local_rank))
        else:
            dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    return world, rank, local_rank


# ------------------------------------------------------------ CPU baseline
def cpu_sample(seconds=10.0, max_steps=None):
    """The oracle's encoder step (OpenMP C restatement) on one sequence of
    the 32-sequence batch; returns (full-config steps/s, cores, sample)."""
    import numpy as np

    from oracle import graphs
    rng = np.random.default_rng(0)
    D, F, V, L = CFG["d_model"], CFG["ffn"], CFG["vocab"], CFG["layers"]
    sizes = []
    for _ in range(L):
        sizes += [D * D, D] * 4 + [D * F, F, F * D, D]
    sizes += [D * V, V]
    params = [(rng.standard_normal(n) * 0.02).astype(np.float32) for n in sizes]
    table = (rng.standard_normal(V * D) * 0.02).astype(np.float32)
    sb = 1
    steps, t0 = 0, time.perf_counter()
    while True:
        tok = rng.integers(0, V, (sb, CFG["seq_len"])).astype(np.int32)
        tgt = rng.integers(0, V, (sb, CFG["seq_len"])).astype(np.int32)
        graphs.encoder_step(params, table, tok, tgt, sb, CFG["seq_len"], D, CFG["heads"], F, L, V)
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds or (max_steps and steps >= max_steps):
            break
    per_sample_step = el / steps
    full_step = per_sample_step * CFG["batch"] / sb
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    return 1.0 / full_step, cores, f"{steps} oracle steps of 1 of 32 sequences (128 tokens), scaled x32; {el:.1f}s"


def run_reference(args, rank, world):
    if rank != 0:
        return
    per_step = []
    cores = None
    sample = ""
    for i in range(args.warmup + args.steps):
        v, cores, sample = cpu_sample(seconds=0.0, max_steps=1)
        if i >= args.warmup:
            per_step.append(1.0 / v)
    total = sum(per_step)
    value = len(per_step) / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "steps/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / len(per_step),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": CFG["batch"] * world, "seq_len": CFG["seq_len"],
                   "parallelism": f"dp{world}"},
        "cpu_baseline": {"value": value, "unit": "steps/s", "cores": cores, "kind": "port",
                         "sample": "per step: " + sample},
        "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference is CUDA-only; its CPU arm is the oracle's C restatement of the same graph "
                "(oracle/mle_oracle.c + oracle/graphs.py) on the host cores",
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ roofline kernel
def roofline_pair(dev, stream, reps=50):
    """The projection layer's backward GEMMs (dX = dY W^T, dW = X^T dY),
    2 * 2 * 4096 * 256 * 4096 FLOP per pair, on `stream`: 3 untimed pairs,
    then `reps` pairs, each between its own CUDA events after a 256 MB write
    that evicts the operands from L2.  Returns (ms per pair, FLOP)."""
    import torch

    from ml_engine_b200 import ops
    M, K, N = TOKENS_PER_STEP, CFG["d_model"], CFG["vocab"]
    g = torch.Generator(device=dev).manual_seed(0)
    X = torch.randn(M, K, device=dev, generator=g)
    W = torch.randn(K, N, device=dev, generator=g) * 0.02
    dY = torch.randn(M, N, device=dev, generator=g) * 1e-3
    dX, dW = torch.zeros(M, K, device=dev), torch.zeros(K, N, device=dev)
    flush = torch.empty(64 * 1024 * 1024, device=dev)  # 256 MB > 126 MB L2
    with torch.cuda.stream(stream):
        for _ in range(3):
            ops.linear_bwd(X, W, dY, dX, dW, None, M, K, N)
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for k0, k1 in evs:
            flush.fill_(1.0)
            k0.record(stream)
            ops.linear_bwd(X, W, dY, dX, dW, None, M, K, N)
            k1.record(stream)
        torch.cuda.synchronize()
    return sum(k0.elapsed_time(k1) for k0, k1 in evs) / reps, 2 * 2.0 * M * K * N


# ------------------------------------------------------------ kernel sweep
def run_sweep(args):
    """linear backward (dX = dY W^T, dW = X^T dY) at M=N=K = n,
    LayerNorm backward over 65536 rows of width w, and the fused clip +
    AdamW over 256 tensors totalling 1e8 parameters.  One JSON line per
    case with achieved FLOP/s or bytes/s against the measured peaks (CUDA
    events around `reps` launches, after warm-up; inputs larger than L2
    except the two smallest GEMMs)."""
    import numpy as np
    import torch

    from ml_engine_b200 import ops
    dev = torch.device("cuda", 0)
    hbm_peak, bf16_peak, kind = load_peaks()
    tf32_peak = bf16_peak / 2
    g = torch.Generator(device=dev).manual_seed(0)

    def timed(fn, reps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    for n in (512, 1024, 2048, 4096, 8192):
        X = torch.randn(n, n, device=dev, generator=g)
        W = torch.randn(n, n, device=dev, generator=g)
        dY = torch.randn(n, n, device=dev, generator=g)
        dX, dW = torch.zeros(n, n, device=dev), torch.zeros(n, n, device=dev)
        ms = timed(lambda: ops.linear_bwd(X, W, dY, dX, dW, None, n, n, n), 20 if n >= 4096 else 100)
        tf = 4.0 * n ** 3 / (ms * 1e-3) / 1e12
        print(json.dumps({"sweep": "linear_bwd", "n": n, "ms": ms, "tflops": tf, "frac_of_tf32": tf / tf32_peak,
                          "frac_of_bf16": tf / bf16_peak, "peak_kind": kind}), flush=True)
        del X, W, dY, dX, dW
    rows = 65536
    for w in (1024, 2048, 4096, 8192):
        x = torch.randn(rows * w, device=dev, generator=g)
        y, mean, sq = torch.empty_like(x), torch.empty(rows, device=dev), torch.empty(rows, device=dev)
        ops.layernorm_fwd(x, y, mean, sq, rows, 1, 1, w)
        gy, gx = torch.randn_like(x), torch.zeros_like(x)
        ms = timed(lambda: ops.layernorm_bwd(y, gy, sq, gx, rows, 1, 1, w), 20)
        gbs = 16.0 * rows * w / (ms * 1e-3) / 1e9   # y, gy, gx read; gx written
        print(json.dumps({"sweep": "layernorm_bwd", "rows": rows, "width": w, "ms": ms, "gbs": gbs,
                          "frac_of_hbm": gbs / hbm_peak, "peak_kind": kind}), flush=True)
        del x, y, gy, gx
    total, nt = 100_000_000, 256
    sizes = np.random.default_rng(0).integers(1, 1000, nt).astype(np.float64)
    sizes = np.maximum(1, (sizes / sizes.sum() * total).astype(np.int64))
    params = []
    for sz in sizes:
        params.append(dict(w=torch.randn(int(sz), device=dev, generator=g) * 0.02,
                           g=torch.randn(int(sz), device=dev, generator=g) * 1e-2,
                           m=torch.zeros(int(sz), device=dev), v=torch.zeros(int(sz), device=dev),
                           t=torch.ones(1, dtype=torch.int32, device=dev)))
    ws = torch.zeros(1, dtype=torch.float64, device=dev)
    views = ops.param_views(params)   # built once, as the engine's optimizer does

    def clip_adam():
        ws.zero_()
        ops.grad_sumsq(views, ws)
        ops.clip_finalize(ws, 1.0)
        ops.adam_update(views, lr=1e-3, adamw=True, clip_ws=ws, write_back_grad=False)
    ms = timed(clip_adam, 10)
    nparam = int(sizes.sum())
    gbs = 32.0 * nparam / (ms * 1e-3) / 1e9   # g read (norm); w, g, m, v read; w, m, v written
    print(json.dumps({"sweep": "clip_adamw", "params": nparam, "tensors": nt, "ms": ms, "gbs": gbs,
                      "frac_of_hbm": gbs / hbm_peak, "peak_kind": kind}), flush=True)


# ------------------------------------------------------------ U-Net workload
def run_unet(args):
    """configs[3] (single GPU): DDPM noise-prediction step on 32 x 3 x 64 x
    64 images, widths 64/128/256, time embedding 256.  x_t = sqrt(abar) x0
    + sqrt(1 - abar) eps with x0, eps ~ N(0, 1) and the linear beta schedule
    1e-4 .. 0.02 at the session's timestep; the step is zero_grad + forward
    + backward + clip(1.0) + AdamW, replayed as a captured CUDA graph."""
    import numpy as np
    import torch

    from ml_engine_b200.session import Session
    dev = torch.device("cuda", 0)
    B, C, S = 32, 3, 64
    t = 500
    betas = np.linspace(1e-4, 0.02, 1000)
    abar = float(np.prod(1.0 - betas[: t + 1]))
    s = Session.unet(batch=B, channels=C, image_size=S, base_width=64, t_embed=256, timestep=t, lr=1e-3, adamw=1,
                     clip_norm=1.0, seed=4321)
    rng = np.random.default_rng(7)
    pool = []
    for _ in range(4):
        x0 = rng.standard_normal(B * C * S * S).astype(np.float32)
        eps = rng.standard_normal(B * C * S * S).astype(np.float32)
        pool.append(((np.sqrt(abar) * x0 + np.sqrt(1 - abar) * eps).astype(np.float32), eps))
    stream = torch.cuda.ExternalStream(s.stream, device=dev)

    def feed(i):
        s.inputs["x_t"][:], s.inputs["noise"][:] = pool[i % len(pool)]

    feed(0)
    s.step()
    s.capture()
    for i in range(max(args.warmup, 3)):
        feed(i)
        s.step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        s.step(upload=False, read_loss=False)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for i in range(args.steps):
        feed(i)
        loss = s.step(upload=True, read_loss=True)
    e3.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e2.elapsed_time(e3) / args.steps
    print(json.dumps({"metric": "train images/s (fwd+bwd+AdamW), configs[3] U-Net", "value": B * 1e3 / ms,
                      "unit": "images/s", "steps_per_s": 1e3 / ms, "ms_per_step": ms, "n_gpus": 1, "steps": args.steps,
                      "warmup": args.warmup, "dtype": "f32 (tf32 tensor-core products)", "data": "synthetic",
                      "config": {"workload": "configs[3]: U-Net 32x3x64x64, widths 64/128/256, t_embed 256",
                                 "global_batch": B},
                      "e2e": {"value": B * 1e3 / e2e_ms, "unit": "images/s", "ms_per_step": e2e_ms,
                              "h2d_bytes_per_step": 2 * B * C * S * S * 4, "d2h_bytes_per_step": 4,
                              "loss_last": loss}}), flush=True)
    s.close()


# ------------------------------------------------------ encoder-decoder workload
def run_encdec(args, rank, world, local_rank):
    """6+6-layer encoder-decoder (d 512, 8 heads, FFN 2048,
    seq 256, vocab 8192), global batch 256 split over the ranks (strong
    scaling); token ids Zipf(s=1.1) over the vocabulary, next-token targets;
    one step = zero_grad + forward + backward + bucketed NCCL allreduce +
    clip(1.0) + AdamW, replayed as a captured CUDA graph."""
    import numpy as np
    import torch

    from ml_engine_b200.session import Session
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    GB, S, V = 256, 256, 8192
    if GB % world:
        raise SystemExit(f"global batch {GB} does not split over {world} ranks")
    B = GB // world
    s = Session.encdec(batch=B, seq_len=S, d_model=512, heads=8, ffn=2048, layers=6, vocab=V, lr=1e-4, adamw=1,
                       clip_norm=1.0, fused_attention=1, seed=2024)
    if world > 1:
        import torch.distributed as dist
        uid = [Session.dp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        s.enable_dp(uid[0], rank, world, bucket_mb=args.bucket_mb or 32)
    stream = torch.cuda.ExternalStream(s.stream, device=dev)
    rng = np.random.default_rng(3000 + rank)
    zipf = 1.0 / np.arange(1, V + 1) ** 1.1
    zipf /= zipf.sum()
    pool = []
    for _ in range(4):
        seq = rng.choice(V, size=(B, S + 1), p=zipf).astype(np.int32)
        src = rng.choice(V, size=(B, S), p=zipf).astype(np.int32)
        pool.append((src.ravel(), seq[:, :S].ravel().copy(), seq[:, 1:].ravel().copy()))

    def feed(i):
        s.inputs["src"][:], s.inputs["tgt_in"][:], s.inputs["tgt_out"][:] = pool[i % len(pool)]

    feed(0)
    s.step()
    s.capture()
    for i in range(max(args.warmup, 3)):
        feed(i)
        s.step()
    import ctypes
    kk, mm, cc = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    s._lib.call("mle_session_graph_counts", s._h, ctypes.addressof(kk), ctypes.addressof(mm), ctypes.addressof(cc))
    smi_index = os.environ.get("CUDA_VISIBLE_DEVICES", str(local_rank)).split(",")[local_rank] \
        if "CUDA_VISIBLE_DEVICES" in os.environ else str(local_rank)
    with ClockSampler(smi_index) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            s.step(upload=False, read_loss=False)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world, dev)
        barrier(world)
        torch.cuda.synchronize()
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        loss = None
        for i in range(args.steps):
            feed(i)
            loss = s.step(upload=True, read_loss=True)
        e3.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        e2e_ms = max_over_ranks(e2.elapsed_time(e3) / args.steps, world, dev)
    if rank == 0:
        print(json.dumps({
            "metric": "train steps/s (fwd+bwd+AdamW), configs[2] encoder-decoder", "value": 1e3 / ms,
            "unit": "steps/s", "tokens_per_s": GB * S * 1e3 / ms, "ms_per_step": ms, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
            "dtype": "f32 (tf32 tensor-core products)", "data": "synthetic (Zipf(1.1) token ids)",
            "config": {"workload": "configs[2]: enc-dec 6+6, d 512, 8 heads, FFN 2048, seq 256, vocab 8192",
                       "global_batch": GB, "per_rank_batch": B, "seq_len": S, "parallelism": f"dp{world}"},
            "e2e": {"value": 1e3 / e2e_ms, "unit": "steps/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": 3 * B * S * 4, "d2h_bytes_per_step": 4, "loss_last": loss},
            "gpu_launches": kk.value * args.steps, "clocks": clocks.summary()}), flush=True)
    s.close()


# ------------------------------------------------------------ native arm
def run_native(args, rank, world, local_rank):
    import numpy as np
    import torch

    from ml_engine_b200.session import Session

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    hbm_peak, tf_peak, peak_kind = load_peaks()

    s = Session.encoder(**CFG, lr=1e-3, adamw=1, clip_norm=1.0, fused_attention=1, seed=1234)
    if world > 1:
        import torch.distributed as dist
        uid = [Session.dp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        s.enable_dp(uid[0], rank, world, bucket_mb=args.bucket_mb or 4)
    stream = torch.cuda.ExternalStream(s.stream, device=dev)

    rng = np.random.default_rng(1000 + rank)
    pool = [(rng.integers(0, CFG["vocab"], TOKENS_PER_STEP).astype(np.int32),
             rng.integers(0, CFG["vocab"], TOKENS_PER_STEP).astype(np.int32)) for _ in range(16)]

    def feed(i):
        tok, tgt = pool[i % len(pool)]
        s.inputs["tokens"][:] = tok
        s.inputs["targets"][:] = tgt

    feed(0)
    s.step()                 # eager step: builds tensor maps, configures kernels
    s.capture()
    for i in range(max(args.warmup, 3)):
        feed(i)
        s.step()
    kernels = memsets = copies = 0
    import ctypes
    kk, mm, cc = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    s._lib.call("mle_session_graph_counts", s._h, ctypes.addressof(kk), ctypes.addressof(mm), ctypes.addressof(cc))
    kernels, memsets, copies = kk.value, mm.value, cc.value

    smi_index = os.environ.get("CUDA_VISIBLE_DEVICES", str(local_rank)).split(",")[local_rank] \
        if "CUDA_VISIBLE_DEVICES" in os.environ else str(local_rank)
    # ---------------------------------------------------------------- value
    with ClockSampler(smi_index) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            s.step(upload=False, read_loss=False)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        dev_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world, dev)

        # ------------------------------------------------------------- e2e
        barrier(world)
        torch.cuda.synchronize()
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        losses = []
        for i in range(args.steps):
            feed(args.warmup + i)
            losses.append(s.step(upload=True, read_loss=True))
        e3.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        e2e_ms = max_over_ranks(e2.elapsed_time(e3) / args.steps, world, dev)
    clk = clocks.summary()

    kern_ms, flops_pair = roofline_pair(dev, stream)
    achieved_tf = flops_pair / (kern_ms * 1e-3) / 1e12
    traffic = None
    prof = ROOT / "profiles" / "traffic.json"
    if prof.exists():
        traffic = json.loads(prof.read_text()).get("proj_bwd_gemm_pair_bytes")

    value = world * 1e3 / dev_ms
    line = {
        "metric": METRIC, "value": value, "unit": "steps/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (tf32 tensor-core products)", "data": "synthetic",
        "tokens_per_s": value * TOKENS_PER_STEP,
        "config": {"workload": WORKLOAD, "global_batch": CFG["batch"] * world, "seq_len": CFG["seq_len"],
                   "parallelism": f"dp{world}", "step": "zero_grad+fwd+bwd+clip(1.0)+AdamW, captured CUDA graph",
                   "l2": "no flush: the step touches ~1 GB (> 126 MB L2) per iteration"},
        "e2e": {"value": world * 1e3 / e2e_ms, "unit": "steps/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": 2 * TOKENS_PER_STEP * 4, "d2h_bytes_per_step": 4,
                "loss_last": losses[-1] if losses else None},
        "roofline": {"bound": "tensor", "kernel": "tcgen05 tf32 GEMM pair of the projection backward (dX, dW)",
                     "achieved": achieved_tf, "peak": tf_peak, "unit": "TFLOP/s", "frac": achieved_tf / tf_peak,
                     "peak_kind": f"{peak_kind} bf16 dense (tf32 dense is half of it)",
                     "frac_of_tf32": achieved_tf / (tf_peak / 2), "traffic": traffic, "ms_per_launch_pair": kern_ms},
        "gpu_launches": kernels * args.steps,
        "launches_per_step": {"kernels": kernels, "memsets": memsets, "copies": copies},
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, sample = cpu_sample(seconds=args.cpu_seconds)
        line["cpu_baseline"] = {"value": v, "unit": "steps/s", "cores": cores, "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    s.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="configs[4] kernel sweep, one JSON line per case")
    ap.add_argument("--config", default="encoder", choices=["encoder", "unet", "encdec"],
                    help="encoder: configs[1], the benchmark line; unet: configs[3] on one GPU; "
                         "encdec: configs[2], global batch 256 over the ranks")
    ap.add_argument("--gemm-pairs", type=int, default=None, choices=[0, 1, 2],
                    help="run large products on CTA pairs (mle_set_gemm_pairs); default: the library's")
    ap.add_argument("--attn-path", default=None, choices=["auto", "fused", "tensor"],
                    help="attention implementation (mle_set_attention_path); default: the library's")
    ap.add_argument("--param-stream", type=int, default=None, choices=[0, 1],
                    help="weight/bias gradients on a second stream (mle_set_param_grad_stream); default: on")
    ap.add_argument("--stage-kblocks", type=int, default=None, choices=[1, 2],
                    help="GEMM k-blocks per pipeline stage (mle_set_gemm_stage_kblocks); default: the library's")
    ap.add_argument("--bucket-mb", type=int, default=None,
                    help="data-parallel gradient bucket size in MiB (mle_session_enable_dp); default 4 for "
                         "configs[1] (its 10.5 MB of gradients then reduce in a few buckets during the "
                         "backward), 32 for configs[2]")
    ap.add_argument("--roofline-only", action="store_true",
                    help="run only the roofline kernel pair (3 untimed + 20 timed pairs)")
    args = ap.parse_args()
    if args.gemm_pairs is not None:
        from ml_engine_b200._lib import kernels
        kernels().call("mle_set_gemm_pairs", args.gemm_pairs)
    if args.attn_path is not None:
        from ml_engine_b200._lib import kernels
        kernels().call("mle_set_attention_path", {"auto": 0, "fused": 1, "tensor": 2}[args.attn_path])
    if args.stage_kblocks is not None:
        from ml_engine_b200._lib import kernels
        kernels().call("mle_set_gemm_stage_kblocks", args.stage_kblocks)
    if args.param_stream is not None:
        from ml_engine_b200._lib import engine
        engine().call("mle_set_param_grad_stream", args.param_stream)
    if args.sweep:
        run_sweep(args)
        return
    if args.config == "unet":
        run_unet(args)
        return
    if args.roofline_only:
        import torch
        dev = torch.device("cuda", 0)
        ms, flops = roofline_pair(dev, torch.cuda.current_stream(dev), reps=20)
        print(json.dumps({"roofline_pair_ms": ms, "flop": flops}))
        return
    world, rank, local_rank = init_ranks()
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.config == "encdec":
            run_encdec(args, rank, world, local_rank)
        else:
            run_native(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
