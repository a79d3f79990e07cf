#!/usr/bin/env python
"""Training-step benchmark of the ML_Engine hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]
                    [--config encdec|encoder|mlp|unet] [--sweep]

Default workload: BASELINE configs[2] -- 6+6-layer encoder-decoder, d_model
512, 8 heads, FFN 2048 (GELU), seq 256, vocab 8192, global batch 256 split
over the ranks (strong scaling), Zipf(1.1) token ids, next-token softmax
cross-entropy, AdamW with clipNorm 1.0.  One step = zero_grad + forward +
backward + bucketed NCCL all-reduce (N > 1) + clip + AdamW over the rank's
batch, replayed as a captured CUDA graph.  `--config encoder` is configs[1]
(batch 32 x seq 128 per rank, weak scaling), `--config mlp` configs[0],
`--config unet` configs[3] (one GPU), `--sweep` the configs[4] kernels.

Legs (CUDA events on the session's stream, max over ranks):
  value     steps/s of the whole job, inputs resident in HBM;
  e2e       the same through the public API with host buffers: every step
            refills the pinned host inputs, uploads them, runs the step and
            reads the loss back;
  bwd_roofline  the backward phase alone (its own captured graph) against
            the algorithmic backward work: tensor FLOP at TF32 plus the
            elementwise/normalisation/softmax bytes at HBM bandwidth;
  roofline  the dominant kernel, the tcgen05 TF32 GEMM, on every Linear
            backward product (dX, dW) of the workload at the rank's token
            count, each after an L2-evicting write;
  ref_cuda  (N = 1, rank 0) the reference's OWN training step -- its
            GraphOperations runtime, layer classes and CUDA kernels compiled
            from its sources (oracle/_ref/librefstep.so) -- on configs[0],
            configs[1] and configs[2] at 32 sequences, with this
            implementation's step at the same shapes beside it;
  cpu_baseline  (N = 1, rank 0) the C oracle's step on the host cores, on a
            bounded sample.
The baseline legs (ref_cuda, cpu_baseline, --impl reference) are the only
code here that runs anything under oracle/; the measured path is the
session ABI of libmle_engine.so.

--impl reference times the reference's path on the host cores: the
reference is CUDA-only, so its CPU arm is the oracle's C restatement of the
same graph (oracle/mle_oracle.c + oracle/graphs.py), all host threads.
"""
from __future__ import annotations

import argparse
import ctypes
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

METRIC = "train steps/s (fwd+bwd+AdamW) at 1/2/4/8 B200; bwd % of roofline"

WORKLOADS = {
    "encdec": dict(
        cfg=dict(seq_len=256, d_model=512, heads=8, ffn=2048, layers=6, vocab=8192),
        global_batch=256, scaling="strong",
        name="configs[2]: encoder-decoder 6+6, d 512, 8 heads, FFN 2048 GELU, seq 256, vocab 8192, "
             "global batch 256 over the ranks"),
    "encoder": dict(
        cfg=dict(seq_len=128, d_model=256, heads=8, ffn=1024, layers=2, vocab=4096),
        per_rank_batch=32, scaling="weak",
        name="configs[1]: 2-layer pre-LN transformer encoder, batch 32 x seq 128 per rank, d256 h8 ffn1024 gelu, "
             "vocab 4096"),
    "mlp": dict(
        cfg=dict(in_features=784, hidden=256, classes=10),
        per_rank_batch=64, scaling="weak",
        name="configs[0]: MLP 784-256(ReLU)-10, batch 64 per rank, softmax cross-entropy"),
}
L2_NOTE = {
    "encdec": "no flush: a step moves ~10^2 GB through HBM (> 126 MB L2)",
    "encoder": "no flush: a step moves ~1 GB through HBM (> 126 MB L2)",
    "mlp": "no flush: the whole step (~2 MB) is L2-resident, as it is for the reference",
}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


BATCH_OVERRIDE = None   # --batch: per-rank batch for profiling runs (not a bench line)


def local_batch(wl, world):
    if BATCH_OVERRIDE:
        return BATCH_OVERRIDE
    w = WORKLOADS[wl]
    if "global_batch" in w:
        if w["global_batch"] % world:
            raise SystemExit(f"global batch {w['global_batch']} does not split over {world} ranks")
        return w["global_batch"] // world
    return w["per_rank_batch"]


def config_dict(wl, world):
    """The `config` object of both arms (identical by construction)."""
    w = WORKLOADS[wl]
    B = local_batch(wl, world)
    d = {"workload": w["name"], "global_batch": B * world, "per_rank_batch": B, "parallelism": f"dp{world}",
         "l2": L2_NOTE[wl]}
    if "seq_len" in w["cfg"]:
        d["seq_len"] = w["cfg"]["seq_len"]
    return d


def units_per_step(wl, B):
    """(tokens or images per step for B sequences/images, unit name)."""
    c = WORKLOADS[wl]["cfg"]
    if wl == "mlp":
        return B, "images/s"
    return B * c["seq_len"], "tokens/s"


# ------------------------------------------------------- algorithmic work
def linear_shapes(wl):
    """(in, out, count) of every Linear in the step's graph."""
    c = WORKLOADS[wl]["cfg"]
    if wl == "mlp":
        return [(c["in_features"], c["hidden"], 1), (c["hidden"], c["classes"], 1)]
    D, F, L, V = c["d_model"], c["ffn"], c["layers"], c["vocab"]
    attn = 4 * L * (1 if wl == "encoder" else 3)   # enc self; dec self + cross
    return [(D, D, attn), (D, F, L * (1 if wl == "encoder" else 2)), (F, D, L * (1 if wl == "encoder" else 2)),
            (D, V, 1)]


def backward_work(wl, B):
    """Algorithmic backward work of one step on B sequences: tensor FLOP
    (Linear dX and dW, 4 attention products per attention block) and the
    bytes the non-GEMM backward ops must move (fp32, each tensor read or
    written once): LayerNorm 16 B/elem, GELU 12, residual Add 12, loss
    gradient 8 B/logit.  The attention's score matrices need not reach HBM
    (the flash kernels keep them on chip), so they add no bytes; its
    recomputed score products are not counted as work either.  The MLP's
    tiny elementwise ops are left out."""
    c = WORKLOADS[wl]["cfg"]
    if wl == "mlp":
        T = B
        return sum(4.0 * T * i * o * n for i, o, n in linear_shapes(wl)), 0.0
    S, D, H, F, L, V = c["seq_len"], c["d_model"], c["heads"], c["ffn"], c["layers"], c["vocab"]
    T = B * S
    flop = sum(4.0 * T * i * o * n for i, o, n in linear_shapes(wl))
    blocks = L if wl == "encoder" else 3 * L
    flop += blocks * 4 * 2.0 * B * H * S * S * (D // H)
    lns = 2 * L if wl == "encoder" else 5 * L
    adds = lns
    ffns = L if wl == "encoder" else 2 * L
    byts = 16.0 * lns * T * D + 12.0 * adds * T * D + 12.0 * ffns * T * F + 8.0 * T * V
    return flop, byts


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
                                          "--format=csv,noheader,nounits", "-lms", "50"],
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
            time.sleep(0.15)   # the last sample of the timed region
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = sorted(v for v in (num(s[0]) for s in self.samples) if v is not None)
        mxs = [v for v in (num(s[1]) for s in self.samples) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[4 + i].strip() == "Active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": max(mxs) if mxs else None,
                "reasons": reasons, "samples": len(self.samples)}


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


def smi_index(local_rank):
    if "CUDA_VISIBLE_DEVICES" in os.environ:
        return os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local_rank]
    return str(local_rank)


# ------------------------------------------------------------ inputs
def input_pool(wl, B, seed, n=4):
    """Seeded synthetic inputs per step: Zipf(1.1) token ids over the
    vocabulary with next-token targets, uniform ids
    (configs[1]), U[0,1) images with uniform labels."""
    import numpy as np
    c = WORKLOADS[wl]["cfg"]
    rng = np.random.default_rng(seed)
    pool = []
    for _ in range(n):
        if wl == "encdec":
            V, S = c["vocab"], c["seq_len"]
            zipf = 1.0 / np.arange(1, V + 1) ** 1.1
            zipf /= zipf.sum()
            seq = rng.choice(V, size=(B, S + 1), p=zipf).astype(np.int32)
            src = rng.choice(V, size=(B, S), p=zipf).astype(np.int32)
            pool.append({"src": src.ravel(), "tgt_in": seq[:, :S].ravel().copy(),
                         "tgt_out": seq[:, 1:].ravel().copy()})
        elif wl == "encoder":
            V, S = c["vocab"], c["seq_len"]
            pool.append({"tokens": rng.integers(0, V, B * S).astype(np.int32),
                         "targets": rng.integers(0, V, B * S).astype(np.int32)})
        else:
            pool.append({"x": rng.random(B * c["in_features"], dtype=np.float32),
                         "labels": rng.integers(0, c["classes"], B).astype(np.int32)})
    return pool


def make_session(wl, B, seed=2024, **kw):
    from ml_engine_b200.session import Session
    c = WORKLOADS[wl]["cfg"]
    if wl == "encdec":
        return Session.encdec(batch=B, **c, lr=1e-4, adamw=1, clip_norm=1.0, fused_attention=1, seed=seed, **kw)
    if wl == "encoder":
        return Session.encoder(batch=B, **c, lr=1e-3, adamw=1, clip_norm=1.0, fused_attention=1, seed=seed, **kw)
    return Session.mlp(batch=B, **c, lr=1e-3, adamw=1, clip_norm=1.0, seed=seed, **kw)


def feed(s, item):
    for k, v in item.items():
        s.inputs[k][:] = v


def time_replays(s, stream, steps):
    """ms per captured device-resident step (CUDA events on the stream)."""
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        s.step(upload=False, read_loss=False)
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / steps


def time_phases(s, stream, steps):
    """Mean ms of (forward incl. zero_grad, backward, all-reduce + clip +
    update) over `steps` replays of the per-phase graphs."""
    import torch
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
    for ev in evs:
        ev[0].record(stream)
        s.phase_replay(0)
        s.phase_replay(1)
        ev[1].record(stream)
        s.phase_replay(2)
        ev[2].record(stream)
        for ph in (3, 4, 5):
            s.phase_replay(ph)
        ev[3].record(stream)
    torch.cuda.synchronize()
    out = [0.0, 0.0, 0.0]
    for ev in evs:
        for i in range(3):
            out[i] += ev[i].elapsed_time(ev[i + 1]) / steps
    return out


# ------------------------------------------------------------ roofline kernel
def roofline_gemms(wl, B, dev, stream, reps=5):
    """The tcgen05 TF32 GEMM on every Linear backward product of the step
    at the rank's token count T (dX = dY W^T and dW = X^T dY, 4 T in out
    FLOP per pair): per distinct shape, 2 untimed pairs, then `reps` pairs
    each between its own CUDA events after a 256 MB write that evicts the
    operands from L2.  Returns (per-shape rows, total FLOP, total ms), the
    totals weighted by how often each shape occurs in one step."""
    import torch

    from ml_engine_b200 import ops
    c = WORKLOADS[wl]["cfg"]
    T = B * c.get("seq_len", 1)
    g = torch.Generator(device=dev).manual_seed(0)
    flush = torch.empty(64 * 1024 * 1024, device=dev)  # 256 MB > 126 MB L2
    rows, tot_flop, tot_ms = [], 0.0, 0.0
    with torch.cuda.stream(stream):
        for fin, fout, count in linear_shapes(wl):
            X = torch.randn(T, fin, device=dev, generator=g)
            W = torch.randn(fin, fout, device=dev, generator=g) * 0.02
            dY = torch.randn(T, fout, device=dev, generator=g) * 1e-3
            dX, dW = torch.zeros(T, fin, device=dev), torch.zeros(fin, fout, device=dev)
            for _ in range(2):
                ops.linear_bwd(X, W, dY, dX, dW, None, T, fin, fout)
            torch.cuda.synchronize()
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
            for k0, k1 in evs:
                flush.fill_(1.0)
                k0.record(stream)
                ops.linear_bwd(X, W, dY, dX, dW, None, T, fin, fout)
                k1.record(stream)
            torch.cuda.synchronize()
            ms = sum(k0.elapsed_time(k1) for k0, k1 in evs) / reps
            flop = 4.0 * T * fin * fout
            rows.append({"shape": f"T{T} x {fin} -> {fout}", "per_step": count, "ms_per_pair": ms,
                         "tflops": flop / (ms * 1e-3) / 1e12})
            tot_flop += count * flop
            tot_ms += count * ms
            del X, W, dY, dX, dW
    return rows, tot_flop, tot_ms


def roofline_only(args):
    """Only the roofline GEMM pairs (for ncu captures of the kernel)."""
    import torch
    dev = torch.device("cuda", 0)
    B = args.roofline_batch or local_batch(args.config, 1)
    rows, flop, ms = roofline_gemms(args.config, B, dev, torch.cuda.current_stream(dev), reps=args.roofline_reps)
    print(json.dumps({"rows": rows, "flop": flop, "ms": ms}))


# ------------------------------------------------------------ reference CUDA
REF_CASES = [
    # name, workload, batch, timed steps
    ("configs[0]", "mlp", 64, 30),
    ("configs[1]", "encoder", 32, 10),
    ("configs[2] at 32 sequences (one rank's share at 8 GPUs)", "encdec", 32, 2),
]


def ref_cuda_leg(dev):
    """The reference's own step (librefstep.so) beside ours, same shapes."""
    import numpy as np
    import torch

    from oracle import ref
    if not ref.step_available():
        return {"unavailable": "oracle/_ref/librefstep.so was not built (the reference source tree was absent "
                               "at build time)"}
    L = ref.step_lib()
    out = {"what": "the reference's GraphOperations runtime, layer classes and CUDA kernels compiled from its "
                   "sources (Engine/{engine,kernels,debug,transformer}.cu), graphs built through its API "
                   "(oracle/ref_step.cu); one step = zero_grad, token gather, forward, backward, clip(1.0), "
                   "AdamW, launched as the reference launches them (legacy stream, its own device syncs); "
                   "CUDA events per phase", "cases": []}
    for name, wl, B, steps in REF_CASES:
        c = WORKLOADS[wl]["cfg"]
        if wl == "mlp":
            args_ = (1, B, c["in_features"], c["hidden"], c["classes"], 0, 0, 0, 0, 0, 0)
        else:
            args_ = (2 if wl == "encoder" else 3, B, 0, 0, 0, c["seq_len"], c["d_model"], c["heads"], c["ffn"],
                     c["layers"], c["vocab"])
        st = L.refstep_create(*args_)
        if st != 0:
            out["cases"].append({"case": name, "error": f"refstep_create: cuda error {st}"})
            L.refstep_destroy()
            continue
        item = input_pool(wl, B, seed=77, n=1)[0]
        for k, v in item.items():
            L.refstep_input_write(k.encode(), v.ctypes.data, v.size)
        ms = (ctypes.c_double * 4)()
        st = L.refstep_time(1, steps, 1e-3, 1, 1.0, ms)
        ref_ms = list(ms)
        L.refstep_destroy()
        torch.cuda.synchronize()
        # this implementation at the same shape
        s = make_session(wl, B)
        stream = torch.cuda.ExternalStream(s.stream, device=dev)
        feed(s, item)
        s.step()
        s.capture()
        for _ in range(3):
            s.step(upload=False, read_loss=False)
        torch.cuda.synchronize()
        ours = time_replays(s, stream, max(steps, 10))
        s.capture_phases()
        f_ms, b_ms, o_ms = time_phases(s, stream, max(3, min(steps, 10)))
        s.close()
        out["cases"].append({
            "case": name, "batch": B, "status": st,
            "ref_ms": {"forward": ref_ms[0], "backward": ref_ms[1], "clip_update": ref_ms[2], "step": ref_ms[3]},
            "ours_ms": {"forward": f_ms, "backward": b_ms, "allreduce_clip_update": o_ms, "step": ours},
            "speedup_step": ref_ms[3] / ours,
            "speedup_bwd_plus_update": (ref_ms[1] + ref_ms[2]) / (b_ms + o_ms)})
    return out


# ------------------------------------------------------------ CPU baseline
def _cpu_problem(wl, seed=0):
    import numpy as np
    c = WORKLOADS[wl]["cfg"]
    rng = np.random.default_rng(seed)
    if wl == "mlp":
        sizes = [c["in_features"] * c["hidden"], c["hidden"], c["hidden"] * c["classes"], c["classes"]]
        return [(rng.standard_normal(n) * 0.05).astype(np.float32) for n in sizes], None
    D, F, V, L = c["d_model"], c["ffn"], c["vocab"], c["layers"]
    sizes = []
    for _ in range(L):
        sizes += [D * D, D] * 4 + [D * F, F, F * D, D]
    if wl == "encdec":
        for _ in range(L):
            sizes += [D * D, D] * 8 + [D * F, F, F * D, D]
    sizes += [D * V, V]
    params = [(rng.standard_normal(n) * 0.02).astype(np.float32) for n in sizes]
    tables = [(rng.standard_normal(V * D) * 0.02).astype(np.float32) for _ in range(2 if wl == "encdec" else 1)]
    return params, tables


def cpu_fwd_bwd(wl, params, tables, B, seed):
    """One oracle forward + backward over B sequences/images (no update)."""
    from oracle import graphs
    c = WORKLOADS[wl]["cfg"]
    item = input_pool(wl, B, seed=seed, n=1)[0]
    if wl == "mlp":
        return graphs.mlp_step(params, item["x"].reshape(B, -1), item["labels"], classes=c["classes"],
                               update=False)
    if wl == "encoder":
        return graphs.encoder_step(params, tables[0], item["tokens"].reshape(B, -1), item["targets"].reshape(B, -1),
                                   B, c["seq_len"], c["d_model"], c["heads"], c["ffn"], c["layers"], c["vocab"],
                                   update=False)
    return graphs.encdec_step(params, tables, item["src"].reshape(B, -1), item["tgt_in"].reshape(B, -1),
                              item["tgt_out"].reshape(B, -1), B, c["seq_len"], c["d_model"], c["heads"], c["ffn"],
                              c["layers"], c["vocab"], update=False)


def cpu_sample_plan(wl, B_full):
    """Sequences (images) per sampled step: the whole batch where the CPU
    finishes it in seconds, one sequence of
    configs[2] (a full configs[2] step is ~10^3 s on the host)."""
    return 1 if wl == "encdec" else B_full


def cpu_step_times(wl, B_full, n_steps, warm=1, params=None):
    """Per sampled step: (estimated full-step seconds, sample seconds).  A
    step's forward+backward is timed on the sample and scaled to the full
    batch; the clip + AdamW over all parameters is timed once per step on
    the gradients the sample produced (it does not scale with the batch)."""
    from oracle import graphs
    params_, tables = _cpu_problem(wl)
    sb = cpu_sample_plan(wl, B_full)
    times = []
    for i in range(warm + n_steps):
        t0 = time.perf_counter()
        r = cpu_fwd_bwd(wl, params_, tables, sb, seed=500 + i)
        t1 = time.perf_counter()
        graphs.clip_and_update([p.ravel() for p in params_], r["grads"], [1] * len(params_), 1e-3, 1.0)
        t2 = time.perf_counter()
        if i >= warm:
            times.append(((t1 - t0) * B_full / sb + (t2 - t1), t2 - t0))
    return times, sb


def cpu_cores():
    """Every host core for the oracle's loops (a launcher such as torchrun
    pins OMP_NUM_THREADS to 1 per rank; the CPU arm runs on rank 0 alone);
    returns the thread count in force."""
    from oracle import ops as orc
    return orc.set_threads(os.cpu_count() or 1)


def cpu_baseline_leg(wl, B_full, seconds):
    cores = cpu_cores()
    times, sb = [], None
    t0 = time.perf_counter()
    while not times or time.perf_counter() - t0 < seconds:
        tt, sb = cpu_step_times(wl, B_full, 1, warm=0 if times else 1)
        times += tt
    full = sum(t for t, _ in times) / len(times)
    spent = sum(s for _, s in times)
    unit = "sequences" if wl != "mlp" else "images"
    return {"value": 1.0 / full, "unit": "steps/s", "cores": cores, "kind": "port",
            "sample": f"{len(times)} sampled steps: forward+backward on {sb} of {B_full} {unit} scaled x{B_full // sb}, "
                      f"plus the clip + AdamW over all parameters once per step; {spent:.1f}s of host time"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    wl = args.config
    B = local_batch(wl, world)
    n_gpu_b = B * world
    # the reference arm runs the whole job's batch (all ranks' shares) on the host
    cores = cpu_cores()
    times, sb = cpu_step_times(wl, n_gpu_b, args.steps, warm=min(args.warmup, 1))
    full = sum(t for t, _ in times) / len(times)
    value = 1.0 / full
    unit = "sequences" if wl != "mlp" else "images"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "steps/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * full,
        "higher_is_better": True, "scaling": WORKLOADS[wl]["scaling"], "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": config_dict(wl, world),
        "cpu_baseline": {"value": value, "unit": "steps/s", "cores": cores, "kind": "port",
                         "sample": f"per step: forward+backward on {sb} of {n_gpu_b} {unit}, scaled "
                                   f"x{n_gpu_b // sb}, plus the clip + AdamW over all parameters; "
                                   f"{min(args.warmup, 1)} warm-up sample"},
        "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference is CUDA-only; its CPU arm is the oracle's C restatement of the same graph "
                "(oracle/mle_oracle.c + oracle/graphs.py, OpenMP) on the host cores",
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ kernel sweep
def run_attention(args):
    """The attention block of configs[2] (8 heads of 64, seq 256, token-major
    [B, S, 512] projections; B = the rank's 256 sequences, or --batch),
    masked (decoder self-attention) and unmasked (encoder, cross), on both
    tensor-core paths: the keys-on-lanes kernels writing P and the score
    gradient to HBM beside tcgen05 GEMMs, and the flash kernels (scores on
    chip, P recomputed from per-key statistics).  Forward and backward
    (reference key gradient, gradients assigned) timed apart with CUDA
    events over `--steps` launches after `--warmup`; one JSON line per
    case, with the algorithmic FLOP of the 2 + 4 products and the bytes the
    flash path must move (Q, K, V, O forward; Q, K, V, dO read and dQ, dK,
    dV written backward)."""
    import torch

    from ml_engine_b200 import ops
    from ml_engine_b200._lib import kernels
    dev = torch.device("cuda", 0)
    hbm_peak, bf16_peak, kind = load_peaks()
    B = args.batch or 256
    H, S, D = 8, 256, 64
    g = torch.Generator(device=dev).manual_seed(0)
    Q, K, V, dO = (torch.randn(B, S, H * D, device=dev, generator=g) for _ in range(4))
    O = torch.empty(B, S, H * D, device=dev)
    dQ, dK, dV = (torch.empty(B, S, H * D, device=dev) for _ in range(3))
    stats = torch.empty(2 * B * H * S, device=dev)
    dvec = torch.empty(B * H * S, device=dev)
    P = torch.empty(B * H, S, S, device=dev)
    ws = torch.empty(B * H * S * S, device=dev)
    scale = 1.0 / 8.0
    old = ops.set_attention_path(ops.ATTN_PATH_TENSOR)

    def timed(fn):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    flop_f, flop_b = 2 * 2.0 * B * H * S * S * D, 4 * 2.0 * B * H * S * S * D
    bytes_f, bytes_b = 4.0 * 4 * B * S * H * D, 7 * 4.0 * B * S * H * D
    try:
        for causal in (1, 0):
            paths = {
                "keys": (lambda: ops.attention_fwd(Q, K, V, P, O, B, H, S, S, D, scale, causal, 1, 1),
                         lambda: kernels().call("mle_attention_bwd_assign", Q.data_ptr(), K.data_ptr(), V.data_ptr(),
                                                P.data_ptr(), dO.data_ptr(), dQ.data_ptr(), dK.data_ptr(),
                                                dV.data_ptr(), None, None, ws.data_ptr(), B, H, S, S, D, scale,
                                                causal, 1, 0, 1, 7, torch.cuda.current_stream().cuda_stream)),
                "flash": (lambda: ops.attention_flash_fwd(Q, K, V, O, stats, B, H, S, S, D, scale, causal, 1),
                          lambda: ops.attention_flash_bwd(Q, K, V, dO, stats, dQ, dK, dV, B, H, S, S, D, scale,
                                                          causal, 0, 1, 7, dvec)),
            }
            for name, (fwd, bwd) in paths.items():
                fwd()
                f_ms, b_ms = timed(fwd), timed(bwd)
                print(json.dumps({"attention": name, "batch": B, "heads": H, "seq": S, "head_dim": D,
                                  "causal": causal, "fwd_ms": f_ms, "bwd_ms": b_ms,
                                  "fwd_tflops": flop_f / (f_ms * 1e-3) / 1e12,
                                  "bwd_tflops": flop_b / (b_ms * 1e-3) / 1e12,
                                  "flash_bytes_fwd_gb": bytes_f / 1e9, "flash_bytes_bwd_gb": bytes_b / 1e9,
                                  "tf32_peak_tflops": bf16_peak / 2, "hbm_peak_gbs": hbm_peak,
                                  "peak_kind": kind}), flush=True)
    finally:
        ops.set_attention_path(old)


def run_sweep(args):
    """linear backward (dX = dY W^T, dW = X^T dY) at M=N=K = n,
    LayerNorm backward and LayerNorm + GELU backward over 65536 rows of
    width w, and the fused clip + AdamW over 256 tensors totalling 1e8 and
    1e9 parameters.  One JSON line per case with achieved FLOP/s or bytes/s
    against the measured peaks (CUDA events around `reps` launches, after
    warm-up; inputs larger than L2 except the two smallest GEMMs)."""
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

    legs = set(args.sweep_only.split(",")) if args.sweep_only else {"linear", "colsum", "layernorm", "optimizer"}
    for n in ((512, 1024, 2048, 4096, 8192) if "linear" in legs else ()):
        X = torch.randn(n, n, device=dev, generator=g)
        W = torch.randn(n, n, device=dev, generator=g)
        dY = torch.randn(n, n, device=dev, generator=g)
        dX, dW = torch.zeros(n, n, device=dev), torch.zeros(n, n, device=dev)
        ms = timed(lambda: ops.linear_bwd(X, W, dY, dX, dW, None, n, n, n), 20 if n >= 4096 else 100)
        tf = 4.0 * n ** 3 / (ms * 1e-3) / 1e12
        print(json.dumps({"sweep": "linear_bwd", "n": n, "ms": ms, "tflops": tf, "frac_of_tf32": tf / tf32_peak,
                          "frac_of_bf16": tf / bf16_peak, "peak_kind": kind}), flush=True)
        if n >= 2048:
            # with the bias gradient: summed by the dW product's epilogue warps
            # (or a separate column-sum launch under --gemm-column-sums 0)
            dB = torch.zeros(n, device=dev)
            ms_b = timed(lambda: ops.linear_bwd(X, W, dY, dX, dW, dB, n, n, n), 20 if n >= 4096 else 100)
            print(json.dumps({"sweep": "linear_bwd_bias", "n": n, "ms": ms_b, "ms_without_bias": ms,
                              "bias_cost_us": 1e3 * (ms_b - ms), "peak_kind": kind}), flush=True)
            del dB
        del X, W, dY, dX, dW
    rows = 65536
    # bias gradient (column sums) and the GELU backward fused with it, at
    # configs[2]'s token count: 4 B/elem read, and 12 B/elem (x, dy read; dx written)
    for w in ((512, 2048) if "colsum" in legs else ()):
        dy = torch.randn(rows * w, device=dev, generator=g)
        db = torch.zeros(w, device=dev)
        ms = timed(lambda: ops.bias_grad(dy, db), 20)
        gbs = 4.0 * rows * w / (ms * 1e-3) / 1e9
        print(json.dumps({"sweep": "bias_grad", "rows": rows, "width": w, "ms": ms, "gbs": gbs,
                          "frac_of_hbm": gbs / hbm_peak, "peak_kind": kind}), flush=True)
        x = torch.randn(rows * w, device=dev, generator=g)
        dx = torch.empty_like(x)
        ms = timed(lambda: ops.act_bwd(ops.GELU, x, dy, dx, bias_grad=db, assign=True), 20)
        gbs = 12.0 * rows * w / (ms * 1e-3) / 1e9
        print(json.dumps({"sweep": "gelu_bwd_bias_grad", "rows": rows, "width": w, "ms": ms, "gbs": gbs,
                          "frac_of_hbm": gbs / hbm_peak, "peak_kind": kind}), flush=True)
        del dy, db, x, dx
    for w in ((1024, 2048, 4096, 8192) if "layernorm" in legs else ()):
        x = torch.randn(rows * w, device=dev, generator=g)
        y, mean, sq = torch.empty_like(x), torch.empty(rows, device=dev), torch.empty(rows, device=dev)
        ops.layernorm_fwd(x, y, mean, sq, rows, 1, 1, w)
        gy, gx = torch.randn_like(x), torch.zeros_like(x)
        ms = timed(lambda: ops.layernorm_bwd(y, gy, sq, gx, rows, 1, 1, w), 20)
        gbs = 16.0 * rows * w / (ms * 1e-3) / 1e9   # y, gy, gx read; gx written
        print(json.dumps({"sweep": "layernorm_bwd", "rows": rows, "width": w, "ms": ms, "gbs": gbs,
                          "frac_of_hbm": gbs / hbm_peak, "peak_kind": kind}), flush=True)
        # LayerNorm + GELU backward: GELU(LN(x)) with the GELU backward
        # writing the LayerNorm output's gradient (assign), then the
        # LayerNorm backward: 12 + 16 B/elem
        a = torch.empty_like(x)
        ops.act_fwd(ops.GELU, y, a)
        gh = torch.empty_like(x)

        def ln_gelu():
            ops.act_bwd(ops.GELU, y, gy, gh, assign=True)
            ops.layernorm_bwd(y, gh, sq, gx, rows, 1, 1, w)
        ms = timed(ln_gelu, 20)
        gbs = 28.0 * rows * w / (ms * 1e-3) / 1e9
        print(json.dumps({"sweep": "layernorm_gelu_bwd", "rows": rows, "width": w, "ms": ms, "gbs": gbs,
                          "frac_of_hbm": gbs / hbm_peak, "peak_kind": kind}), flush=True)
        del x, y, gy, gx, a, gh
    totals = [int(float(x)) for x in args.sweep_optimizer_params.split(",")] if "optimizer" in legs else []
    for total in totals:
        nt = 256
        sizes = np.random.default_rng(0).integers(1, 1000, nt).astype(np.float64)
        sizes = np.maximum(1, (sizes / sizes.sum() * total).astype(np.int64))
        params = []
        for sz in sizes:
            params.append(dict(w=torch.empty(int(sz), device=dev).normal_(0, 0.02, generator=g),
                               g=torch.empty(int(sz), device=dev).normal_(0, 1e-2, generator=g),
                               m=torch.zeros(int(sz), device=dev), v=torch.zeros(int(sz), device=dev),
                               t=torch.ones(1, dtype=torch.int32, device=dev)))
        ws = torch.zeros(1, dtype=torch.float64, device=dev)
        views = ops.param_views(params)   # built once, as the engine's optimizer does

        def clip_adam():
            ws.zero_()
            ops.grad_sumsq(views, ws)
            ops.clip_finalize(ws, 1.0)
            ops.adam_update(views, lr=1e-3, adamw=True, clip_ws=ws, write_back_grad=False)
        ms = timed(clip_adam, 10 if total <= 100_000_000 else 3)
        nparam = int(sizes.sum())
        gbs = 32.0 * nparam / (ms * 1e-3) / 1e9   # g read (norm); w, g, m, v read; w, m, v written
        print(json.dumps({"sweep": "clip_adamw", "params": nparam, "tensors": nt, "ms": ms, "gbs": gbs,
                          "frac_of_hbm": gbs / hbm_peak, "peak_kind": kind}), flush=True)
        fws = ops.clip_adam_workspace(views)   # the one-launch form the engine takes by default
        ms = timed(lambda: ops.clip_adam(fws, lr=1e-3, max_norm=1.0, adamw=True, write_back_grad=False),
                   10 if total <= 100_000_000 else 3)
        gbs = 32.0 * nparam / (ms * 1e-3) / 1e9
        print(json.dumps({"sweep": "clip_adamw_one_launch", "params": nparam, "tensors": nt, "ms": ms, "gbs": gbs,
                          "frac_of_hbm": gbs / hbm_peak, "peak_kind": kind}), flush=True)
        del params, views, fws
        torch.cuda.empty_cache()


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
        pool.append({"x_t": (np.sqrt(abar) * x0 + np.sqrt(1 - abar) * eps).astype(np.float32), "noise": eps})
    stream = torch.cuda.ExternalStream(s.stream, device=dev)
    feed(s, pool[0])
    s.step()
    s.capture()
    for i in range(max(args.warmup, 3)):
        feed(s, pool[i % 4])
        s.step()
    torch.cuda.synchronize()
    ms = time_replays(s, stream, args.steps)
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    loss = None
    for i in range(args.steps):
        feed(s, pool[i % 4])
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


# ------------------------------------------------------------ native arm
def run_native(args, rank, world, local_rank):
    import torch

    from ml_engine_b200.session import Session

    wl = args.config
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    hbm_peak, bf16_peak, peak_kind = load_peaks()
    tf32_peak = bf16_peak / 2
    B = local_batch(wl, world)
    s = make_session(wl, B, seed=2024)
    if world > 1:
        import torch.distributed as dist
        uid = [Session.dp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        s.enable_dp(uid[0], rank, world, bucket_mb=args.bucket_mb)
    stream = torch.cuda.ExternalStream(s.stream, device=dev)
    pool = input_pool(wl, B, seed=3000 + rank)

    feed(s, pool[0])
    s.step()                 # eager step: builds tensor maps, configures kernels
    s.capture()
    for i in range(max(args.warmup, 3)):
        feed(s, pool[i % len(pool)])
        s.step()
    kk, mm, cc = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    s._lib.call("mle_session_graph_counts", s._h, ctypes.addressof(kk), ctypes.addressof(mm), ctypes.addressof(cc))
    kernels, memsets, copies = kk.value, mm.value, cc.value

    with ClockSampler(smi_index(local_rank)) as clocks:
        # ---------------------------------------------------------- value
        barrier(world)
        torch.cuda.synchronize()
        dev_ms = max_over_ranks(time_replays(s, stream, args.steps), world, dev)
        # ------------------------------------------------------------ e2e
        barrier(world)
        torch.cuda.synchronize()
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        losses = []
        for i in range(args.steps):
            feed(s, pool[(args.warmup + i) % len(pool)])
            losses.append(s.step(upload=True, read_loss=True))
        e3.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        e2e_ms = max_over_ranks(e2.elapsed_time(e3) / args.steps, world, dev)
    clk = clocks.summary()

    # ------------------------------------------------- backward vs roofline
    s.capture_phases()
    barrier(world)
    f_ms, b_ms, o_ms = time_phases(s, stream, max(3, min(args.steps, 10)))
    b_ms = max_over_ranks(b_ms, world, dev)
    bflop, bbytes = backward_work(wl, B)
    t_roof = bflop / (tf32_peak * 1e12) * 1e3 + bbytes / (hbm_peak * 1e9) * 1e3
    bwd = {"ms": b_ms, "forward_ms": f_ms, "allreduce_clip_update_ms": o_ms, "algorithmic_tflop": bflop / 1e12,
           "algorithmic_elementwise_gb": bbytes / 1e9, "achieved_tflops": bflop / (b_ms * 1e-3) / 1e12,
           "roofline_ms": t_roof, "frac": t_roof / b_ms,
           "tensor_frac_of_tf32": bflop / (b_ms * 1e-3) / 1e12 / tf32_peak,
           "how": "backward phase replayed alone (its own captured graph, CUDA events; with N > 1 the graph "
                  "also holds the gradient all-reduce it starts); roofline time = "
                  "algorithmic tensor FLOP at TF32 dense (half the measured bf16 peak) + algorithmic "
                  "non-GEMM backward bytes at the measured HBM copy bandwidth"}
    s.close()   # the remaining legs allocate their own buffers
    torch.cuda.empty_cache()

    units, unit_name = units_per_step(wl, B)
    value = 1e3 / dev_ms
    line = {
        "metric": METRIC, "value": value, "unit": "steps/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms, "higher_is_better": True,
        "scaling": WORKLOADS[wl]["scaling"], "vs_baseline": None,
        "dtype": "f32 (tf32 tensor-core products, fp32 accumulation)", "data": "synthetic (seeded)",
        unit_name.replace("/", "_per_"): value * units * world,
        "config": config_dict(wl, world),
        "e2e": {"value": 1e3 / e2e_ms, "unit": "steps/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": int(sum(v.nbytes for v in pool[0].values())), "d2h_bytes_per_step": 4,
                "loss_last": losses[-1] if losses else None},
        "bwd_roofline": bwd,
        "gpu_launches": kernels * args.steps,
        "launches_per_step": {"kernels": kernels, "memsets": memsets, "copies": copies},
        "clocks": clk,
    }
    if rank == 0 and not args.no_roofline:
        rows, gflop, gms = roofline_gemms(wl, B, dev, torch.cuda.current_stream(dev))
        achieved = gflop / (gms * 1e-3) / 1e12
        traffic = traffic_alg = None
        prof = ROOT / "profiles" / "traffic.json"
        if prof.exists():
            tr = json.loads(prof.read_text()).get(wl)
            if tr:
                # captured for the profile's token count; every operand but
                # the weights grows with the tokens a rank processes
                scale = B * WORKLOADS[wl]["cfg"].get("seq_len", 1) / tr.get("tokens", 1)
                traffic = tr.get("bytes_per_launch") * scale
                traffic_alg = tr.get("algorithmic_bytes_per_launch") * scale
        line["roofline"] = {
            "bound": "tensor", "kernel": "gemm_tf32_kernel (tcgen05 kind::tf32, TMA, TMEM): every Linear backward "
                                         "product of the step (dX, dW) at the rank's token count",
            "achieved": achieved, "peak": bf16_peak, "unit": "TFLOP/s", "frac": achieved / bf16_peak,
            "peak_kind": f"{peak_kind} bf16 dense burst (tf32 dense is half of it)",
            "frac_of_tf32": achieved / tf32_peak, "traffic": traffic,
            "traffic_note": "DRAM bytes per launch from profiles/traffic.json (ncu capture at 1/8 of the tokens, "
                            "scaled); algorithmic bytes per launch: " + (f"{traffic_alg:.4g}" if traffic_alg else "n/a"),
            "per_shape": rows}
    if rank == 0 and world == 1 and not args.no_ref_cuda:
        line["ref_cuda"] = ref_cuda_leg(dev)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_leg(wl, B, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--config", default="encdec", choices=["encdec", "encoder", "mlp", "unet"],
                    help="encdec: configs[2], global batch 256 over the ranks (the benchmark line); encoder: "
                         "configs[1] per rank; mlp: configs[0] per rank; unet: configs[3] on one GPU")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-cuda", action="store_true")
    ap.add_argument("--no-roofline", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="configs[4] kernel sweep, one JSON line per case")
    ap.add_argument("--sweep-only", default=None,
                    help="comma list of sweep legs to run: linear, colsum, layernorm, optimizer (default: all)")
    ap.add_argument("--sweep-optimizer-params", default="1e8,1e9",
                    help="parameter totals of the optimizer legs (comma list)")
    ap.add_argument("--attention", action="store_true",
                    help="configs[2]'s attention block on both tensor-core paths, one JSON line per case")
    ap.add_argument("--gemm-pairs", type=int, default=None, choices=[0, 1, 2],
                    help="run large products on CTA pairs (mle_set_gemm_pairs); default: the library's")
    ap.add_argument("--attn-path", default=None, choices=["auto", "fused", "tensor"],
                    help="attention implementation (mle_set_attention_path); default: the library's")
    ap.add_argument("--param-stream", type=int, default=None, choices=[0, 1],
                    help="weight/bias gradients on a second stream (mle_set_param_grad_stream); default: on")
    ap.add_argument("--gemm-store-path", type=int, default=None, choices=[0, 1],
                    help="assigned GEMM outputs through TMA bulk stores (0) or warp stores (1; the library default)")
    ap.add_argument("--fused-optimizer", type=int, default=None, choices=[0, 1],
                    help="norm, clip and AdamW as one cooperative launch (1, the library default) or as the "
                         "sum-of-squares, finalize and update launches (0) (mle_set_fused_optimizer)")
    ap.add_argument("--attn-flash", type=int, default=None, choices=[0, 1],
                    help="flash attention kernels where they apply (1, the library default) or the keys-on-lanes "
                         "path (0) (mle_set_attention_flash)")
    ap.add_argument("--add-norm-fusion", type=int, default=None, choices=[0, 1],
                    help="forward residual Add + LayerNorm as one pass (1, the library default) or two launches (0) "
                         "(mle_set_add_norm_fusion)")
    ap.add_argument("--gemm-column-sums", type=int, default=None, choices=[0, 1],
                    help="Linear bias gradients from the dW product's epilogue (1, the library default) or a "
                         "separate column-sum launch (0) (mle_set_gemm_column_sums)")
    ap.add_argument("--bucket-mb", type=int, default=0,
                    help="data-parallel gradient bucket size in MiB (mle_session_enable_dp); 0: the library's "
                         "choice from the gradient total (mle_dp_auto_bucket_mb)")
    ap.add_argument("--roofline-only", action="store_true",
                    help="run only the roofline GEMM pairs of --config (2 untimed + --roofline-reps timed pairs "
                         "per shape)")
    ap.add_argument("--roofline-batch", type=int, default=None,
                    help="sequences for --roofline-only (default: the workload's per-rank batch at one GPU)")
    ap.add_argument("--roofline-reps", type=int, default=5)
    ap.add_argument("--batch", type=int, default=None,
                    help="profiling aid: this many sequences per rank instead of the workload's (the JSON line is "
                         "then not the benchmark's)")
    args = ap.parse_args()
    if args.batch:
        global BATCH_OVERRIDE
        BATCH_OVERRIDE = args.batch
    if args.gemm_pairs is not None:
        from ml_engine_b200._lib import kernels
        kernels().call("mle_set_gemm_pairs", args.gemm_pairs)
    if args.attn_path is not None:
        from ml_engine_b200._lib import kernels
        kernels().call("mle_set_attention_path", {"auto": 0, "fused": 1, "tensor": 2}[args.attn_path])
    if args.gemm_store_path is not None:
        from ml_engine_b200._lib import kernels
        kernels().call("mle_set_gemm_store_path", args.gemm_store_path)
    if args.param_stream is not None:
        from ml_engine_b200._lib import engine
        engine().call("mle_set_param_grad_stream", args.param_stream)
    if args.attn_flash is not None:
        from ml_engine_b200._lib import kernels
        kernels().call("mle_set_attention_flash", args.attn_flash)
    if args.add_norm_fusion is not None:
        from ml_engine_b200._lib import engine
        engine().call("mle_set_add_norm_fusion", args.add_norm_fusion)
    if args.gemm_column_sums is not None:
        from ml_engine_b200._lib import kernels
        kernels().call("mle_set_gemm_column_sums", args.gemm_column_sums)
    if args.fused_optimizer is not None:
        from ml_engine_b200._lib import engine
        engine().call("mle_set_fused_optimizer", args.fused_optimizer)
    if args.sweep:
        run_sweep(args)
        return
    if args.attention:
        run_attention(args)
        return
    if args.config == "unet":
        run_unet(args)
        return
    if args.roofline_only:
        roofline_only(args)
        return
    world, rank, local_rank = init_ranks()
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_native(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
