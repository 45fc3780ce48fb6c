#!/usr/bin/env python3
"""Benchmark of the policy-sampling hot path on B200.

Workload: bimanual Diffusion Policy ConditionalUnet1D
(action 14, horizon 64, condition 284, dims 512/1024/2048, kernel 5, 8 groups,
step embedding 128), bf16 weights / fp32 accumulation, 10-step DDIM (eta 0),
global batch 4096 sharded over the ranks (strong scaling), seeded synthetic
inputs and PyTorch-default random-init weights (no datasets or checkpoints are
reachable).  One step = one complete DDIM-10 sample of the rank's shard.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Rank 0 prints one JSON line.  `value` is device-timed (CUDA events on the
launching stream, inputs resident in HBM, max over ranks); `e2e` is the same
metric through the host-buffer C ABI (host->device inputs and device->host
actions inside the timed region).  `--impl reference` times the reference's own
CPU core (oracle/_ref) on the host cores on a bounded sample of the workload.

After the timed region the engine's device error word is read (a bounded
device wait that timed out fails the run), and the actions of the last timed
step are checked against the reference core on sampled rows of every rank's
shard (`parity_max_abs`; the run exits non-zero above the bf16 bar 2e-2).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

from flowedge_b200 import checkpoint as ck  # noqa: E402
from flowedge_b200.shard import gather_rows, max_over_ranks, shard_range, shard_seed  # noqa: E402

METRIC = "DDIM action chunks/s at b=4096 (bimanual U-Net, 10-step DDIM)"
UNIT = "chunks/s"
GLOBAL_BATCH = int(os.environ.get("FLOWEDGE_BENCH_BATCH", "4096"))
STEPS = 10
SEED = 0
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of the 36 conv
# GEMM launches of one denoising forward, per shard size, from one ncu capture
# of this script's first forward:
#   FLOWEDGE_BENCH_BATCH=<shard> ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,dram__bytes_write.sum
#       --clock-control none -k regex:tc_gemm -c 80 --csv --log-file traffic.csv
#       python bench.py --steps 1 --warmup 1 --no-cpu-baseline --no-extras --no-parity
# (launches 1-36 after the FiLM-condition GEMM).  Other shard sizes report null.
CONV_TRAFFIC_PER_FORWARD = {4096: 32.39e9, 1024: 7.22e9}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _checkpoint(path: Path, spec, bf16_round: bool):
    """Seeded random-init U-Net; with bf16_round the 2-D/3-D weights are
    rounded to bf16 and stored as fp32, so the bf16 engine and the fp32
    reference core run identical weights."""
    if path.exists():
        return path
    tensors, meta = ck.diffusion_tensors(spec, seed=SEED)
    if bf16_round:
        tensors = {k: (ck.bf16_bits_to_f32(ck.to_bf16_bits(v)) if v.ndim >= 2 else v) for k, v in tensors.items()}
    tmp = path.with_suffix(f".tmp{os.getpid()}")
    ck.write_checkpoint(tmp, tensors, metadata=meta)
    os.replace(tmp, path)
    return path


def _inputs(spec, batch, offset=0):
    rng = np.random.default_rng(SEED + 1)
    cond = rng.standard_normal((GLOBAL_BATCH, spec.condition_dim), dtype=np.float32)
    noise = rng.standard_normal((GLOBAL_BATCH, spec.horizon, spec.action_dim), dtype=np.float32)
    return (np.ascontiguousarray(cond[offset:offset + batch]),
            np.ascontiguousarray(noise[offset:offset + batch]))


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def _peaks():
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return data.get("bf16_tflops_sustained", data.get("bf16_tflops")), "measured (sustained bf16)"
    return 1590.0, "fallback"


# ---------------------------------------------------------------------------
# CPU: the reference core on the host cores


class ReferencePool:
    """The reference core on the host cores: `threads` engines sharing one
    weight store (`fe_weights_load` + `fe_engine_create_from_weights`, one
    worker thread = the caller each), the throughput form of the CPU baseline
    (one engine per host thread)."""

    def __init__(self, path: Path, threads: int):
        from oracle import reference

        self.lib = reference.lib()
        self.weights = self.lib.fe_weights_load(str(path).encode())
        if not self.weights:
            raise RuntimeError(self.lib.fe_engine_last_error().decode())
        self.threads = threads
        self.engines = [reference.ReferenceEngine.from_weights(self.weights, 0) for _ in range(threads)]

    def sample(self, cond, noise):
        """DDIM-10 actions of every row (rows spread round-robin over the
        engines); returns (actions, seconds)."""
        out = np.empty_like(noise)

        def work(i):
            e = self.engines[i]
            for j in range(i, cond.shape[0], self.threads):
                out[j] = e.sample_diffusion(cond[j], noise[j], STEPS)

        t0 = time.perf_counter()
        pool = [threading.Thread(target=work, args=(i,)) for i in range(min(self.threads, cond.shape[0]))]
        for t in pool:
            t.start()
        for t in pool:
            t.join()
        return out, time.perf_counter() - t0

    def close(self):
        for e in self.engines:
            e.close()
        self.lib.fe_weights_free(self.weights)


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _reference_leg(path: Path, spec, steps: int, warmup: int):
    """The C4 reference measurement shared by `--impl reference` and the
    in-line `cpu_baseline`: one step = one DDIM-10 chunk per host thread (rows
    0..threads-1 of the global batch), after `warmup` untimed steps of the same
    size.  Returns (chunks/s, per-step seconds, threads, the rows' actions)."""
    threads = os.cpu_count() or 1
    cond, noise = _inputs(spec, threads)
    pool = ReferencePool(path, threads)
    for _ in range(warmup):
        pool.sample(cond, noise)
    times, actions = [], None
    for _ in range(steps):
        actions, secs = pool.sample(cond, noise)
        times.append(secs)
    pool.close()
    return threads * steps / sum(times), times, threads, actions


def _reference_rows(path: Path, spec, rows) -> np.ndarray:
    """Reference-core DDIM-10 actions of the given global rows (parity check)."""
    cond, noise = _inputs(spec, GLOBAL_BATCH)
    pool = ReferencePool(path, min(len(rows), os.cpu_count() or 1))
    out, _ = pool.sample(cond[list(rows)], noise[list(rows)])
    pool.close()
    return out


def run_reference(args):
    world, rank, _ = _dist()
    if rank != 0:
        return 0
    spec = ck.BIMANUAL
    path = _checkpoint(Path(args.workdir) / "bench_c4_bf16w.safetensors", spec, True)
    value, times, threads, _ = _reference_leg(path, spec, args.steps, args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000 * sum(times) / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "C4 bimanual U-Net DDIM-10 (reference fp32 CPU core on the bf16-rounded weights)",
                   "global_batch": GLOBAL_BATCH, "horizon": spec.horizon, "action_dim": spec.action_dim},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                         "cpu_model": _cpu_model(),
                         "sample": f"{threads} chunks per step (rows 0..{threads - 1}), {threads} engines x 1 thread, "
                                   f"shared weights, {args.warmup} warm-up steps of the same size"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _latency_cpu(fn, iters: int, warmup: int = 2) -> dict:
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(iters):
        t0 = time.perf_counter()
        fn()
        times.append((time.perf_counter() - t0) * 1000.0)
    times.sort()
    return {"p50_ms": times[len(times) // 2], "p99_ms": times[min(len(times) - 1, int(len(times) * 0.99))],
            "iters": iters}


def _cpu_latency_legs(workdir: Path) -> dict:
    """Batch-1 latency of the other workloads on the reference core, threads = 1
    (one engine, caller thread only) and all cores (one engine with
    min(nproc, 8) workers, the reference's maximum pool): PushT U-Net fp32
    DDIM-10, flow head Euler-10 / RK4-4 given the condition, Mamba 8 x 512
    prefill of 128 tokens, and Mamba -> flow Euler-10 (fe_engine_sample)."""
    from oracle import reference

    nproc = os.cpu_count() or 1
    rng = np.random.default_rng(7)
    cond = rng.standard_normal(132).astype(np.float32)
    noise = rng.standard_normal((16, 2)).astype(np.float32)
    c = rng.standard_normal(512).astype(np.float32)
    x0 = rng.standard_normal(350).astype(np.float32)
    tokens = np.arange(128, dtype=np.int32)
    pusht, flow, mamba = _latency_checkpoints(workdir)
    out = {}
    for label, threads in (("threads_1", 0), ("all_cores", min(nproc, 8))):
        e = reference.ReferenceEngine(pusht, threads=threads)
        # one fp32 DDIM-10 call takes about a second on one core: 10 timed calls there
        out.setdefault("c1_pusht_b1_ddim10_fp32", {})[label] = _latency_cpu(
            lambda: e.sample_diffusion(cond, noise, 10), 10 if threads == 0 else 20)
        e.close()
        e = reference.ReferenceEngine(flow, threads=threads)
        out.setdefault("c2_flow_b1_euler10_fp32", {})[label] = _latency_cpu(
            lambda: e.sample_condition(c, x0, 10, "euler"), 50)
        out.setdefault("c2_flow_b1_rk4_4_fp32", {})[label] = _latency_cpu(
            lambda: e.sample_condition(c, x0, 4, "rk4"), 50)
        e.close()
        e = reference.ReferenceEngine(mamba, threads=threads)
        out.setdefault("c3_mamba_b1_prefill128_fp32", {})[label] = _latency_cpu(lambda: e.run(tokens, 512), 20)
        out.setdefault("c3_mamba_flow_b1_sample_euler10_fp32", {})[label] = _latency_cpu(
            lambda: e.sample(tokens, x0, 10, "euler"), 20)
        e.close()
        for leg in out.values():
            leg[label]["workers"] = threads
    return out


def _latency_checkpoints(workdir: Path):
    workdir.mkdir(parents=True, exist_ok=True)
    pusht = _checkpoint(workdir / "bench_c1_pusht.safetensors", ck.PUSHT, False)
    flow = workdir / "bench_c2_flow.safetensors"
    if not flow.exists():
        ck.write_checkpoint(flow, ck.flow_tensors(ck.FLOW_C2, seed=SEED))
    mamba = workdir / "bench_c3_mamba_flow.safetensors"
    if not mamba.exists():
        t = ck.mamba_tensors(ck.MAMBA_C3, seed=SEED)
        t.update(ck.flow_tensors(ck.FLOW_C2, seed=SEED + 1))
        ck.write_checkpoint(mamba, t)
    return pusht, flow, mamba


# ---------------------------------------------------------------------------
# GPU


def run_ours(args):
    import torch

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        # bounded: a rank that fails leaves the others' next collective with an
        # error instead of a hang (rank 0's checkpoint write precedes the first)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=240),
                                device_id=torch.device("cuda", local))
    from flowedge_b200 import Engine
    from flowedge_b200.engine import device_malloc_count

    spec = ck.BIMANUAL
    workdir = Path(args.workdir)
    workdir.mkdir(parents=True, exist_ok=True)
    path = workdir / "bench_c4_bf16w.safetensors"
    if rank == 0:
        _checkpoint(path, spec, True)
    if dist is not None:
        dist.barrier()
    assert GLOBAL_BATCH % world == 0  # equal shards: the actions are all-gathered
    offset, shard = shard_range(GLOBAL_BATCH, world, rank)
    seed = shard_seed(SEED, offset)
    cond, noise = _inputs(spec, shard, offset=offset)
    engine = Engine(path, threads=0, device=local, precision="bf16", max_batch=shard)

    # a dedicated (non-default) stream: the engine enqueues on it and the
    # CUDA events are recorded on it
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    d_cond = torch.from_numpy(cond).cuda()
    d_noise = torch.from_numpy(noise).cuda()
    d_action = torch.empty((shard, spec.horizon, spec.action_dim), dtype=torch.float32, device="cuda")

    def step():
        engine.sample_diffusion_device(d_cond.data_ptr(), d_noise.data_ptr(), shard, d_action.data_ptr(), STEPS,
                                       "ddim", seed, stream.cuda_stream)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    mallocs0 = device_malloc_count()
    launches0 = engine.kernel_launches
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            step()
        stop.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(stop)
    launches = engine.kernel_launches - launches0
    # the device error word: a bounded device wait that timed out inside the
    # timed region fails the run here instead of yielding a throughput number
    engine.synchronize()
    if dist is not None:
        dist.barrier()
    ms_max = max_over_ranks(ms, dist, "cuda")
    value = GLOBAL_BATCH * args.steps / (ms_max / 1000.0)
    mallocs = device_malloc_count() - mallocs0

    # e2e through the host-buffer public API (inputs/outputs in host memory)
    out = np.empty_like(noise)
    engine.sample_diffusion_batch(cond, noise, STEPS, "ddim", seed)  # warm the host-API path
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e2e_steps = max(1, min(args.steps, 3))
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        out[:] = engine.sample_diffusion_batch(cond, noise, STEPS, "ddim", seed)
    e2e_s = time.perf_counter() - t0
    e2e_value = GLOBAL_BATCH * e2e_steps / max_over_ranks(e2e_s, dist, "cuda")

    # rows of the last timed step that are checked against the reference core:
    # rows 0..P-1 of the single shard, or the first two rows of every rank's shard
    n_par = 0 if args.no_parity else (min(os.cpu_count() or 1, shard) if world == 1 else min(2, shard))
    par_rows = [r * shard + i for r in range(world) for i in range(n_par)]
    par_got = d_action[:n_par].cpu().numpy() if world == 1 else None

    # results gathered to every rank after the timed region (timed separately)
    gather = None
    if dist is not None:
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        gather_rows(d_action, dist)  # untimed: the first gather sets up NCCL's channels
        dist.barrier()
        torch.cuda.synchronize()
        g0.record(stream)
        gathered = gather_rows(d_action, dist)
        g1.record(stream)
        torch.cuda.synchronize()
        gather = {"op": "all_gather of the actions", "bytes": int(gathered.numel() * 4),
                  "ms": max_over_ranks(g0.elapsed_time(g1), dist, "cuda")}
        if rank == 0 and par_rows:
            par_got = gathered.reshape(GLOBAL_BATCH, spec.horizon, spec.action_dim)[par_rows].cpu().numpy()
        del gathered

    # dominant kernel: the tcgen05 conv GEMMs of one denoise forward
    prof = engine.profile_diffusion(shard)
    peak, peak_kind = _peaks()
    achieved = prof["conv_flops"] / (prof["conv_ms"] / 1000.0) / 1e12
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "C4 bimanual U-Net (A14 H64 cond284, dims 512/1024/2048) DDIM-10, bf16 weights "
                                   "fp32 accumulate", "global_batch": GLOBAL_BATCH, "per_gpu_batch": shard,
                       "horizon": spec.horizon, "action_dim": spec.action_dim, "parallelism": f"batch shards x{world}",
                       "l2": "working set above L2 (each activation tensor 268 MB at b=4096, weights 0.5 GB)"},
            "clocks": clocks.summary(),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(cond.nbytes + noise.nbytes),
                    "d2h_bytes_per_step": int(out.nbytes)},
            "gpu_launches": int(launches),
            # conv FLOPs of the chunks processed per second by each GPU, over the measured peak
            "per_gpu_tensor_frac": value / world * STEPS * prof["conv_flops"] / shard / (peak * 1e12),
            "device_mallocs_in_timed_region": int(mallocs),
            "roofline": {"bound": "tensor", "kernel": "tc_gemm_kernel (conv GEMMs of one denoise)",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": CONV_TRAFFIC_PER_FORWARD.get(shard),
                         "traffic_unit": "DRAM bytes per forward (the 36 conv launches achieved is taken over), "
                                         "from an ncu capture at this shard size",
                         "conv_share_of_forward": prof["conv_ms"] / prof["forward_ms"],
                         "conv_launches_per_forward": prof["conv_launches"]},
        }
    if gather is not None and line is not None:
        line["gather"] = gather
    if world == 1 and not args.no_extras:
        line["extra"] = _extras(Path(args.workdir), local)
    expected = None
    if world == 1 and not args.no_cpu_baseline:
        # the same measurement as `--impl reference` (one warm-up step, three timed)
        cpu_value, times, threads, expected = _reference_leg(path, spec, 3, 1)
        line["cpu_baseline"] = {"value": cpu_value, "unit": UNIT, "cores": threads, "kind": "reference",
                                "nproc": os.cpu_count(), "cpu_model": _cpu_model(),
                                "sample": f"{threads} chunks per step (rows 0..{threads - 1}), {threads} engines x 1 "
                                          f"thread, 1 warm-up + 3 timed steps ({sum(times):.1f} s)"}
        value_t1 = _reference_single_thread(path, spec)
        line["cpu_baseline"]["threads_1"] = {"value": value_t1, "unit": UNIT, "cores": 1,
                                             "sample": "1 chunk (row 0), one engine, caller thread only"}
        if not args.no_extras:
            line["cpu_baseline"]["latency_b1"] = _cpu_latency_legs(Path(args.workdir))
            line["cpu_baseline"]["c5_smolvla"] = _smolvla_cpu_baseline(threads)
    parity_bad = False
    if rank == 0 and par_rows:
        if expected is None or expected.shape[0] < len(par_rows):
            expected = _reference_rows(path, spec, par_rows)
        err = float(np.abs(par_got - expected[:len(par_rows)]).max())
        parity_bad = not err <= 2e-2
        line["parity_max_abs"] = err
        line["parity"] = {"rows": len(par_rows), "bar": 2e-2, "against": "reference CPU core on the same "
                          "bf16-rounded weights (fp32)", "which": "first rows of every rank's shard, last timed step"}
    engine.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    if parity_bad:
        print(f"parity check failed: max-abs {line['parity_max_abs']:.3g} above 2e-2", file=sys.stderr)
        return 1
    return 0


def _reference_single_thread(path: Path, spec) -> float:
    """threads = 1: one reference engine, caller thread only, one chunk."""
    from oracle import reference

    cond, noise = _inputs(spec, 1)
    e = reference.ReferenceEngine(path, threads=0)
    t0 = time.perf_counter()
    e.sample_diffusion(cond[0], noise[0], STEPS)
    secs = time.perf_counter() - t0
    e.close()
    return 1.0 / secs


def _latency(fn, iters):
    import torch

    from flowedge_b200.engine import device_malloc_count

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    mallocs0 = device_malloc_count()
    times = []
    for _ in range(iters):
        t0 = time.perf_counter()
        fn()
        times.append((time.perf_counter() - t0) * 1000.0)
    times.sort()
    return {"p50_ms": times[len(times) // 2], "p99_ms": times[min(len(times) - 1, int(len(times) * 0.99))],
            "iters": iters, "device_mallocs": int(device_malloc_count() - mallocs0)}


def _smolvla_flops(spec) -> float:
    """Algorithmic FLOPs of one SmolVLA chunk through one Euler step
    (smolvla_action_expert.cc:209-394): every projection once, attention over
    the valid keys (cross: the prefix; self: causal over the action tokens)."""
    w, a, attn, kv, mlp, layers = (spec.expert_width, spec.action_dim, spec.attention_width, spec.kv_width,
                                   spec.mlp_width, spec.layers)
    cross = layers // 2
    self_layers = layers - cross
    per_token = 2 * (layers * (w * attn + attn * w + 3 * mlp * w) + self_layers * 2 * kv * w)
    per_token += 2 * (a * w + 2 * w * w + w * w) + 2 * w * a
    self_keys = spec.chunk + 1 + (spec.prefix if spec.cache_width == kv else 0) * 2
    per_token += 4 * attn * (cross * spec.prefix + self_layers * self_keys / 2)
    return float(per_token * spec.chunk)


def _extras(workdir: Path, device: int):
    """The other workloads (PushT U-Net, flow head, Mamba encoder, SmolVLA-shaped
    expert), through the public host-buffer API
    (synchronous calls: host->device inputs and device->host outputs included)."""
    import torch

    from flowedge_b200 import Engine

    out = {}
    rng = np.random.default_rng(7)
    # C1: PushT U-Net, batch 1, DDIM-10 (fp32 weights; and the bf16-weight mode)
    pusht, flow, mamba = _latency_checkpoints(workdir)
    cond = rng.standard_normal(132).astype(np.float32)
    noise = rng.standard_normal((16, 2)).astype(np.float32)
    for prec in ("fp32", "bf16"):
        e = Engine(pusht, threads=0, device=device, precision=prec)
        out[f"c1_pusht_b1_ddim10_{prec}"] = _latency(lambda: e.sample_diffusion(cond, noise, 10), 1000)
        e.close()
    # C2: flow head 350 / 1024 x 3 / 512, Euler-10 and RK4-4
    c = rng.standard_normal(512).astype(np.float32)
    x0 = rng.standard_normal(350).astype(np.float32)
    for prec in ("fp32", "bf16"):
        e = Engine(flow, threads=0, device=device, precision=prec, max_batch=4096)
        out[f"c2_flow_b1_euler10_{prec}"] = _latency(lambda: e.sample_condition(c, x0, steps=10, method="euler"), 200)
        out[f"c2_flow_b1_rk4_4_{prec}"] = _latency(lambda: e.sample_condition(c, x0, steps=4, method="rk4"), 200)
        cb = torch.from_numpy(rng.standard_normal((4096, 512)).astype(np.float32)).cuda()
        xb = torch.from_numpy(rng.standard_normal((4096, 350)).astype(np.float32)).cuda()
        ob = torch.empty_like(xb)
        st = torch.cuda.Stream()
        run = lambda: e.sample_condition_device(cb.data_ptr(), xb.data_ptr(), 4096, ob.data_ptr(), 10, "euler",
                                                st.cuda_stream)
        for _ in range(3):
            run()
        st.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(st)
        for _ in range(5):
            run()
        ev1.record(st)
        st.synchronize()
        out[f"c2_flow_b4096_euler10_{prec}_actions_per_s"] = 4096 * 5 / (ev0.elapsed_time(ev1) / 1000.0)
        e.close()
    # C3: Mamba 8 x 512 (L = 128) -> C2 flow head
    tokens = np.arange(128, dtype=np.int32)
    for prec in ("fp32", "bf16"):
        e = Engine(mamba, threads=0, device=device, precision=prec, max_batch=1024)
        out[f"c3_mamba_b1_prefill128_{prec}"] = _latency(lambda: e.run(tokens), 100)
        out[f"c3_mamba_flow_b1_sample_euler10_{prec}"] = _latency(lambda: e.sample(tokens, x0, 10, "euler"), 100)
        e.reset()
        out[f"c3_mamba_decode_token_{prec}"] = _latency(lambda: e.step(5), 500)
        tb = np.ascontiguousarray(np.tile(tokens, (1024, 1)))
        e.run_batch(tb[:2])
        t0 = time.perf_counter()
        e.run_batch(tb)
        # host API: every position's hidden state comes back (1024 x 128 x 512 fp32 = 268 MB)
        out[f"c3_mamba_b1024_prefill128_{prec}_seq_per_s"] = 1024 / (time.perf_counter() - t0)
        # device buffers, last hidden state only (what feeds the flow head), CUDA events
        dt_ = torch.from_numpy(tb).cuda()
        dl = torch.empty((1024, 512), dtype=torch.float32, device="cuda")
        st = torch.cuda.Stream()
        for _ in range(2):
            e.run_device(dt_.data_ptr(), 1024, 128, dl.data_ptr(), st.cuda_stream)
        st.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(st)
        for _ in range(3):
            e.run_device(dt_.data_ptr(), 1024, 128, dl.data_ptr(), st.cuda_stream)
        ev1.record(st)
        st.synchronize()
        out[f"c3_mamba_b1024_prefill128_{prec}_device_seq_per_s"] = 3 * 1024 / (ev0.elapsed_time(ev1) / 1000.0)
        e.close()
    # C5: SmolVLA-shaped action expert (bf16 by construction), Euler-10, one
    # fixed 241-slot prefix of width 960 shared by the batch
    spec = ck.SMOLVLA_C5
    sv = workdir / "bench_c5_smolvla.safetensors"
    if not sv.exists():
        ck.write_checkpoint(sv, ck.smolvla_tensors(spec, seed=SEED), matrices="bf16")
    keys, values, mask = ck.smolvla_prefix(spec, SEED + 1)
    noise1 = rng.standard_normal((spec.chunk, spec.action_dim)).astype(np.float32)
    e = Engine(sv, threads=0, device=device)
    out["c5_smolvla_b1_euler10_bf16"] = _latency(lambda: e.smolvla_sample(noise1, 10, keys, values, mask), 100)
    batch = 512
    nb = rng.standard_normal((batch, spec.chunk, spec.action_dim)).astype(np.float32)
    e.smolvla_reserve(batch, spec.chunk, spec.prefix, True)
    dn, dk, dv = (torch.from_numpy(x).cuda() for x in (nb, keys, values))
    dm = torch.from_numpy(mask).cuda()
    do = torch.empty_like(dn)
    st = torch.cuda.Stream()
    run = lambda: e.smolvla_sample_device(dn.data_ptr(), batch, spec.chunk, 10, dk.data_ptr(), dv.data_ptr(),
                                          dm.data_ptr(), spec.prefix, True, do.data_ptr(), st.cuda_stream)
    for _ in range(2):
        run()
    st.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(st)
    for _ in range(3):
        run()
    ev1.record(st)
    st.synchronize()
    sec = ev0.elapsed_time(ev1) / 1000.0 / 3
    e.smolvla_sample_batch(nb, 10, keys, values, mask, shared_prefix=True)
    t0 = time.perf_counter()
    e.smolvla_sample_batch(nb, 10, keys, values, mask, shared_prefix=True)
    e2e = time.perf_counter() - t0
    peak, peak_kind = _peaks()
    tflops = batch * 10 * _smolvla_flops(spec) / sec / 1e12
    out["c5_smolvla_b512_euler10_bf16"] = {
        "chunks_per_s": batch / sec, "e2e_chunks_per_s": batch / e2e, "ms_per_call": sec * 1000.0,
        "tflops": tflops, "frac_of_peak": tflops / peak, "peak_kind": peak_kind,
        "flops_per_chunk_step": _smolvla_flops(spec)}
    e.close()
    return out


def _smolvla_cpu_baseline(threads: int) -> dict:
    """The reference cannot load the SmolVLA-shaped expert's shapes (12 heads of
    60, a 960-wide prefix; smolvla_action_expert.cc:120-128), so its CPU figure is the numpy
    restatement of the same algorithm (oracle/restate.py) on the host cores."""
    from oracle import restate

    spec = ck.SMOLVLA_C5
    model = restate.SmolVLAExpert(ck.smolvla_tensors(spec, seed=SEED))
    keys, values, mask = ck.smolvla_prefix(spec, SEED + 1)
    noise = np.random.default_rng(SEED).standard_normal((spec.chunk, spec.action_dim)).astype(np.float32)
    t0 = time.perf_counter()
    model.sample(noise, 10, keys, values, mask)
    sec = time.perf_counter() - t0
    return {"value": 1.0 / sec, "unit": "chunks/s", "cores": threads, "kind": "port",
            "sample": "1 chunk, Euler-10, numpy restatement (BLAS threads = host cores)"}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workdir", default=os.environ.get("FLOWEDGE_BENCH_DIR", "/tmp/flowedge_bench"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the C1/C2/C3 latency and throughput extras")
    ap.add_argument("--no-parity", action="store_true", help="skip the check against the reference core")
    args = ap.parse_args()
    Path(args.workdir).mkdir(parents=True, exist_ok=True)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
