#!/usr/bin/env python
"""Benchmark of the fused DFC-AdamW step (param-updates/s and HBM GB/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N=1 (default) -- multi-tensor step on one GPU: the 62 FP32 tensors of
ResNet-18 (CIFAR: 3x3 stem, no max-pool, 10 classes; 11,173,962 params),
params N(0,0.02), grads N(0,1e-3), packed moments (bf16 high half + 16-bit
error-feedback residual) warmed for 10 steps, one fused launch per step
through DFCAdamW.step().
N>1 (under torchrun) -- ZeRO-1 sharded step over a flat 2^30-element FP32
parameter vector: bf16 compressed gradients with error feedback, reduction
of the bf16 gradients, fused packed step on the rank's 1/N shard, FP32
parameter broadcast (strong scaling: the vector is fixed, ranks split its
state).  --transport auto picks the measured fastest: one fused kernel over
NVLink peer memory up to 4 ranks, the same kernel through NVSwitch
multicast beyond; nccl (reduce-scatter + step + all-gather) on request.

Prints one JSON line on rank 0.  Timing: W untimed steps, then K steps
between barrier + synchronize, CUDA events on the launching stream, max over
ranks.  Inputs (313 MB per step at N=1, GBs per rank at N>1) are larger
than the 126 MB L2.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "param-updates/s and HBM GB/s (% of 8 TB/s) for fused step at 1/2/4/8 B200"
UNIT = "param-updates/s"
STEP_BYTES_PER_PARAM = 28  # p r+w 8, g r 4, m r+w 8, v r+w 8
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
BETAS = (0.9, 0.999)
LR, EPS, WD = 1e-3, 1e-8, 0.01


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU work budget of the cpu_baseline sample")
    ap.add_argument("--no-clocks", action="store_true",
                    help="skip the nvidia-smi clock sampler (profiling runs)")
    ap.add_argument("--no-replay", action="store_true",
                    help="skip the replay-record codec measurement")
    ap.add_argument("--replay-only", action="store_true",
                    help="measure only the replay-record codec (one GPU) and print its JSON")
    ap.add_argument("--replay-batch", type=int, default=65536,
                    help="records per codec launch")
    ap.add_argument("--kernels-only", action="store_true",
                    help="measure only the compression, gradient-statistics and sign-fiber "
                         "kernels (one GPU) over --elems elements and print their JSON")
    ap.add_argument("--elems", type=int, default=None,
                    help="--kernels-only: elements per buffer (default 2^30)")
    ap.add_argument("--no-sharded-1gpu", action="store_true",
                    help="N=1: skip the one-GPU run of the sharded compressed-gradient step")
    ap.add_argument("--no-host-overhead", action="store_true",
                    help="skip the host-overhead measurement (profiling runs)")
    ap.add_argument("--transport", choices=("auto", "peer", "nvls", "nccl"), default="auto",
                    help="N>1: fused kernel over NVLink peer memory, the same kernel over "
                         "NVSwitch multicast, NCCL collectives, or the measured fastest for N")
    ap.add_argument("--fused-ctas", type=int, default=None,
                    help="N>1 peer/nvls: CTAs per SM of the fused kernel (0: one per tile)")
    ap.add_argument("--bucket-elems", type=int, default=None,
                    help="N>1: elements per pipelined bucket (default: ShardedDFCAdamW's)")
    ap.add_argument("--overlap-buckets", action="store_true",
                    help="N>1 peer/nvls: fused kernels of neighbouring buckets on two streams")
    ap.add_argument("--fuse-compression", action=argparse.BooleanOptionalAction, default=None,
                    help="N>1 peer/nvls: compress bucket b+1 inside bucket b's fused kernel "
                         "(default: ShardedDFCAdamW's)")
    ap.add_argument("--overlap-barrier", action=argparse.BooleanOptionalAction, default=None,
                    help="with --fuse-compression: each bucket's kernel starts its compression "
                         "while the barrier before it waits (default: ShardedDFCAdamW's)")
    ap.add_argument("--side-priority", type=int, default=None,
                    help="N>1 peer/nvls: CUDA priority of the fused kernel's stream "
                         "(lower is higher; default: ShardedDFCAdamW's)")
    ap.add_argument("--compress-ctas", type=int, default=None,
                    help="N>1 peer/nvls: CTAs per SM of the compression beside it (0: 8)")
    return ap.parse_args()


# ----------------------------------------------------------------------------
# environment helpers
# ----------------------------------------------------------------------------
def measured_hbm_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(kernel: str):
    """DRAM bytes (read + written) per launch of ``kernel`` from one ncu
    capture, kept in profiles/traffic.json; None if absent."""
    path = os.path.join(REPO, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return float(json.load(f)[kernel]["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError, TypeError):
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons every 200 ms, in the background."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        self.samples = []
        self.error = None
        try:
            props = torch.cuda.get_device_properties(device)
            self.gpu_id = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        except AttributeError:
            self.gpu_id = str(device.index or 0)
        self.proc = None

    def start(self, wait_s: float = 5.0):
        """Start sampling; return once the first sample has arrived (or after
        wait_s), so that nvidia-smi's start-up lies outside a timed region."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_id}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError as e:
            self.error = str(e)
            return self
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        t0 = time.perf_counter()
        while not self.samples and time.perf_counter() - t0 < wait_s:
            time.sleep(0.02)
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 9:
                self.samples.append(parts)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=5)
        return self.summary()

    def summary(self):
        if self.error or not self.samples:
            return {"error": self.error or "no nvidia-smi samples"}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if s[5 + i].lower().startswith("active")})
        power = [float(s[3]) for s in self.samples if s[3].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples),
                "power_w_max": max(power) if power else None}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if n_gpus != world:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------
# workload
# ----------------------------------------------------------------------------
def resnet18_params(device, seed=0, align=64):
    """62 ResNet-18 parameters as views of one flat FP32 buffer (offsets
    aligned to 64 elements), N(0, 0.02)."""
    from t3st_b200.workloads import resnet18_cifar_shapes

    shapes = resnet18_cifar_shapes()
    sizes = [math.prod(s) for s in shapes]
    offs, o = [], 0
    for n in sizes:
        offs.append(o)
        o += (n + align - 1) // align * align
    gen = torch.Generator(device=device).manual_seed(seed)
    flat_p = torch.zeros(o, device=device)
    flat_g = torch.zeros(o, device=device)
    params = []
    for s, n, off in zip(shapes, sizes, offs):
        p = torch.nn.Parameter(flat_p[off:off + n].view(s))
        p.data.normal_(0.0, 0.02, generator=gen)
        p.grad = flat_g[off:off + n].view(s)
        params.append(p)
    return params, flat_p, flat_g, gen, sum(sizes)


def fill_grads(params, gen, std=1e-3):
    for p in params:
        p.grad.normal_(0.0, std, generator=gen)


# ----------------------------------------------------------------------------
# CPU baseline (reference algorithm as PyTorch CPU ops; oracle/torch_port.py)
# ----------------------------------------------------------------------------
def cpu_port_rate(shapes, seconds: float, packed: bool, max_params: int | None = None,
                  threads: int | None = None, fiber: bool = True):
    """Time the reference step restated as CPU torch ops on (a prefix of)
    the workload's tensors; returns (updates/s, description, threads).
    packed=False is the reference's own algorithm (remote/torch_fiber.py:
    68-117, FP32 moments, sign fiber on unless fiber=False)."""
    from oracle import torch_port

    torch.set_num_threads(threads or os.cpu_count() or 1)
    gen = torch.Generator().manual_seed(1)
    tensors = []
    total = 0
    for s in shapes:
        n = math.prod(s)
        if max_params is not None and tensors and total + n > max_params:
            break
        p = torch.randn(n, generator=gen) * 0.02
        g = torch.randn(n, generator=gen) * 1e-3
        m = torch.zeros(n, dtype=torch.int32 if packed else torch.float32)
        v = torch.zeros(n, dtype=torch.int32 if packed else torch.float32)
        tensors.append((p, g, m, v))
        total += n

    def one(step):
        for p, g, m, v in tensors:
            if packed:
                torch_port.step_packed(p, g, m, v, LR, BETAS, EPS, WD, step)
            else:
                torch_port.step_fp32(p, g, m, v, LR, BETAS, EPS, WD, step, fiber=fiber)

    one(1)
    t0 = time.perf_counter()
    steps = 0
    while True:
        steps += 1
        one(steps + 1)
        el = time.perf_counter() - t0
        if el >= seconds or (steps >= 3 and el * (steps + 1) / steps > 3 * seconds):
            break
    rate = total * steps / el
    fmt = "packed" if packed else ("fp32 sign-fiber" if fiber else "fp32 fiber-off")
    desc = (f"{len(tensors)} of {len(shapes)} ResNet-18 tensors ({total} params), {steps} "
            f"steps, {fmt} moments, {torch.get_num_threads()} threads")
    nthreads = torch.get_num_threads()
    torch.set_num_threads(os.cpu_count() or 1)
    return rate, desc, nthreads


def cpu_variants(shapes, seconds: float):
    """The reference CPU step in its other settings: fiber off, one thread,
    and the packed-word restatement (a format the reference lacks)."""
    out = []
    for packed, fiber, threads in ((False, False, None), (False, True, 1), (False, False, 1),
                                   (True, True, None)):
        rate, desc, nt = cpu_port_rate(shapes, seconds, packed=packed, threads=threads,
                                       fiber=fiber)
        out.append({"moment_format": "packed" if packed else "fp32", "enable_fiber": fiber,
                    "threads": nt, "value": rate, "unit": UNIT, "sample": desc})
    return out


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU path (remote/torch_fiber.py:
    68-117 restated op for op as torch CPU ops, bit-identical to it: FP32
    moments, sign fiber on, the reference's defaults) on the host cores,
    rank 0 only, K+W bounded steps.  The reference has no packed moment
    format; its FP32 path gives the same trajectory bit for bit.  At N=1 the
    sample is a prefix of the ResNet-18 tensors; at N>1 a prefix of the flat
    2^30-element ZeRO-1 vector (the reference has no distributed code: its
    step over the whole vector on one host is the comparison)."""
    if rank != 0:
        return
    from oracle import torch_port
    from t3st_b200.workloads import resnet18_cifar_shapes

    shapes = resnet18_cifar_shapes() if world == 1 else [(ZERO_PARAMS,)]
    torch.set_num_threads(os.cpu_count() or 1)
    total_params = sum(math.prod(s) for s in shapes)
    # calibrate on the ResNet-18 step, then bound the sample so the run takes <~2 min
    rate_full, _, _ = cpu_port_rate(resnet18_cifar_shapes(), 0.5, packed=False)
    budget = 120.0
    per_step = budget / max(1, args.steps + args.warmup)
    # and to at most 2^25 elements (512 MB of host state): the CPU rate per
    # element does not depend on the sample size
    max_params = max(4096, min(total_params, int(rate_full * per_step), 1 << 25))
    gen = torch.Generator().manual_seed(1)
    tensors, total = [], 0
    for s in shapes:
        n = math.prod(s)
        if tensors and total + n > max_params:
            break
        n = min(n, max_params)  # the flat vector: a prefix
        tensors.append((torch.randn(n, generator=gen) * 0.02, torch.randn(n, generator=gen) * 1e-3,
                        torch.zeros(n), torch.zeros(n)))
        total += n
    step = 0
    for _ in range(args.warmup):
        step += 1
        for p, g, m, v in tensors:
            torch_port.step_fp32(p, g, m, v, LR, BETAS, EPS, WD, step, fiber=True)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step += 1
        for p, g, m, v in tensors:
            torch_port.step_fp32(p, g, m, v, LR, BETAS, EPS, WD, step, fiber=True)
    el = time.perf_counter() - t0
    value = total * args.steps / el
    if world == 1:
        sample = (f"{len(tensors)} of {len(shapes)} ResNet-18 (CIFAR) tensors, {total} of "
                  f"{total_params} params per step, FP32 sign-fiber moments, torch CPU ops")
        workload = "resnet18-cifar multi-tensor DFC-AdamW step (reference CPU path)"
    else:
        sample = (f"first {total} of the {total_params} elements of the flat vector per step, "
                  f"FP32 sign-fiber moments, torch CPU ops")
        workload = ("flat 2^30-element FP32 vector DFC-AdamW step on one host "
                    "(reference CPU path; the reference has no distributed code)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": workload, "tensors": len(shapes), "params": total_params,
                   "moment_format": "fp32 sign-fiber (the reference's own format; it has no "
                                    "packed format, and both give the same trajectory)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample, "cpu_model": cpu_model()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# our arm, one GPU
# ----------------------------------------------------------------------------
LEAD_IN_STEPS = 3  # untimed steps queued ahead of the timed region


def run_single(args, device):
    from t3st_b200 import DFCAdamW
    from t3st_b200.workloads import resnet18_cifar_shapes

    # the clock sampler starts before any GPU work, so that nvidia-smi's
    # start-up is long over when the timed region begins
    sampler = None if args.no_clocks else ClockSampler(device).start()
    params, flat_p, flat_g, gen, n_params = resnet18_params(device)
    opt = DFCAdamW(params, lr=LR, betas=BETAS, eps=EPS, weight_decay=WD,
                   moment_format="packed")
    for _ in range(10):  # warm the packed moments with fresh gradients
        fill_grads(params, gen)
        opt.step()
    fill_grads(params, gen)
    for _ in range(max(3, args.warmup)):
        opt.step()
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream(device)
    K = args.steps
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t_wall = time.perf_counter()
    # e0 is queued behind a few untimed steps, so the timed region starts
    # with the GPU busy and the launch queue ahead of it (not with the host
    # latency of a first launch onto an idle stream)
    for _ in range(LEAD_IN_STEPS):
        opt.step()
    e0.record(stream)
    for _ in range(K):
        opt.step()
    e1.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t_wall
    clocks = {"skipped": "--no-clocks"}
    if sampler is not None:
        # keep the GPU busy with the same step while the clock sampler
        # collects enough samples (untimed)
        t_extra = time.perf_counter()
        while time.perf_counter() - t_extra < max(0.0, 1.5 - wall):
            for _ in range(200):
                opt.step()
            torch.cuda.synchronize()
        clocks = sampler.stop()

    total_ms = e0.elapsed_time(e1)
    kernel_ms = total_ms / K  # one launch per step, launched back to back
    value = n_params * K / (total_ms / 1e3)
    launches_per_step = 1  # 62 segments, 1 hyper set: one dfc_mt_step launch

    peak, peak_kind = measured_hbm_peak()
    algo_bytes = STEP_BYTES_PER_PARAM * n_params
    achieved = algo_bytes / (kernel_ms / 1e3) / 1e9
    traffic = profiled_traffic("dfc_step_resnet18")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": K,
        "warmup": args.warmup, "ms_per_step": total_ms / K, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {
            "workload": "resnet18-cifar multi-tensor DFC-AdamW step: 62 FP32 tensors, "
                        "11,173,962 params, packed moments (bf16 hi + 16-bit residual lo), "
                        "FP32 grads, one fused launch per step via DFCAdamW.step()",
            "tensors": len(params), "params": n_params, "moment_format": "packed",
            "algorithmic_bytes_per_param": STEP_BYTES_PER_PARAM,
            "l2": "inputs 313 MB per step > 126 MB L2 (no flush)",
            "parallelism": "single GPU",
            "timed_region": f"CUDA events on the launching stream; e0 queued behind "
                            f"{LEAD_IN_STEPS} untimed in-flight steps, then K steps, e1, "
                            f"synchronize",
        },
        "hbm_gbs": algo_bytes * K / (total_ms / 1e3) / 1e9,
        "hbm_pct_of_8tbs": 100.0 * algo_bytes * K / (total_ms / 1e3) / 1e9 / NOMINAL_HBM_GBS,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                     "traffic": traffic,
                     "kernel": "dfc::step_kernel<PACKED>, timed-region average per launch"},
        "gpu_launches": K * launches_per_step,
        "clocks": clocks,
        "host_wall_ms_per_step": wall / K * 1e3,
    }

    line["reference_default_format"] = run_fp32_format(args, device, peak)
    line["bf16_params"] = run_lowp_params(args, device, peak)
    if not args.no_sharded_1gpu:
        line["sharded_1gpu"] = run_sharded_1gpu(device, peak, peak_kind)
    if not args.no_host_overhead:
        line["host_us_per_step"] = host_overhead_us(opt)
    if not args.no_e2e:
        line["e2e"] = run_e2e(opt, params, flat_p, flat_g, gen, n_params, device, K)
    if not args.no_cpu_baseline:
        rate, desc, cores = cpu_port_rate(resnet18_cifar_shapes(), args.cpu_seconds, packed=False)
        line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
                                "sample": desc + " (the reference's own format and defaults)",
                                "cpu_model": cpu_model(),
                                "variants": cpu_variants(resnet18_cifar_shapes(),
                                                         args.cpu_seconds / 4)}
    if not args.no_replay:
        line["replay"] = run_replay(device, peak, peak_kind, n=args.replay_batch,
                                    cpu=not args.no_cpu_baseline)
    return line


REPLAY_BATCH = 65536                   # records per launch (805 MB of FP32 images)
REPLAY_ENCODE_BYTES = 3072 * 4 + 8 + 1552   # image + label + task in, record out
REPLAY_DECODE_BYTES = 1552 + 3072 * 4 + 12  # record in, image + label + task + status out


def run_replay(device, peak, peak_kind, n=REPLAY_BATCH, cpu=True, reps=10):
    """The replay-record codec (dfc_replay_encode / dfc_replay_decode) on a
    batch of 65,536 records, each launch timed with CUDA events on the
    launching stream; beside it the CPU codec (the oracle's restatement of
    the reference's per-record numpy + zlib codec, one thread)."""
    from oracle import replay as R
    from t3st_b200 import _lib

    g = torch.Generator(device=device).manual_seed(3)
    x = torch.rand((n, 3072), generator=g, device=device)
    y = torch.randint(0, 100, (n,), generator=g, device=device, dtype=torch.int32)
    t = torch.randint(0, 10, (n,), generator=g, device=device, dtype=torch.int32)
    rec = torch.empty((n, 1552), dtype=torch.uint8, device=device)
    out = torch.empty((n, 3072), device=device)
    meta = torch.empty((3, n), dtype=torch.int32, device=device)
    lib = _lib.lib()
    stream = torch.cuda.current_stream(device)

    def enc():
        _lib.check("dfc_replay_encode", lib.dfc_replay_encode(
            x.data_ptr(), 3072, y.data_ptr(), t.data_ptr(), n, rec.data_ptr(), 1552,
            stream.cuda_stream))

    def dec():
        _lib.check("dfc_replay_decode", lib.dfc_replay_decode(
            rec.data_ptr(), 1552, n, out.data_ptr(), meta[0].data_ptr(), meta[1].data_ptr(),
            meta[2].data_ptr(), stream.cuda_stream))

    res = {"batch_records": n, "launches_timed": 2 * reps,
           "l2": f"{n * 3072 * 4 / 1e6:.0f} MB of images per launch (L2 126 MB; no flush)"}
    for name, fn, nbytes in (("encode", enc, REPLAY_ENCODE_BYTES), ("decode", dec, REPLAY_DECODE_BYTES)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        sec = e0.elapsed_time(e1) / 1e3 / reps
        gbs = n * nbytes / sec / 1e9
        res[name] = {"records_per_s": n / sec, "us_per_launch": sec * 1e6,
                     "algorithmic_bytes_per_record": nbytes,
                     "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                                  "frac": gbs / peak, "peak_source": f"{peak_kind} hbm_gbs"}}
    if int(meta[2].abs().sum()) != 0:
        raise RuntimeError("replay bench: a record failed its CRC check")
    if cpu:
        xs, ys, ts = x[:2000].cpu().numpy(), y[:2000].cpu().numpy(), t[:2000].cpu().numpy()
        t0 = time.perf_counter()
        k = 0
        while k < len(xs) and (time.perf_counter() - t0 < 2.0 or k < 100):
            R.decode(R.encode(xs[k], int(ys[k]), int(ts[k])))
            k += 1
        el = time.perf_counter() - t0
        res["cpu_baseline"] = {"value": k / el, "unit": "records/s (encode + decode)", "cores": 1,
                               "kind": "port",
                               "sample": f"{k} records through the numpy + zlib codec"}
    return res


def run_lowp_params(args, device, peak, dtype=torch.bfloat16, K=300):
    """The same 62-tensor step with 16-bit parameters and gradients (the
    reference's bf16/fp16 parameter support, remote/torch_fiber.py:45, 83,
    114-116): packed moments stay FP32 words, so an update moves 22 bytes
    (p r+w 4, g 2, m r+w 8, v r+w 8).  Timed like the headline line."""
    from t3st_b200 import DFCAdamW
    from t3st_b200.workloads import resnet18_cifar_shapes

    gen = torch.Generator(device=device).manual_seed(2)
    shapes = resnet18_cifar_shapes()
    params = [torch.nn.Parameter(torch.empty(s, device=device).normal_(0.0, 0.02, generator=gen)
                                 .to(dtype)) for s in shapes]
    for p in params:
        p.grad = torch.empty(p.shape, device=device).normal_(0.0, 1e-3, generator=gen).to(dtype)
    n_params = sum(p.numel() for p in params)
    opt = DFCAdamW(params, lr=LR, betas=BETAS, eps=EPS, weight_decay=WD, moment_format="packed")
    for _ in range(10 + max(3, args.warmup)):
        opt.step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(LEAD_IN_STEPS):
        opt.step()
    e0.record(stream)
    for _ in range(K):
        opt.step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / K
    gbs = 22 * n_params / (ms / 1e3) / 1e9
    return {"param_dtype": str(dtype).replace("torch.", ""), "moment_format": "packed",
            "value": n_params / (ms / 1e3), "unit": UNIT, "ms_per_step": ms, "steps": K,
            "algorithmic_bytes_per_param": 22, "hbm_gbs": gbs, "frac_of_measured_hbm": gbs / peak,
            "kernel": "dfc::step_kernel<PACKED, bf16 grad, bf16 param>"}


def run_fp32_format(args, device, peak, K=300):
    """The same step in the reference's own moment format (FP32 words, sign
    fiber on: DFCAdamW's defaults), timed the same way."""
    from t3st_b200 import DFCAdamW

    params, _, _, gen, n_params = resnet18_params(device, seed=1)
    opt = DFCAdamW(params, lr=LR, betas=BETAS, eps=EPS, weight_decay=WD)
    for _ in range(10):
        fill_grads(params, gen)
        opt.step()
    fill_grads(params, gen)
    for _ in range(max(3, args.warmup)):
        opt.step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        opt.step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / K
    gbs = STEP_BYTES_PER_PARAM * n_params / (ms / 1e3) / 1e9
    return {"moment_format": "fp32", "enable_fiber": True, "value": n_params / (ms / 1e3),
            "unit": UNIT, "ms_per_step": ms, "steps": K, "hbm_gbs": gbs,
            "frac_of_measured_hbm": gbs / peak,
            "kernel": "dfc::step_kernel<SIGNFIBER> (6 CTAs/SM)"}


def run_fiber_kernels(words, device, peak, K):
    """Sign-fiber payload I/O (dfc_fiber_write / dfc_fiber_read, C ABI) over
    one range of second-moment words: bit 31 of each word is one payload
    bit.  A write reads and rewrites each word and reads the packed byte
    (8.125 B per bit); a read reads each word and writes the byte (4.125 B).
    CUDA events over K calls each; the payload must read back unchanged."""
    from t3st_b200 import _lib

    lib = _lib.lib()
    nbits = words.numel()
    nbytes = nbits // 8
    ranges = np.zeros(1, dtype=_lib.WORDRANGE_DTYPE)
    ranges[0] = (words.data_ptr(), nbits)
    payload = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device=device,
                            generator=torch.Generator(device=device).manual_seed(5))
    back = torch.empty_like(payload)
    stream = torch.cuda.current_stream(device)

    def write():
        _lib.check("dfc_fiber_write", lib.dfc_fiber_write(
            _lib.ptr(ranges), 1, 0, nbytes * 8, payload.data_ptr(), stream.cuda_stream))

    def read():
        _lib.check("dfc_fiber_read", lib.dfc_fiber_read(
            _lib.ptr(ranges), 1, 0, nbytes * 8, back.data_ptr(), stream.cuda_stream))

    write()
    read()
    torch.cuda.synchronize()
    if not torch.equal(back, payload):
        raise RuntimeError("fiber bench: payload did not read back")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out = {"bits": nbytes * 8, "calls": K}
    for name, fn, per_bit in (("write", write, 8.125), ("read", read, 4.125)):
        e0.record(stream)
        for _ in range(K):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / K
        gbs = nbytes * 8 * per_bit / (ms / 1e3) / 1e9
        out[name] = {"ms_per_call": ms, "bits_per_s": nbytes * 8 / (ms / 1e3),
                     "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                                  "frac": gbs / peak, "algorithmic_bytes_per_bit": per_bit}}
    return out


def run_sharded_1gpu(device, peak, peak_kind, K=30):
    """The N>1 workload on one GPU: ShardedDFCAdamW over the flat 2^30-element
    vector with bf16 error-feedback compression (no collective at one rank):
    compression over P, then the packed step reading the bf16 gradients.
    The one-GPU point of the sharded compressed-gradient step's 1..8 series."""
    from t3st_b200.zero import ShardedDFCAdamW

    P = ZERO_PARAMS
    gen = torch.Generator(device=device).manual_seed(1234)
    param = torch.nn.Parameter(torch.empty(P, device=device).normal_(0.0, 0.02, generator=gen))
    opt = ShardedDFCAdamW([param], lr=LR, betas=BETAS, eps=EPS, weight_decay=WD,
                          moment_format="packed", compress_grads=True)
    del param
    opt.flat_grad[:P].normal_(0.0, 1e-3, generator=gen)
    for _ in range(3):
        opt.step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        opt.step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / K
    hbm_bytes = 12 * P + 26 * P  # compression over P, step over P with bf16 gradients
    gbs = hbm_bytes / (ms / 1e3) / 1e9
    launches = 2 * opt.n_buckets
    del opt
    torch.cuda.empty_cache()
    out = {"workload": "ShardedDFCAdamW at one rank over the flat 2^30-element FP32 vector: "
                       "bf16 error-feedback compression + packed step (bf16 gradients)",
           "params": P, "steps": K, "ms_per_step": ms, "value": P / (ms / 1e3), "unit": UNIT,
           "gpu_launches_per_step": launches,
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                        "frac": gbs / peak, "peak_source": f"{peak_kind} hbm_gbs",
                        "algorithmic_bytes_per_param": 38}}
    out.update(run_kernels(device, peak, P))
    torch.cuda.empty_cache()
    return out


def run_kernels(device, peak, P, K=10):
    """The kernels beside the step, each over P elements on its own buffers
    (inputs larger than L2 from 2^26 elements on), K launches between CUDA
    events: the error-feedback compression (12 B/elem), the gradient
    statistics (4 B/elem read, two passes) and the sign-fiber payload write
    and read through the C ABI."""
    from t3st_b200 import kernels

    gen = torch.Generator(device=device).manual_seed(4321)
    g = torch.empty(P, device=device).normal_(0.0, 1e-3, generator=gen)
    comp = torch.zeros(P, dtype=torch.int16, device=device)
    resid = torch.zeros(P, dtype=torch.int16, device=device)
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        kernels.compress_ef(g, comp, resid)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(K):
        kernels.compress_ef(g, comp, resid)
    e1.record(stream)
    torch.cuda.synchronize()
    c_ms = e0.elapsed_time(e1) / K
    c_gbs = 12 * P / (c_ms / 1e3) / 1e9
    del comp, resid
    # per-buffer gradient statistics (sum of squares, max, non-finite count)
    # over the FP32 gradient: 4 B/elem read, two passes (tiles, then records)
    kernels.grad_stats([g])
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(K):
        kernels.grad_stats([g])
    e1.record(stream)
    torch.cuda.synchronize()
    s_ms = e0.elapsed_time(e1) / K
    s_gbs = 4 * P / (s_ms / 1e3) / 1e9
    # second-moment words for the fiber: the gradient buffer's bits will do
    fiber = run_fiber_kernels(g, device, peak, K)
    del g
    torch.cuda.empty_cache()
    return {"compress_kernel": {"ms_per_launch": c_ms, "elements": P, "launches": K,
                                "roofline": {"bound": "hbm", "achieved": c_gbs, "peak": peak,
                                             "unit": "GB/s", "frac": c_gbs / peak,
                                             "algorithmic_bytes_per_elem": 12}},
            "grad_stats_kernels": {"ms_per_call": s_ms, "elements": P, "calls": K,
                                   "roofline": {"bound": "hbm", "achieved": s_gbs, "peak": peak,
                                                "unit": "GB/s", "frac": s_gbs / peak,
                                                "algorithmic_bytes_per_elem": 4}},
            "fiber_kernels": fiber}


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_e2e(opt, params, flat_p, flat_g, gen, n_params, device, K):
    """Same step through the public API with every step's gradients copied in
    from pinned host memory and its updated params copied back out, both
    PCIe directions kept busy:

      - gradients alternate between two device buffers (each parameter's
        .grad is re-pointed every step, as backward re-creates gradients; the
        step follows new gradient tensors), so the upload of step t+1's
        gradients runs while step t computes;
      - step t's parameters are copied on the device into one of two staging
        buffers right after the step, and go to the host from there, so step
        t+1 never waits for a download.

    Every step uploads 4 B and downloads 4 B per parameter."""
    host_g = torch.empty(flat_g.numel(), dtype=torch.float32, pin_memory=True)
    host_p = torch.empty(flat_p.numel(), dtype=torch.float32, pin_memory=True)
    host_g.copy_(flat_g.cpu())
    main = torch.cuda.current_stream(device)
    h2d = torch.cuda.Stream(device)
    d2h = torch.cuda.Stream(device)
    gbuf = [flat_g, torch.empty_like(flat_g)]
    stage = [torch.empty_like(flat_p), torch.empty_like(flat_p)]
    views = []
    for buf in gbuf:
        base = flat_g.data_ptr()
        views.append([buf[(p.grad.data_ptr() - base) // 4:(p.grad.data_ptr() - base) // 4 + p.numel()]
                      .view_as(p) for p in params])
    Ke = max(3, min(K, 300))

    def run(steps):
        stepped = [None, None]   # step that last read gradient buffer i
        staged = [None, None]    # device copy into staging buffer i
        sent = [None, None]      # download from staging buffer i
        for t in range(steps):
            i = t % 2
            if stepped[i] is not None:
                h2d.wait_event(stepped[i])
            with torch.cuda.stream(h2d):
                gbuf[i].copy_(host_g, non_blocking=True)
            uploaded = h2d.record_event()
            for p, g in zip(params, views[i]):
                p.grad = g
            main.wait_event(uploaded)
            opt.step()
            stepped[i] = main.record_event()
            if sent[i] is not None:
                main.wait_event(sent[i])
            stage[i].copy_(flat_p)
            staged[i] = main.record_event()
            d2h.wait_event(staged[i])
            with torch.cuda.stream(d2h):
                host_p.copy_(stage[i], non_blocking=True)
            sent[i] = d2h.record_event()
        for ev in sent:
            if ev is not None:
                main.wait_event(ev)

    run(3)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(main)
    run(Ke)
    e1.record(main)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    for p, g in zip(params, views[0]):  # leave the optimizer on its first gradient buffer
        p.grad = g
    return {"value": n_params * Ke / (ms / 1e3), "unit": UNIT, "steps": Ke,
            "h2d_bytes_per_step": flat_g.numel() * 4, "d2h_bytes_per_step": flat_p.numel() * 4,
            "path": "DFCAdamW.step() with grads H2D from pinned host and params D2H to pinned "
                    "host every step; gradients double-buffered on the device, parameters "
                    "staged by a device copy, so both PCIe directions stay busy"}


def host_overhead_us(opt, n=200) -> float:
    """Host time of one DFCAdamW.step() call, measured while the GPU is held
    busy by a sleep kernel so that no call waits for the device."""
    torch.cuda.synchronize()
    torch.cuda._sleep(int(2e9))
    t0 = time.perf_counter()
    for _ in range(n):
        opt.step()
    dt = time.perf_counter() - t0
    torch.cuda.synchronize()
    return dt / n * 1e6


# ----------------------------------------------------------------------------
# our arm, N GPUs: ZeRO-1 over a flat 2^30-element parameter vector
# ----------------------------------------------------------------------------
ZERO_PARAMS = 1 << 30
NVLINK_GBS = 770.0  # measured peer copy per direction on this pool's B200s


def time_sharded_alone(device, group, K=10):
    """The same ZeRO-1 workload with a one-rank process group on this GPU
    (compression + packed step over the whole vector, no exchange): the
    one-GPU point of the series, measured in the same run.  Returns ms per
    step (max over the ranks, which all run it at once)."""
    from t3st_b200.zero import ShardedDFCAdamW

    P = ZERO_PARAMS
    gen = torch.Generator(device=device).manual_seed(1234)
    param = torch.nn.Parameter(torch.empty(P, device=device).normal_(0.0, 0.02, generator=gen))
    opt = ShardedDFCAdamW([param], lr=LR, betas=BETAS, eps=EPS, weight_decay=WD,
                          moment_format="packed", compress_grads=True, process_group=group)
    del param
    opt.flat_grad[:P].normal_(0.0, 1e-3, generator=gen)
    for _ in range(3):
        opt.step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        opt.step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / K
    del opt
    torch.cuda.empty_cache()
    return ms


def nccl_all_gather_gbs(P, world, device, reps=5):
    """Inbound GB/s per rank of NCCL's all-gather of the FP32 vector (each
    rank receives 4P(N-1)/N bytes): the fabric rate NCCL gets on this box
    for the parameter broadcast, max time over ranks."""
    import torch.distributed as dist

    out = torch.empty(P, dtype=torch.float32, device=device)
    piece = torch.ones(P // world, dtype=torch.float32, device=device)
    for _ in range(2):
        dist.all_gather_into_tensor(out, piece)
    torch.cuda.synchronize()
    dist.barrier()
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        dist.all_gather_into_tensor(out, piece)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / reps, world, device)
    del out, piece
    torch.cuda.empty_cache()
    return 4 * P * (world - 1) / world / (ms / 1e3) / 1e9


def run_sharded(args, rank, world, device):
    import torch.distributed as dist

    from t3st_b200.zero import ShardedDFCAdamW

    sampler = ClockSampler(device).start() if (rank == 0 and not args.no_clocks) else None
    P = ZERO_PARAMS
    peak, peak_kind = measured_hbm_peak()
    # the one-GPU point of the same workload, every rank at once, no exchange
    alone_group, _ = dist.new_subgroups(group_size=1)
    ms_alone = max_over_ranks(time_sharded_alone(device, alone_group), world, device)
    frac_alone = 38 * P / (ms_alone / 1e3) / 1e9 / peak   # 12 B compress + 26 B step
    ag_gbs = nccl_all_gather_gbs(P, world, device)

    gen = torch.Generator(device=device).manual_seed(1234)  # same params on every rank
    param = torch.nn.Parameter(torch.empty(P, device=device).normal_(0.0, 0.02, generator=gen))
    opt = ShardedDFCAdamW([param], lr=LR, betas=BETAS, eps=EPS, weight_decay=WD,
                          moment_format="packed", transport=args.transport,
                          fused_ctas_per_sm=args.fused_ctas,
                          compress_ctas_per_sm=args.compress_ctas,
                          **({} if args.side_priority is None else
                             {"side_stream_priority": args.side_priority}),
                          **({"overlap_buckets": True} if args.overlap_buckets else {}),
                          **({} if args.fuse_compression is None else
                             {"fuse_compression": args.fuse_compression}),
                          **({} if args.overlap_barrier is None else
                             {"overlap_barrier": args.overlap_barrier}),
                          **({} if args.bucket_elems is None else
                             {"bucket_elems": args.bucket_elems}))
    del param
    ggen = torch.Generator(device=device).manual_seed(100 + rank)  # per-rank gradients
    opt.flat_grad[:P].normal_(0.0, 1e-3, generator=ggen)
    for _ in range(max(3, args.warmup)):
        opt.step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(device)
    K = args.steps
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    opt.step()  # untimed lead-in step: e0 is queued behind it
    e0.record(stream)
    for _ in range(K):
        opt.step()
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ms = max_over_ranks(e0.elapsed_time(e1), world, device)
    clocks = sampler.stop() if sampler is not None else {"skipped": "rank > 0 or --no-clocks"}
    if opt.peer_status():
        raise RuntimeError(f"a cross-GPU barrier gave up (status {opt.peer_status()})")
    value = P * K / (ms / 1e3)
    # roofline: the slower of the bytes through this rank's HBM and its NVLink
    # bytes.  HBM counts the peers' traffic into this GPU's memory too.
    if opt.transport == "nvls":
        # compress over P; own step reads p, m, v and writes m, v (20 B/elem of
        # the shard); the switch reads all of this rank's bf16 gradients (2P)
        # and writes every rank's FP32 parameters here (4P)
        hbm_bytes = 12 * P + 20 * P // world + 6 * P
        # in: the reduced bf16 piece + every rank's FP32 parameters (own included,
        # through the switch); out: all bf16 gradients + the FP32 piece once
        nvl_bytes = max(2 * P // world + 4 * P, 2 * P + 4 * P // world)
    else:
        # compress over P; step over the shard (26 B/elem: bf16 gradient, p, m,
        # v, p written); the peers' reads of this rank's bf16 gradients for
        # their pieces and their FP32 parameter writes here: 6 B/elem of the rest
        hbm_bytes = 12 * P + 26 * P // world + 6 * P * (world - 1) // world
        nvl_bytes = 6 * P * (world - 1) // world  # bf16 RS + FP32 AG, per direction
    t_hbm = hbm_bytes / (peak * 1e9)
    t_nvl = nvl_bytes / (NVLINK_GBS * 1e9)
    roof_rate = P / max(t_hbm, t_nvl)
    t_nvl_ag = nvl_bytes / (ag_gbs * 1e9)
    roof_rate_ag = P / max(t_hbm, t_nvl_ag)
    line = None
    if rank == 0:
        frac = value / roof_rate
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms / K, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {
                "workload": "ZeRO-1 sharded DFC-AdamW step over a flat 2^30-element FP32 "
                            "parameter vector: bf16 error-feedback compression, reduce of "
                            "the bf16 gradients, packed-moment step on the rank's 1/N, FP32 "
                            "parameter broadcast (peer: one fused kernel over NVLink peer "
                            "memory between two barriers; nvls: the same kernel reducing and "
                            "broadcasting through NVSwitch multicast; nccl: reduce-scatter + "
                            "step + all-gather)",
                "params": P, "moment_format": "packed", "parallelism": f"zero1-dp{world}",
                "transport": opt.transport,
                "fused_ctas_per_sm": opt.fused_ctas,
                "bucket_elems": opt.bucket, "buckets": opt.n_buckets,
                "compress_ctas_per_sm": getattr(opt.kernels, "compress_ctas", None),
                "side_stream_priority": opt.side_stream_priority,
                "overlap_buckets": opt.overlap_buckets,
                "fuse_compression": opt.fuse_compression,
                "overlap_barrier": opt.overlap_barrier,
                "l2": "inputs 4+ GB per rank per step > 126 MB L2 (no flush)",
                "timed_region": "CUDA events on the launching stream; e0 queued behind one "
                                "untimed in-flight step; max over ranks",
            },
            "roofline": {"bound": "nvlink" if t_nvl > t_hbm else "hbm",
                         "achieved": value, "peak": roof_rate, "unit": UNIT,
                         "frac": frac,
                         "hbm_bytes_per_rank": hbm_bytes, "nvlink_bytes_per_rank": nvl_bytes,
                         "hbm_peak_gbs": peak, "hbm_peak_source": f"{peak_kind} hbm_gbs",
                         "nvlink_gbs": NVLINK_GBS,
                         "nvlink_source": "measured peer copy per direction on this pool",
                         "traffic": None},
            # the same roofline with the fabric rate NCCL's all-gather of the FP32
            # vector reaches on this box in this run (a pattern-specific rate)
            "roofline_fabric_measured": {
                "nvlink_gbs": ag_gbs, "source": "NCCL all_gather_into_tensor of the 2^30 FP32 "
                                               "vector, inbound bytes per rank / time, this run",
                "bound": "nvlink" if t_nvl_ag > t_hbm else "hbm", "peak": roof_rate_ag,
                "unit": UNIT, "frac": value / roof_rate_ag},
            # the one-GPU point of this workload (measured in this run) and the
            # scaling efficiency as the north star defines it: roofline fraction
            # at N over roofline fraction at 1
            "one_gpu_same_workload": {
                "value": P / (ms_alone / 1e3), "unit": UNIT, "ms_per_step": ms_alone,
                "roofline_frac": frac_alone,
                "roofline": "38 B/elem (12 compression + 26 step) at the measured HBM peak"},
            "roofline_frac_ratio_vs_1gpu": frac / frac_alone,
            # the same ratio with the NVLink term at the NCCL bus bandwidth measured in
            # this run (the all-gather rate above), as the sharded roofline is defined
            # over the measured NCCL bandwidth; the line above uses 770 GB/s
            "roofline_frac_ratio_vs_1gpu_nccl_rate": (value / roof_rate_ag) / frac_alone,
            # per step: peer/nvls -- a barrier and a fused kernel per bucket, the
            # closing barrier, and a compression per bucket (fused: only bucket 0's
            # runs alone); nccl -- a compression and a step per bucket
            "gpu_launches": K * ((2 * opt.n_buckets + 2 if opt.fuse_compression
                                  else 3 * opt.n_buckets + 1)
                                 if opt.transport in ("peer", "nvls") else 2 * opt.n_buckets),
            "clocks": clocks,
        }
    if not args.no_e2e:
        e2e = run_sharded_e2e(opt, P, device, world)
        if rank == 0:
            line["e2e"] = e2e
    return line


def run_sharded_e2e(opt, P, device, world, steps=3):
    """Public API with host buffers: each rank's gradients come from pinned
    host memory and its updated parameters go back to it every step."""
    import torch.distributed as dist

    host_g = torch.empty(P, dtype=torch.float32, pin_memory=True)
    host_p = torch.empty(P, dtype=torch.float32, pin_memory=True)
    host_g.copy_(opt.flat_grad[:P])
    stream = torch.cuda.current_stream(device)
    opt.flat_grad[:P].copy_(host_g, non_blocking=True)
    opt.step()
    host_p.copy_(opt.flat_param[:P], non_blocking=True)
    dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        opt.flat_grad[:P].copy_(host_g, non_blocking=True)
        opt.step()
        host_p.copy_(opt.flat_param[:P], non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world, device)
    return {"value": P * steps / (ms / 1e3), "unit": UNIT, "steps": steps,
            "h2d_bytes_per_step": P * 4, "d2h_bytes_per_step": P * 4,
            "path": "ShardedDFCAdamW.step() with each rank's grads H2D from pinned host and "
                    "params D2H to pinned host every step"}


def main():
    args = parse_args()
    rank, world, local = (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
                          int(os.environ.get("LOCAL_RANK", "0")))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    rank, world, local = dist_setup(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.kernels_only:
        if rank == 0:
            peak, _ = measured_hbm_peak()
            print(json.dumps(run_kernels(device, peak, args.elems or ZERO_PARAMS)), flush=True)
        return
    if args.replay_only:
        if rank == 0:
            peak, peak_kind = measured_hbm_peak()
            print(json.dumps({"replay": run_replay(device, peak, peak_kind, n=args.replay_batch,
                                                   cpu=not args.no_cpu_baseline)}), flush=True)
        return
    if world == 1:
        line = run_single(args, device)
    else:
        line = run_sharded(args, rank, world, device)
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
