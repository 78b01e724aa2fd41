"""Benchmark: SignRound v2 block tuning of a Qwen2.5-7B-architecture block on B200.

Metric: Qwen2.5-7B-arch W2 g64 tuning, blocks/s (and wall-s per
model) at 1/2/4/8 B200.  A *step* is one pass of the hot path over one
calibration batch: block forward on the fake-quantized weights, the outlier-
suppressed loss, backward, and the signed update of V/alpha/beta -- one
iteration of ``_tune`` (reference mround/pipeline/runner.py:914-937).  A block
is 200 such steps plus 4 forward passes over each of the 16 batches (score
before, score after, targets, advance), so

    blocks/s = 1 / (200 * t_step + 64 * t_forward_batch)

with both times measured here with CUDA events on the launching stream
(t_forward in a second timed region right after the K steps).

Workload: one block of the Qwen2.5-7B architecture (hidden 3584, 28/4 heads,
SwiGLU 18944, QKV bias), random-init N(0, 0.02) bf16 weights, W2 asym g64;
16 calibration batches of 8 x 2048 Zipf(1.1) tokens, block-0 inputs (token
embeddings, float32) -- synthetic stand-ins for pile-10k and the checkpoint.
Every batch input (8 x 2048 x 3584 float32 = 235 MB) is larger than L2, so
no flush is needed between steps.  Under torchrun each of N ranks holds 8/N
sequences of every batch (strong scaling: the global batch is fixed).

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
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

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ITERS = 200
N_BATCHES = 16
BATCH = 8
SEQ = 2048
PASSES_PER_BATCH = 4
METRIC = "Qwen2.5-7B-arch W2g64 tuning: blocks/s (wall-s/model in 'wall_s_model')"
UNIT = "blocks/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--arch", default="qwen2.5-7b")
    ap.add_argument("--bits", type=int, default=2)
    ap.add_argument("--group", type=int, default=64)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--exchange", default="auto", choices=["auto", "p2p", "copy", "nccl"],
                    help="weight-gradient exchange at N > 1 (default: the runner's choice by "
                         "rank count -- fused GEMM peer stores up to 4 ranks, NCCL at 8)")
    ap.add_argument("--gather", default="codes", choices=["codes", "operands"],
                    help="what the ranks all-gather after the row-sharded step at N > 1: "
                         "codes and per-group scale / zero point (default) or the operands")
    ap.add_argument("--precision", default="tuning", choices=["tuning", "bf16x3"],
                    help="tuning: the runner's default (tf32 backward GEMMs); bf16x3: three "
                         "bf16 products in every GEMM")
    return ap.parse_args()


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event reasons sampled every 10 ms during the timed region.

    Reads NVML (found by the CUDA device's UUID, so it is the GPU this rank
    drives); falls back to ``nvidia-smi -lms 200`` when NVML is unavailable.
    Nothing here changes a GPU setting.  A timed region shorter than the first
    sample still records one sample, taken when the region ends.
    """

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
               ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device) -> None:
        self.device = device
        self.samples: list[tuple[float, float, set]] = []
        self.proc = None
        self.handle = None
        self.stop = threading.Event()
        self.thread = None

    def _nvml_handle(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(self.device).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(
                uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:  # noqa: BLE001 -- any NVML failure selects the fallback
            return None, None

    def _nvml_sample(self):
        nv = self.nvml
        sm = float(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM))
        mx = float(nv.nvmlDeviceGetMaxClockInfo(self.handle, nv.NVML_CLOCK_SM))
        mask = int(nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle))
        self.samples.append((sm, mx, {n for n, bit in self.REASONS if mask & bit}))

    def _nvml_loop(self):
        while not self.stop.wait(0.01):
            self._nvml_sample()

    def __enter__(self):
        self.nvml, self.handle = self._nvml_handle()
        if self.handle is not None:
            self.thread = threading.Thread(target=self._nvml_loop, daemon=True)
            self.thread.start()
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._smi_read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _smi_read(self):
        names = [n for n, _ in self.REASONS]
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm, mx = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            self.samples.append((sm, mx, {n for n, f in zip(names, parts[5:9])
                                          if f.lower().startswith("active")}))

    def __exit__(self, *exc):
        self.stop.set()
        if self.handle is not None:
            self.thread.join(timeout=1)
            if not self.samples:
                self._nvml_sample()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self) -> dict:
        sm = [s[0] for s in self.samples]
        reasons = set().union(*(s[2] for s in self.samples)) if self.samples else set()
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(s[1] for s in self.samples) if sm else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "source": "nvml" if self.handle is not None else "nvidia-smi"}


# DRAM bytes (read + write) per K3 launch, averaged over the 11 weight GEMMs of
# one 7B step (16384 tokens, N=1, the tuning form: forward bf16x3, backward
# tf32), from one ncu capture of each shape's warm launch:
#   ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum
#       --clock-control none -k regex:gemm_kernel --csv
#       python -m mround_b200.kernel_sweep --gemm-all 16384
# (50.8 GB per step for 17.8 GB of operands and outputs).
GEMM_TRAFFIC_7B = 4.62e9


# ----------------------------------------------------------------- workload
def build_workload(args, dist, device):
    from mround_b200.pipeline.arch import get_arch
    from mround_b200.pipeline.block import DeviceBlock, Precision
    from mround_b200.pipeline.model import SyntheticModel, zipf_tokens

    arch = get_arch(args.arch)
    model = SyntheticModel(arch, seed=0)
    tokens = zipf_tokens(arch.vocab, N_BATCHES * BATCH, SEQ, seed=42)
    batches = [tokens[i * BATCH:(i + 1) * BATCH] for i in range(N_BATCHES)]
    embed = model.embed_tokens()
    rows = dist.shard(BATCH)
    inputs = []
    for b in batches:
        ids = torch.as_tensor(b[rows], dtype=torch.long)
        inputs.append(embed[ids].float().to(device).contiguous())
    block = DeviceBlock(arch, model.block(0), device)
    prec = Precision()
    with torch.no_grad():
        targets = [block.forward_fused(x, prec, False)[0] for x in inputs]
    return arch, model, block, inputs, targets


def make_tuner(args, block, dist):
    from mround_b200.pipeline.runner import QuantizationRunner
    from mround_b200.schemes import QuantScheme, TuningConfig

    from mround_b200.pipeline.block import Precision

    scheme = QuantScheme(bits=args.bits, group_size=args.group, symmetry="asym")
    runner = QuantizationRunner(scheme, TuningConfig(iters=ITERS), dist=dist,
                                exchange=args.exchange, gather=args.gather,
                                precision=Precision() if args.precision == "bf16x3" else None)
    return runner.tuner_for(block, "model.layers.0")


def timed(fn, n, dist, device):
    """Run fn(i) n times between barriers; device time (CUDA events), max over ranks."""
    dist.barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(n):
        fn(i)
    end.record()
    torch.cuda.synchronize(device)
    dist.barrier()
    ms = start.elapsed_time(end)
    return dist.max_scalar(ms, device)


def block_seconds(t_step_ms, t_fwd_ms):
    return (ITERS * t_step_ms + PASSES_PER_BATCH * N_BATCHES * t_fwd_ms) / 1e3


# ----------------------------------------------------------------- e2e
class HostStreams:
    """Calibration shards in pinned host memory, copied to the device per step
    on a side stream (double-buffered) -- the path for streams that do not stay
    resident in HBM."""

    def __init__(self, inputs, targets, device):
        self.host = [(x.cpu().pin_memory(), t.cpu().pin_memory()) for x, t in zip(inputs, targets)]
        self.device = device
        self.copy = torch.cuda.Stream(device)
        self.slots = [(torch.empty_like(inputs[0]), torch.empty_like(targets[0])) for _ in range(2)]
        self.ready = [torch.cuda.Event(), torch.cuda.Event()]
        self.free = [torch.cuda.Event(), torch.cuda.Event()]
        self.h2d_bytes = inputs[0].numel() * 4 * 2

    def prefetch(self, i, b):
        slot = i % 2
        with torch.cuda.stream(self.copy):
            self.copy.wait_event(self.free[slot])
            x, t = self.slots[slot]
            hx, ht = self.host[b]
            x.copy_(hx, non_blocking=True)
            t.copy_(ht, non_blocking=True)
            self.ready[slot].record(self.copy)

    def get(self, i):
        slot = i % 2
        torch.cuda.current_stream().wait_event(self.ready[slot])
        return self.slots[slot]

    def release(self, i):
        self.free[i % 2].record(torch.cuda.current_stream())


# ----------------------------------------------------------------- cpu
def cpu_run(args, model, arch, *, max_steps: int, budget_s: float, warmup: int = 0):
    """The oracle's ``_tune`` restatement timed at full size on this host's cores.

    Two calibration batches of 8 x 2048 Zipf tokens (the GPU arm's first two),
    their targets from the dense block (the first of these forwards also warms
    the thread pool and the allocator), then ``oracle.block_tuner.tune_block``
    as the reference's loop runs it: one scoring pass (a forward and loss per
    batch, timed) and full-batch steps -- fake-quant of every weight, block
    forward, outlier-suppressed loss, backward, signSGD update -- until
    ``max_steps`` steps or ``budget_s`` seconds of steps (at least one), after
    ``warmup`` untimed steps.
    Nothing is extrapolated from a smaller batch: the block time is 200 timed
    step means plus 64 timed forward means."""
    from mround_b200.pipeline.model import zipf_tokens
    from oracle.block_tuner import LINEARS, OracleBlock, tune_block

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ob = OracleBlock(arch, model.block(0), {p: args.bits for p in LINEARS}, args.group)
    tokens = zipf_tokens(arch.vocab, 2 * BATCH, SEQ, seed=42)
    embed = model.embed_tokens()
    inputs = [embed[torch.as_tensor(tokens[i * BATCH:(i + 1) * BATCH], dtype=torch.long)].float()
              for i in range(2)]
    with torch.no_grad():
        targets = [ob.forward(x) for x in inputs]
    res = tune_block(ob, inputs, targets, iters=ITERS, lr0=1.0 / ITERS, suppress=args.bits < 4,
                     max_steps=max_steps, step_budget_s=budget_s, warmup_steps=warmup)
    steps = res["steps_run"]
    t_step = res["step_seconds"] / steps
    t_fwd = res["score_seconds"] / len(inputs)
    blk = ITERS * t_step + PASSES_PER_BATCH * N_BATCHES * t_fwd
    return {
        "value": 1.0 / blk, "unit": UNIT, "cores": threads, "kind": "port",
        "sample": (f"torch-CPU float32 restatement of the reference's loop (oracle/block_tuner.py; "
                   f"the reference's MLX code cannot run without MLX): {steps} full step(s) of one "
                   f"{args.arch} block on a {BATCH}x{SEQ} batch ({t_step:.2f} s each) and a timed "
                   f"scoring pass over 2 batches ({t_fwd:.2f} s per forward); block time = "
                   f"{ITERS} x step + {PASSES_PER_BATCH * N_BATCHES} x forward"),
        "t_step_s": t_step, "t_forward_s": t_fwd, "steps_timed": steps, "warmup_steps": warmup,
    }


# ----------------------------------------------------------------- main
def _claim_stdout():
    """Route everything written to fd 1 (NCCL's banner, library prints) to
    stderr; the returned stream is the only writer of the real stdout, so the
    run prints exactly one JSON line there."""
    saved = os.dup(1)
    os.dup2(2, 1)
    sys.stdout = sys.stderr
    return os.fdopen(saved, "w")


def main():
    args = parse()
    out_stream = _claim_stdout()
    from mround_b200.pipeline.dist import init_from_env

    if args.impl == "reference":
        return reference_arm(args, out_stream)

    dist = init_from_env()
    device = torch.device("cuda", torch.cuda.current_device())
    from mround_b200 import kernels
    from mround_b200._native import lib

    if lib().mr_device_check() != 0:
        raise SystemExit("libmround_b200 needs an sm_100 device")
    arch, model, block, inputs, targets = build_workload(args, dist, device)
    tuner = make_tuner(args, block, dist)

    def step(i):
        b = i % N_BATCHES
        tuner.step(inputs[b], targets[b], i, ITERS)

    for i in range(args.warmup):
        step(i)
    launches0 = kernels.LAUNCHES[0]
    with ClockSampler(device) as clocks:
        ms_steps = timed(lambda i: step(args.warmup + i), args.steps, dist, device)
    launches = kernels.LAUNCHES[0] - launches0
    t_step = ms_steps / args.steps
    n_fwd = min(N_BATCHES, max(4, args.steps))
    ms_fwd = timed(lambda i: tuner.batch_loss(inputs[i % N_BATCHES], targets[i % N_BATCHES]),
                   n_fwd, dist, device)
    t_fwd = ms_fwd / n_fwd
    blk_s = block_seconds(t_step, t_fwd)
    value = 1.0 / blk_s

    # GEMM roofline: per-launch events over one instrumented step
    kernels.GEMM_EVENTS = []
    step(args.warmup + args.steps)
    torch.cuda.synchronize(device)
    ev, kernels.GEMM_EVENTS = kernels.GEMM_EVENTS, None
    gemm_ms = sum(s.elapsed_time(e) for s, e, _, _ in ev)
    alg_flops = sum(f for _, _, f, _ in ev)
    exe_flops = sum(f * p for _, _, f, p in ev)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    peak = peaks.get("bf16_tflops_sustained")
    peak_src = "of measured (bf16_tflops_sustained)"
    if peak is None:
        peak, peak_src = 1400.0, "of fallback (sustained 1.4 PFLOP/s)"
    achieved = alg_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms else 0.0

    # end to end: streams in pinned host memory, per-step H2D + loss D2H
    e2e = None
    if not args.no_e2e:
        hs = HostStreams(inputs[:4], targets[:4], device)
        host_loss = torch.empty((), dtype=torch.float64).pin_memory()

        def e2e_step(i):
            x, t = hs.get(i)
            loss = tuner.step(x, t, i, ITERS)
            hs.release(i)
            hs.prefetch(i + 2, (i + 2) % 4)
            host_loss.copy_(loss, non_blocking=True)

        hs.prefetch(0, 0)
        hs.prefetch(1, 1)
        for i in range(2):
            e2e_step(i)
        ms_e2e = timed(lambda i: e2e_step(2 + i), args.steps, dist, device)

        def e2e_fwd(i):
            x, t = hs.get(i)
            loss = tuner.batch_loss(x, t)
            hs.release(i)
            hs.prefetch(i + 2, (i + 2) % 4)
            host_loss.copy_(loss, non_blocking=True)

        base = 2 + args.steps
        ms_e2e_fwd = timed(lambda i: e2e_fwd(base + i), n_fwd, dist, device)
        blk_e2e = block_seconds(ms_e2e / args.steps, ms_e2e_fwd / n_fwd)
        e2e = {"value": 1.0 / blk_e2e, "unit": UNIT, "h2d_bytes_per_step": hs.h2d_bytes,
               "d2h_bytes_per_step": 8,
               "path": "BlockTuner.step on pinned-host calibration shards, double-buffered H2D"}
        torch.cuda.synchronize(device)

    out = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_step,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": ("fp32 semantics on tcgen05 (float32 accumulate): forward GEMMs as the "
                  "three-product bf16 split, backward GEMMs as one tf32 product"
                  if tuner.precision.grad_weight == 4 else
                  "fp32 via bf16x3 split tcgen05 GEMMs (float32 accumulate)"),
        "data": "synthetic (random-init N(0,0.02) weights, Zipf(1.1) tokens)",
        "config": {"workload": f"{args.arch} block SignRound step, W{args.bits} asym g{args.group}, "
                               f"global batch {BATCH}x{SEQ}, {ITERS} it/block, {N_BATCHES} batches",
                   "global_batch": BATCH, "seq_len": SEQ, "parallelism": f"dp{dist.world}",
                   "gradient_exchange": ("none" if dist.world == 1 else
                                         "NCCL reduce-scatter" if tuner.peer is None else
                                         "dW GEMM, then copy-engine transfers of each owner's rows"
                                         if tuner.peer.streams is not None else
                                         "fused dW GEMM -> reduce-scatter over NVLink peer stores"),
                   "operand_gather": ("none" if dist.world == 1 else
                                      "codes + per-group scale/zero point"
                                      if any(sh.codes is not None
                                             for sh in tuner._shards.values()) else
                                      "bf16 hi/lo + tf32 operands"),
                   "l2": "inputs larger than L2 (235 MB per batch input)"},
        "ms_forward_batch": t_fwd, "block_seconds": blk_s, "wall_s_model": blk_s * arch.layers,
        "gpu_launches": launches,
        "roofline": {"bound": "tensor", "kernel": "mround_b200 gemm_kernel (K3)",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": peak_src,
                     "executed_tflops": exe_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms else 0.0,
                     "executed_frac": (exe_flops / (gemm_ms / 1e3) / 1e12) / peak if gemm_ms else 0.0,
                     "gemm_share_of_step": gemm_ms / t_step if t_step else None,
                     "traffic": GEMM_TRAFFIC_7B if args.arch == "qwen2.5-7b" and dist.world == 1 else None,
                     "traffic_unit": "bytes per weight-GEMM K3 launch (DRAM read + write), ncu capture of each shape"},
        "clocks": clocks.summary(),
        "e2e": e2e,
    }
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        try:
            out["cpu_baseline"] = cpu_run(args, model, arch, max_steps=1, budget_s=0.0)
        except Exception as exc:  # noqa: BLE001 - the baseline is reported, not required
            out["cpu_baseline"] = {"value": None, "error": str(exc)}
    if dist.rank == 0:
        print(json.dumps(out), file=out_stream, flush=True)
    tuner.close()
    if dist.world > 1:
        import torch.distributed as tdist

        tdist.destroy_process_group()


def reference_arm(args, out_stream):
    """The reference path's CPU implementation (the oracle restatement; the
    reference's MLX loop cannot run here), timed on this host's cores: full
    8 x 2048 steps after one untimed warm-up step (``--warmup 0`` skips it),
    at most ``--steps`` of them and as many as fit in two minutes (at least
    one); ``steps`` and ``warmup`` in the line are the numbers run."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from mround_b200.pipeline.arch import get_arch
    from mround_b200.pipeline.model import SyntheticModel

    arch = get_arch(args.arch)
    model = SyntheticModel(arch, seed=0)
    res = cpu_run(args, model, arch, max_steps=max(1, args.steps), budget_s=120.0,
                  warmup=min(1, args.warmup))
    cpu = {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": res["value"], "unit": UNIT,
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": res["steps_timed"],
        "warmup": res["warmup_steps"], "ms_per_step": res["t_step_s"] * 1e3, "ms_forward_batch": res["t_forward_s"] * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (random-init N(0,0.02) weights, Zipf(1.1) tokens)",
        "config": {"workload": f"{args.arch} block SignRound step, W{args.bits} asym g{args.group}, "
                               f"global batch {BATCH}x{SEQ}, {ITERS} it/block, {N_BATCHES} batches",
                   "global_batch": BATCH, "seq_len": SEQ, "parallelism": "cpu"},
        "cpu_baseline": cpu,
        "e2e": {"value": res["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), file=out_stream, flush=True)


if __name__ == "__main__":
    main()
