"""Kernel sweep: HBM throughput of K1, K2, K5, K6 (and K7).

Shapes 896x896, 4864x896, 3584x3584, 18944x3584 (bf16 weights N(0, 0.02)
with 0.1 % outliers x20; V ~ U(-0.5, 0.5); alpha, beta ~ U(0.5, 1.0); upstream
gradient N(0, 1e-3)), bits {2, 3, 4, 8}, groups {32, 64, 128}.  Each launch is
timed alone with CUDA events on the launching stream, after writing a buffer
larger than L2 (so every launch starts cold), median of ``reps``.

Algorithmic bytes per launch (per weight, plus per group):
  K1 fq_forward        read W 2 + V 4, write Wq hi+lo 4            = 10 B (+ 8 B/group)
  K2 ste_signsgd       read dWq 4 + W 2 + V 4, write V 4 + Wq 4    = 18 B (+16 B/group)
  K5 pack_mlx          read W 2 + V 4, write bits/8                 (+12 B/group)
  K6 deltaloss (3 w.)  read g 4 + W 2                               = 6 B

K8 (the scale search) is bound by float32 issue, not HBM: every weight is
read once (2 B) but evaluated against ~200 candidates at ~8 float32 operations
each; it is reported as candidate-element evaluations per second beside its
bandwidth.

``--attention`` times K7's attention-side kernels instead, at the 7B step's
shapes (8 x 2048 tokens, 28 query / 4 key-value heads of 128): the causal
softmax (reads the scores up to each row's position, 4 B, and writes P hi+lo,
4 B, up to the band limit) and its backward (reads dP 4 B and P hi+lo 4 B up
to the position, writes dS hi+lo up to the band limit), RoPE with the head
re-layout and its backward (4 B read + 4 B of hi+lo written per q/k/v element),
and the head merge of the attention output (the same per element).

Other modes (measurement drivers of the profiles):
  --gemm SHAPE TOKENS [--tf32]  one weight GEMM of the 7B step, three launches
                                (the driver of a K3 ncu capture);
  --gemm-table TOKENS           every weight GEMM of the 7B step timed as the
                                bf16 split and as one tf32 product;
  --gemm-all TOKENS             every weight GEMM in the tuning step's form, two
                                launches each (the driver of per-shape ncu counters);
  --step STEPS                  tuning steps of a 7B block, the last between
                                cudaProfilerStart/Stop (a one-step launch list);
  --exchange [--tf32]           the block's weight-gradient exchange, under
                                torch.distributed.run;
  --block-k2                    K2 over the seven linears of a block of each
                                benchmark architecture: one launch per member
                                against one segmented launch.

Usage: python -m mround_b200.kernel_sweep [--reps N] [--quick | --attention | ...]
Prints one JSON line per case, then a summary line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics

import torch

from mround_b200 import kernels

SHAPES = [(896, 896), (4864, 896), (3584, 3584), (18944, 3584)]
BITS = (2, 3, 4, 8)
GROUPS = (32, 64, 128)


def _peak() -> tuple[float, str]:
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    try:
        with open(os.path.join(here, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "of measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "of fallback"


def _case(rows, cols, group, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    w = torch.randn(rows, cols, device=device, generator=g) * 0.02
    hot = torch.rand(rows, cols, device=device, generator=g) < 0.001
    w = torch.where(hot, w * 20.0, w).to(torch.bfloat16)
    v = torch.rand(rows, cols, device=device, generator=g) - 0.5
    ng = cols // group
    a = 0.5 + 0.5 * torch.rand(rows, ng, device=device, generator=g)
    b = 0.5 + 0.5 * torch.rand(rows, ng, device=device, generator=g)
    gq = torch.randn(rows, cols, device=device, generator=g) * 1e-3
    return w, v, a, b, gq


def _time(fn, flush, reps):
    out = []
    for _ in range(reps):
        flush.add_(1.0)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        out.append(s.elapsed_time(e))
    return statistics.median(out)


def run(reps: int = 5, quick: bool = False) -> list[dict]:
    device = torch.device("cuda")
    peak, src = _peak()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=device)  # 256 MB > L2
    shapes = SHAPES[-1:] if quick else SHAPES
    results = []
    for rows, cols in shapes:
        for group in GROUPS:
            for bits in BITS:
                w, v, a, b, gq = _case(rows, cols, group, rows + bits + group, device)
                n = rows * cols
                ng = n // group
                hi, lo = torch.empty_like(w), torch.empty_like(w)
                out = torch.zeros(3, dtype=torch.float64, device=device)
                cases = {
                    "K1_fq_forward": (lambda: kernels.fq_forward(w, v, a, b, bits=bits, group=group,
                                                                 eps=1e-8, wq_hi=hi, wq_lo=lo),
                                      10 * n + 8 * ng),
                    "K2_ste_signsgd": (lambda: kernels.ste_signsgd(gq, w, v, a, b, bits=bits, group=group,
                                                                   eps=1e-8, lr=1e-9, lo=0.1, hi=1.0,
                                                                   wq_hi=hi, wq_lo=lo),
                                       18 * n + 16 * ng),
                    "K5_pack_mlx": (lambda: kernels.pack_mlx(w, v, a, b, bits=bits, group=group, eps=1e-8),
                                    6 * n + n * bits // 8 + 12 * ng),
                    "K6_deltaloss": (lambda: kernels.deltaloss(gq, w, bits=(2, 3, 4), group=group,
                                                               eps=1e-8, out=out),
                                     6 * n),
                }
                from mround_b200.core.scale_search import candidates

                cands = candidates(bits)
                cases["K8_scale_search"] = (
                    lambda: kernels.scale_search(w, bits=bits, group=group, candidates=cands,
                                                 out=a),
                    2 * n + 4 * ng)
                for name, (fn, nbytes) in cases.items():
                    if name == "K6_deltaloss" and bits != 2:
                        continue  # one pass scores every width; timed once per shape/group
                    fn()
                    torch.cuda.synchronize()
                    ms = _time(fn, flush, reps)
                    gbs = nbytes / (ms * 1e-3) / 1e9
                    rec = {"kernel": name, "rows": rows, "cols": cols, "bits": bits, "group": group,
                           "ms": ms, "bytes": nbytes, "gbs": gbs, "frac": gbs / peak,
                           "peak_gbs": peak, "peak_source": src}
                    if name == "K8_scale_search":
                        rec["candidates"] = len(cands)
                        rec["evals_per_s"] = n * len(cands) / (ms * 1e-3)
                    results.append(rec)
                    print(json.dumps(rec), flush=True)
    big = [r for r in results if r["rows"] * r["cols"] >= 3584 * 3584]
    summary = {}
    for name in sorted({r["kernel"] for r in results} - {"K8_scale_search"}):
        sel = [r["frac"] for r in big if r["kernel"] == name]
        if sel:
            summary[name] = {"median_frac_large": statistics.median(sel), "min_frac_large": min(sel),
                             "max_frac_large": max(sel)}
    k8 = [r for r in big if r["kernel"] == "K8_scale_search"]
    if k8:
        summary["K8_scale_search"] = {"median_ms_large": statistics.median(r["ms"] for r in k8),
                                      "median_evals_per_s": statistics.median(r["evals_per_s"]
                                                                              for r in k8)}
    print(json.dumps({"summary": summary, "peak_gbs": peak, "peak_source": src}), flush=True)
    return results


def attention(reps: int = 5, batch: int = 8, heads: int = 28, seq: int = 2048) -> list[dict]:
    device = torch.device("cuda")
    peak, src = _peak()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=device)
    rows = batch * heads * seq
    g = torch.Generator(device=device).manual_seed(seq)
    scores = torch.randn(rows, seq, device=device, generator=g) * 3.0
    dp = torch.randn(rows, seq, device=device, generator=g)
    live = sum((p // 4 + 1) * 4 for p in range(seq)) * (rows // seq)
    band = sum(min(seq, (p // 128 + 2) * 128) for p in range(seq)) * (rows // seq)
    scale = 1.0 / 128 ** 0.5
    state = {}

    def fwd():
        state["p"] = kernels.softmax_causal_split(scores, rows, seq, scale, True)

    def bwd():
        kernels.softmax_bwd_split(dp, state["p"], rows, seq, scale, True)

    hq, hkv, d = heads, 4, 128
    tokens = batch * seq
    width = (hq + 2 * hkv) * d
    qkv = torch.randn(tokens, width, device=device, generator=g)
    ang = torch.rand(seq, d // 2, device=device, generator=g) * 6.0
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    dq = torch.randn(batch, hq, seq, d, device=device, generator=g)
    dk = torch.randn(batch, hkv, seq, d, device=device, generator=g)
    dv = torch.randn(batch, hkv, seq, d, device=device, generator=g)
    o_heads = torch.randn(batch, hq, seq, d, device=device, generator=g)

    def rope():
        kernels.rope_split(qkv, cos, sin, batch, seq, hq, hkv, d)

    def rope_bwd():
        kernels.rope_bwd_split(dq, dk, dv, cos, sin, batch, seq, hq, hkv, d)

    def merge():
        kernels.heads_split(o_heads, batch, seq, hq, d, merge=True)

    results = []
    for name, fn, nbytes in (("K7_softmax_causal", fwd, 4 * live + 4 * band),
                             ("K7_softmax_bwd", bwd, 8 * live + 4 * band),
                             ("K7_rope", rope, 8 * tokens * width),
                             ("K7_rope_bwd", rope_bwd, 8 * tokens * width),
                             ("K7_heads_merge", merge, 8 * tokens * hq * d)):
        fn()
        torch.cuda.synchronize()
        ms = _time(fn, flush, reps)
        gbs = nbytes / (ms * 1e-3) / 1e9
        rec = {"kernel": name, "rows": rows, "cols": seq, "ms": ms, "bytes": nbytes, "gbs": gbs,
               "frac": gbs / peak, "peak_gbs": peak, "peak_source": src}
        results.append(rec)
        print(json.dumps(rec), flush=True)
    return results


# ----------------------------------------------------------------- K3 shapes
# The weight GEMMs of one Qwen2.5-7B block step at ``tokens`` rows of
# activation (16384 = the 8 x 2048 batch on one GPU; 2048 = one sequence per
# GPU at eight): name -> (m, n, k, A K-major, B K-major).
H7, KV7, I7 = 3584, 512, 18944


def gemm_shapes(tokens: int) -> dict[str, tuple[int, int, int, bool, bool]]:
    out = {}
    for name, rows, cols in (("qkv", H7 + 2 * KV7, H7), ("o", H7, H7), ("gu", 2 * I7, H7),
                             ("down", H7, I7)):
        out[f"fwd_{name}"] = (tokens, rows, cols, True, True)
        if name != "qkv":  # the tuning step does not form the block-input gradient
            out[f"dX_{name}"] = (tokens, cols, rows, True, False)
        out[f"dW_{name}"] = (rows, cols, tokens, False, False)
    return out


def _gemm_operands(m, n, k, ak, bk, tf32: bool, device):
    a_shape = (m, k) if ak else (k, m)
    b_shape = (n, k) if bk else (k, n)
    a = torch.randn(a_shape, device=device)
    b = torch.randn(b_shape, device=device)
    if tf32:
        return (kernels.round_tf32(a, out=a),), (kernels.round_tf32(b, out=b),), a_shape, b_shape
    ops = kernels.split_bf16(a), kernels.split_bf16(b)
    del a, b
    return ops[0], ops[1], a_shape, b_shape


def _launch(aop, bop, c, m, n, k, ak, bk, a_shape, b_shape, tf32: bool):
    if tf32:
        kernels.gemm_tf32(aop[0], bop[0], c, m=m, n=n, k=k, a_kmajor=ak, b_kmajor=bk,
                          lda=a_shape[1], ldb=b_shape[1], ldc=n)
    else:
        kernels.gemm(aop[0], aop[1], bop[0], bop[1], c, m=m, n=n, k=k, a_kmajor=ak, b_kmajor=bk,
                     lda=a_shape[1], ldb=b_shape[1], ldc=n, precision=3)


def gemm_probe(name: str, tokens: int, tf32: bool) -> None:
    """One weight-GEMM shape launched three times: the driver of an ncu
    capture of K3 (``-k regex:gemm_kernel -s 2 -c 1`` takes the third)."""
    m, n, k, ak, bk = gemm_shapes(tokens)[name]
    aop, bop, a_shape, b_shape = _gemm_operands(m, n, k, ak, bk, tf32, "cuda")
    c = torch.empty(m, n, device="cuda")
    for _ in range(3):
        _launch(aop, bop, c, m, n, k, ak, bk, a_shape, b_shape, tf32)
    torch.cuda.synchronize()
    print(json.dumps({"probe": name, "tokens": tokens, "tf32": tf32}), flush=True)


def gemm_all(tokens: int) -> None:
    """Every weight GEMM of the 7B step in the tuning step's form (forward as
    the bf16 split, dX and dW as one tf32 product), two launches each in the
    order of ``gemm_shapes``: under ncu with ``-k regex:gemm_kernel`` the
    second launch of each pair is the warm one, ``2 * i + 1`` for shape i."""
    for name, (m, n, k, ak, bk) in gemm_shapes(tokens).items():
        tf32 = not name.startswith("fwd")
        aop, bop, a_shape, b_shape = _gemm_operands(m, n, k, ak, bk, tf32, "cuda")
        c = torch.empty(m, n, device="cuda")
        for _ in range(2):
            _launch(aop, bop, c, m, n, k, ak, bk, a_shape, b_shape, tf32)
        torch.cuda.synchronize()
        print(json.dumps({"probe": name, "tokens": tokens, "tf32": tf32, "m": m, "n": n, "k": k}),
              flush=True)
        del aop, bop, c


def gemm_table(tokens: int, reps: int = 5) -> list[dict]:
    """Every weight GEMM of the 7B step, as the three-product bf16 split and
    as one tf32 product: device time (CUDA events, median of ``reps``, after
    a warm-up launch), algorithmic TF/s (2 m n k per launch) and executed
    TF/s in bf16-product units (3 for the split, 2 for tf32)."""
    peak = None
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    try:
        with open(os.path.join(here, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        peak = 1590.0
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    out = []
    for name, (m, n, k, ak, bk) in gemm_shapes(tokens).items():
        for tf32 in (False, True):
            aop, bop, a_shape, b_shape = _gemm_operands(m, n, k, ak, bk, tf32, "cuda")
            c = torch.empty(m, n, device="cuda")
            fn = lambda: _launch(aop, bop, c, m, n, k, ak, bk, a_shape, b_shape, tf32)  # noqa: E731
            fn()
            torch.cuda.synchronize()
            ms = _time(fn, flush, reps)
            alg = 2.0 * m * n * k / (ms * 1e-3) / 1e12
            cost = kernels.TF32_PRODUCT_COST if tf32 else 3
            rec = {"gemm": name, "form": "tf32" if tf32 else "bf16x3", "m": m, "n": n, "k": k,
                   "ms": ms, "alg_tflops": alg, "executed_tflops": alg * cost,
                   "executed_frac_burst": alg * cost / peak}
            out.append(rec)
            print(json.dumps(rec), flush=True)
            del aop, bop, c
    return out


# ----------------------------------------------------------------- block K2
def block_k2(reps: int = 5, bits: int = 2, group: int = 64) -> list[dict]:
    """K2 over the seven linears of one block of each benchmark architecture:
    seven launches (one per member) against one segmented launch
    (``ste_signsgd_segments``), each timed cold (after a 256 MB write), with
    the configuration-2 byte count (18 B/weight + 16 B/group, hi/lo operands)."""
    from mround_b200.pipeline.arch import get_arch

    device = torch.device("cuda")
    peak, src = _peak()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=device)
    out = []
    for name in ("smollm2-135m", "qwen2.5-0.5b", "qwen2.5-3b", "qwen2.5-7b"):
        shapes = get_arch(name).linear_shapes()
        segs, nbytes = [], 0
        for i, (rows, cols) in enumerate(shapes.values()):
            w, v, a, b, gq = _case(rows, cols, group, 7 + i, device)
            segs.append({"gq": gq, "w": w, "v": v, "alpha": a, "beta": b, "bits": bits,
                         "lr": 1e-9, "lo": 0.1, "hi": 1.0, "wq_hi": torch.empty_like(w),
                         "wq_lo": torch.empty_like(w)})
            nbytes += 18 * rows * cols + 16 * rows * (cols // group)

        def each():
            for sg in segs:
                kernels.ste_signsgd(sg["gq"], sg["w"], sg["v"], sg["alpha"], sg["beta"],
                                    bits=bits, group=group, eps=1e-8, lr=sg["lr"], lo=0.1,
                                    hi=1.0, wq_hi=sg["wq_hi"], wq_lo=sg["wq_lo"])

        def grouped():
            kernels.ste_signsgd_segments(segs, group=group, eps=1e-8)

        # K9: the whole block's operands (bf16 hi/lo + tf32) rebuilt from codes,
        # as every rank does after the codes gather (9 B/weight + 8 B/group)
        fused = [(sum(shapes[p][0] for p in ("self_attn.q_proj", "self_attn.k_proj",
                                               "self_attn.v_proj")), shapes["self_attn.q_proj"][1]),
                 shapes["self_attn.o_proj"],
                 (2 * shapes["mlp.gate_proj"][0], shapes["mlp.gate_proj"][1]),
                 shapes["mlp.down_proj"]]
        bufs, k9_bytes = [], 0
        for rows, cols in fused:
            ng = rows * cols // group
            bufs.append((torch.randint(0, 1 << bits, (rows, cols), dtype=torch.uint8,
                                       device=device),
                         torch.rand(ng, device=device) * 1e-2, torch.rand(ng, device=device) * 3,
                         torch.empty(rows, cols, dtype=torch.bfloat16, device=device),
                         torch.empty(rows, cols, dtype=torch.bfloat16, device=device),
                         torch.empty(rows, cols, device=device)))
            k9_bytes += 9 * rows * cols + 8 * ng

        def dequant_block():
            for codes, sc, zp, hi, lo, t32 in bufs:
                kernels.dequant_split(codes, sc, zp, group=group, symmetric=False, wq_hi=hi,
                                      wq_lo=lo, wq_t32=t32)

        dequant_block()
        torch.cuda.synchronize()
        ms = _time(dequant_block, flush, reps)
        gbs = k9_bytes / (ms * 1e-3) / 1e9
        rec = {"kernel": "K9_dequant_block", "arch": name, "launches": len(bufs),
               "bytes": k9_bytes, "ms": ms, "gbs": gbs, "frac": gbs / peak, "peak_gbs": peak,
               "peak_source": src}
        out.append(rec)
        print(json.dumps(rec), flush=True)
        del bufs
        for form, fn in (("per_member", each), ("segmented", grouped)):
            fn()
            torch.cuda.synchronize()
            ms = _time(fn, flush, reps)
            gbs = nbytes / (ms * 1e-3) / 1e9
            rec = {"kernel": "K2_block", "arch": name, "form": form, "launches": 7 if form ==
                   "per_member" else 1, "bytes": nbytes, "ms": ms, "gbs": gbs, "frac": gbs / peak,
                   "peak_gbs": peak, "peak_source": src}
            out.append(rec)
            print(json.dumps(rec), flush=True)
        del segs
    return out


# ----------------------------------------------------------------- one step
def step_probe(steps: int, arch_name: str = "qwen2.5-7b", tokens: int = 2048,
               batch: int = 8) -> None:
    """``steps`` tuning steps of one block (W2 asym g64, the runner's default
    precision) on random block-0 inputs, the last one between
    cudaProfilerStart/Stop -- the launch list of one step under
    ``ncu --profile-from-start off``."""
    from mround_b200.pipeline.arch import get_arch
    from mround_b200.pipeline.block import DeviceBlock
    from mround_b200.pipeline.model import SyntheticModel
    from mround_b200.pipeline.runner import QuantizationRunner
    from mround_b200.schemes import QuantScheme, TuningConfig

    arch = get_arch(arch_name)
    block = DeviceBlock(arch, SyntheticModel(arch, seed=0).block(0), "cuda")
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(batch, tokens, arch.hidden, device="cuda", generator=g) * 0.02
    runner = QuantizationRunner(QuantScheme(bits=2, group_size=64, symmetry="asym"),
                                TuningConfig(iters=200))
    tuner = runner.tuner_for(block, "model.layers.0")
    target = tuner.output(x) + 1e-3
    for i in range(steps - 1):
        tuner.step(x, target, i, 200)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    tuner.step(x, target, steps - 1, 200)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    print(json.dumps({"probe": "step", "arch": arch_name, "steps": steps,
                      "precision": str(runner.precision)}), flush=True)


# ----------------------------------------------------------------- exchange
def exchange_probe(tf32: bool = False) -> None:
    """The weight-gradient exchange of one Qwen2.5-7B block across ranks
    (run under ``torch.distributed.run``).  For the block's four fused weight
    gradients at the step's per-rank token count (16384 / N), four ways, each
    averaged over 10 iterations after 3 warm-up ones, CUDA events, max over
    ranks: ``gemm`` (the dW GEMMs alone, the lower bound), ``nccl`` (dW GEMM,
    then an async NCCL reduce-scatter), ``p2p`` (the dW GEMM stores its rows
    into the owners' slots over NVLink, then each owner's ordered sum) and
    ``copy`` (dW GEMM locally, the copy engines move each owner's rows, the
    same sum).  Rank 0 prints one line per way."""
    import torch.distributed as tdist

    from mround_b200.pipeline.dist import init_from_env
    from mround_b200.pipeline.peer import PeerExchange

    shapes = [(H7 + 2 * KV7, H7), (H7, H7), (2 * I7, H7), (H7, I7)]
    dist = init_from_env("nccl", timeout_s=120.0)
    world, rank = dist.world, dist.rank
    dev = torch.device("cuda", torch.cuda.current_device())
    t = 16384 // world
    gen = torch.Generator(device=dev).manual_seed(rank)
    ins = []
    for rows, cols in shapes:
        dy = torch.randn(t, rows, device=dev, generator=gen)
        x = torch.randn(t, cols, device=dev, generator=gen)
        if tf32:
            ins.append(((None, None, kernels.round_tf32(dy)), (None, None, kernels.round_tf32(x))))
        else:
            ins.append(((*kernels.split_bf16(dy), None), (*kernels.split_bf16(x), None)))
    grads = [torch.empty(r, c, device=dev) for r, c in shapes]
    shards = [torch.empty(r // world, c, device=dev) for r, c in shapes]
    peer = PeerExchange(dist, shapes, dev) if world > 1 else None
    copier = PeerExchange(dist, shapes, dev, copy_engine=True) if world > 1 else None
    epoch = 0

    def dw(dy, x, g, rows, cols):
        if tf32:
            kernels.gemm_tf32(dy[2], x[2], g, m=rows, n=cols, k=t, a_kmajor=False, b_kmajor=False,
                              lda=rows, ldb=cols, ldc=cols)
        else:
            kernels.gemm(dy[0], dy[1], x[0], x[1], g, m=rows, n=cols, k=t, a_kmajor=False,
                         b_kmajor=False, lda=rows, ldb=cols, ldc=cols, precision=3)

    def step(way: str) -> None:
        nonlocal epoch
        if way == "p2p":
            epoch += 1
            for (rows, cols), (dy, x), ex in zip(shapes, ins, peer.layers):
                kw = dict(m=rows, n=cols, k=t, a_kmajor=False, b_kmajor=False, lda=rows, ldb=cols,
                          dst_ptrs=ex.dst_ptrs, ldd=cols, rows_per_rank=ex.rows_per_rank,
                          flag_ptrs=ex.flag_ptrs, done=ex.done, epoch=epoch)
                if tf32:
                    kernels.gemm_rs_tf32(dy[2], x[2], **kw)
                else:
                    kernels.gemm_rs(dy[0], dy[1], x[0], x[1], precision=3, **kw)
            for ex, out in zip(peer.layers, shards):
                kernels.reduce_slots(ex.slots, ex.flags, epoch, out)
            return
        if way == "copy":
            epoch += 1
            for (rows, cols), (dy, x), g, ex in zip(shapes, ins, grads, copier.layers):
                dw(dy, x, g, rows, cols)
                ex.epoch = epoch
                ex.send(g)
            for ex in copier.layers:
                ex.wait_copies()
            for ex, out in zip(copier.layers, shards):
                kernels.reduce_slots(ex.slots, ex.flags, epoch, out)
            return
        works = []
        for (rows, cols), (dy, x), g, out in zip(shapes, ins, grads, shards):
            dw(dy, x, g, rows, cols)
            if way == "nccl" and world > 1:
                works.append(tdist.reduce_scatter_tensor(out, g, async_op=True))
        for w in works:
            w.wait()

    ways = ("gemm", "nccl", "p2p", "copy") if world > 1 else ("gemm",)
    for way in ways:
        for _ in range(3):
            step(way)
        dist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(10):
            step(way)
        end.record()
        torch.cuda.synchronize()
        ms = dist.max_scalar(start.elapsed_time(end) / 10, dev)
        status = int(kernels.lib().mr_peer_status(1))
        if rank == 0:
            print(json.dumps({"probe": "exchange", "world": world, "way": way,
                              "form": "tf32" if tf32 else "bf16x3", "ms_per_block": ms,
                              "peer_status": status}), flush=True)
    dist.barrier()
    if peer is not None:
        peer.close()
        copier.close()
    if world > 1:
        tdist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--attention", action="store_true", help="K7 attention-side kernels")
    ap.add_argument("--gemm", nargs=2, metavar=("SHAPE", "TOKENS"),
                    help="launch one 7B weight GEMM three times (ncu driver)")
    ap.add_argument("--gemm-table", type=int, metavar="TOKENS",
                    help="time every 7B weight GEMM as bf16x3 and tf32")
    ap.add_argument("--gemm-all", type=int, metavar="TOKENS",
                    help="every 7B weight GEMM in the tuning form, two launches each (ncu driver)")
    ap.add_argument("--tf32", action="store_true", help="--gemm / --exchange: tf32 operands")
    ap.add_argument("--step", type=int, metavar="STEPS",
                    help="7B tuning steps, the last between cudaProfilerStart/Stop")
    ap.add_argument("--exchange", action="store_true",
                    help="weight-gradient exchange of a 7B block (under torch.distributed.run)")
    ap.add_argument("--block-k2", action="store_true",
                    help="K2 over a block's seven linears: per-member against one launch")
    args = ap.parse_args()
    if args.attention:
        attention(args.reps)
    elif args.gemm:
        gemm_probe(args.gemm[0], int(args.gemm[1]), args.tf32)
    elif args.gemm_table:
        gemm_table(args.gemm_table, args.reps)
    elif args.gemm_all:
        gemm_all(args.gemm_all)
    elif args.step:
        step_probe(args.step)
    elif args.exchange:
        exchange_probe(args.tf32)
    elif args.block_k2:
        block_k2(args.reps)
    else:
        run(args.reps, args.quick)


if __name__ == "__main__":
    main()
