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

Usage: python -m mround_b200.kernel_sweep [--reps N] [--quick | --attention]
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


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--attention", action="store_true")
    args = ap.parse_args()
    if args.attention:
        attention(args.reps)
    else:
        run(args.reps, args.quick)


if __name__ == "__main__":
    main()
