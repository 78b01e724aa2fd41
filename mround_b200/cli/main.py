"""``mround-b200 quantize`` -- the reference's ``mround quantize`` flags on B200.

Restates the ``quantize`` sub-command of reference mround/cli/main.py:41-245,
529-583: same flags and defaults; ``eval`` and ``doctor`` are not on the tuning
path and are not provided.  The model argument is a local Llama/Qwen2
checkpoint directory or a synthetic architecture (``synthetic:qwen2.5-7b``).  Under torchrun each rank takes a shard of every
calibration batch.
"""

from __future__ import annotations

import argparse
import os
import sys

from mround_b200 import __version__
from mround_b200.exceptions import MRoundError

__all__ = ["build_parser", "main"]


def _widths(text: str) -> tuple[int, ...]:
    try:
        return tuple(int(x) for x in text.split(",") if x.strip())
    except ValueError as exc:
        raise argparse.ArgumentTypeError(f"--options takes comma-separated widths, got {text!r}") from exc


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(prog="mround-b200", description="SignRound v2 on B200")
    parser.add_argument("--version", action="version", version=f"mround-b200 {__version__}")
    sub = parser.add_subparsers(dest="command", required=True)
    q = sub.add_parser("quantize", help="Quantize a model and write an MLX checkpoint.")
    q.add_argument("model", help="a local Llama/Qwen2 checkpoint directory, or synthetic:<arch>[@seed] "
                   "(e.g. synthetic:qwen2.5-7b)")
    q.add_argument("--output-dir", "-o", required=True)
    q.add_argument("--bits", type=int, default=4)
    q.add_argument("--group-size", type=int, default=64)
    q.add_argument("--asym", action="store_true", help="Asymmetric codes with a zero point.")
    q.add_argument("--average-bits", type=float, default=None)
    q.add_argument("--format", default="mlx", choices=["mlx"])
    q.add_argument("--options", type=_widths, default=(2, 3, 4))
    q.add_argument("--remainder-bits", type=int, default=None)
    q.add_argument("--iters", type=int, default=200)
    q.add_argument("--samples", type=int, default=128)
    q.add_argument("--seq-len", type=int, default=2048)
    q.add_argument("--batch-size", type=int, default=8)
    q.add_argument("--micro-batches", type=int, default=1)
    q.add_argument("--calibration", default="auto")
    q.add_argument("--seed", type=int, default=None, help="Calibration seed.")
    q.add_argument("--allow-dense", action="store_true",
                   help="Accept any block coverage (min_block_coverage=0).")
    q.add_argument("--memory-budget", type=int, default=None)
    q.add_argument("--skip-memory-check", action="store_true")
    q.add_argument("--dry-run", action="store_true", help="Resolve and validate, then stop.")
    q.add_argument("--resume-dir", default=None,
                   help="Record each finished block here; rerunning the same command with "
                        "the same directory continues after the last finished block.")
    q.add_argument("--scoring-samples", type=int, default=None,
                   help="Sequences for the mixed-precision scoring pass (api scoring_samples).")
    q.add_argument("--scoring-seq-len", type=int, default=None,
                   help="Tokens per scoring sequence (api scoring_seq_len).")
    q.add_argument("--sensitivity-gradients", default="auto",
                   choices=["auto", "own_width", "widest"])
    return parser


def _quantize(args: argparse.Namespace) -> int:
    from mround_b200.api import MIN_BLOCK_COVERAGE, _resolve_scheme, quantize
    from mround_b200.schemes import Symmetry, TuningConfig

    symmetry = Symmetry.ASYMMETRIC if args.asym else Symmetry.SYMMETRIC
    tuning = TuningConfig(iters=args.iters, n_samples=args.samples, seq_len=args.seq_len,
                          batch_size=args.batch_size, micro_batches=args.micro_batches)
    if args.dry_run:
        scheme, widths = _resolve_scheme(bits=args.bits, group_size=args.group_size,
                                         symmetry=symmetry, average_bits=args.average_bits,
                                         candidate_bits=args.options,
                                         remainder_bits=args.remainder_bits, scheme=None,
                                         scale_init=None)
        print(f"scheme {scheme}, widths {sorted(widths)}, tuning {tuning}")
        return 0
    result = quantize(args.model, output_dir=args.output_dir, bits=args.bits,
                      group_size=args.group_size, symmetry=symmetry, average_bits=args.average_bits,
                      candidate_bits=args.options, remainder_bits=args.remainder_bits,
                      tuning=tuning, calibration=args.calibration, export_format=args.format,
                      seed=args.seed, memory_budget=args.memory_budget,
                      scoring_samples=args.scoring_samples, scoring_seq_len=args.scoring_seq_len,
                      sensitivity_gradients=args.sensitivity_gradients,
                      memory_check=not args.skip_memory_check,
                      min_block_coverage=0.0 if args.allow_dense else MIN_BLOCK_COVERAGE,
                      resume_dir=args.resume_dir)
    if int(os.environ.get("RANK", "0")) == 0:
        if result.summary is not None:
            print(result.summary.describe())
        print(result.describe())
    return 0


def main(argv: list[str] | None = None) -> int:
    args = build_parser().parse_args(argv)
    try:
        if args.command == "quantize":
            return _quantize(args)
    except MRoundError as exc:
        print(f"mround-b200: {exc}", file=sys.stderr)
        return 2
    finally:
        from mround_b200.pipeline.dist import shutdown

        shutdown()
    return 1


if __name__ == "__main__":
    raise SystemExit(main())
