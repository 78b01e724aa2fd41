"""Public entry point: quantize a model and write an MLX checkpoint, on B200.

``quantize`` keeps the reference's signature and flow
(mround/api.py:366-794): resolve the scheme, refuse what the export cannot
hold, load the model, build calibration, optionally score and plan mixed
precision, run the block loop, round the remainder to nearest, export, write
``mround_run.json``.  Differences, all refusals rather than substitutions:

- the model is a local Llama/Qwen2 checkpoint directory (config.json +
  safetensors, bf16 linears; :mod:`mround_b200.pipeline.loader`) or a
  synthetic architecture (``"synthetic:<arch>[@seed]"``, e.g.
  ``"synthetic:qwen2.5-7b"``) -- Hub downloads need a network;
- calibration ``"auto"`` is Zipf(1.1) token ids over the vocabulary (the
  reference's pile-10k is not available offline);
- every scheme the reference defines runs on the device (asymmetric and
  symmetric observed range, and the searched v2 scale below 4 bits on
  symmetric runs, ``default_scale_init``);
- ``memory_budget``/``memory_check`` are accepted and recorded, the Mac
  memory and time rules (mround/planner/memory.py, timing.py) are not applied.
"""

from __future__ import annotations

import dataclasses
import json
import time
from collections.abc import Mapping, Sequence
from pathlib import Path
from typing import Any

import torch

from mround_b200.exceptions import (
    ArchitectureError,
    CalibrationError,
    SchemeError,
    UnsupportedSchemeError,
)
from mround_b200.formats.mlx_export import export_mlx, require_mlx_representable
from mround_b200.pipeline.arch import get_arch
from mround_b200.pipeline.dist import DistContext, init_from_env
from mround_b200.pipeline.model import SyntheticModel, zipf_tokens
from mround_b200.pipeline.resume import ResumeStore, run_fingerprint
from mround_b200.pipeline.runner import QuantizationRunner, RunSummary
from mround_b200.pipeline.tuning import QuantizedLayer
from mround_b200.schemes import (
    LOW_BIT_THRESHOLD,
    SUPPORTED_BITS,
    QuantScheme,
    ScaleInit,
    Symmetry,
    TuningConfig,
)

__all__ = ["QuantizeResult", "Storage", "default_scale_init", "load_model", "quantize",
           "quantize_round_to_nearest"]

MIN_BLOCK_COVERAGE = 0.5
DEFAULT_SEED = 42


@dataclasses.dataclass(frozen=True, slots=True)
class Storage:
    stored_bytes: int
    weights: int

    @property
    def bits_per_weight(self) -> float:
        return 8.0 * self.stored_bytes / self.weights if self.weights else 0.0

    @property
    def compression(self) -> float:
        return 16.0 / self.bits_per_weight if self.bits_per_weight else 0.0


@dataclasses.dataclass(frozen=True, slots=True)
class QuantizeResult:
    output_dir: Path
    summary: RunSummary | None
    scheme_by_layer: dict[str, QuantScheme]
    config_path: Path
    storage: Storage
    skipped: tuple[tuple[str, str], ...] = ()
    mixed: dict[str, Any] | None = None

    def describe(self) -> str:
        return (f"{len(self.scheme_by_layer)} modules tuned, {len(self.skipped)} left dense, "
                f"{self.storage.bits_per_weight:.2f} bits per weight overall "
                f"({self.storage.compression:.2f}x smaller)")


def default_scale_init(narrowest_width: int, symmetry: Symmetry) -> ScaleInit:
    """Searched below 4 bits on symmetric schemes, observed range otherwise
    (reference mround/api.py:116-153)."""
    if Symmetry(symmetry) is not Symmetry.SYMMETRIC:
        return ScaleInit.OBSERVED_RANGE
    return ScaleInit.SEARCHED if narrowest_width < LOW_BIT_THRESHOLD else ScaleInit.OBSERVED_RANGE


def load_model(model):
    """A synthetic architecture (``"synthetic:<arch>[@seed]"``), a local
    Hugging Face checkpoint directory (config.json + safetensors; Llama or
    Qwen2), or an already-built model object."""
    from mround_b200.pipeline.loader import CheckpointModel, is_checkpoint_dir

    if isinstance(model, (SyntheticModel, CheckpointModel)):
        return model
    text = str(model)
    if text.startswith("synthetic:"):
        spec = text.split(":", 1)[1]
        name, _, seed = spec.partition("@")
        return SyntheticModel(get_arch(name), seed=int(seed) if seed else 0)
    if is_checkpoint_dir(text):
        return CheckpointModel(text)
    raise ArchitectureError(
        f"cannot load {text!r}: give a local checkpoint directory (config.json + safetensors) "
        "or \"synthetic:<arch>[@seed]\"; there is no network for Hub downloads")


def _resolve_scheme(*, bits, group_size, symmetry, average_bits, candidate_bits, remainder_bits,
                    scheme, scale_init) -> tuple[QuantScheme, set[int]]:
    if scheme is not None:
        resolved = scheme
    else:
        widths = set(candidate_bits) if average_bits is not None else {bits}
        init = ScaleInit(scale_init) if scale_init is not None else default_scale_init(min(widths), symmetry)
        resolved = QuantScheme(bits=bits, group_size=group_size, symmetry=symmetry, scale_init=init)
    widths = {resolved.bits}
    if average_bits is not None:
        cands = sorted(set(int(b) for b in candidate_bits))
        for b in cands:
            if b not in SUPPORTED_BITS:
                raise SchemeError(f"candidate width {b} is not supported")
        if not cands or not (cands[0] <= average_bits <= cands[-1]):
            raise SchemeError(f"average_bits={average_bits} lies outside the candidate range {cands}")
        widths = set(cands)
        if remainder_bits is not None:
            widths.add(int(remainder_bits))
    return resolved, widths


def _remainder_width(average_bits: float, candidates: Sequence[int], remainder_bits: int | None) -> int:
    """Width of the tensors outside the blocks: the packable width nearest the
    average, ties toward more bits, ``min(8, max(2, floor(avg + 0.5)))``
    (reference mround/api.py:1645-1653)."""
    if remainder_bits is not None:
        return int(remainder_bits)
    return min(8, max(2, int(average_bits + 0.5)))


def _calibration(model: SyntheticModel, tuning: TuningConfig, seed: int | None,
                 calibration: str) -> list:
    if calibration not in ("auto", "zipf"):
        raise CalibrationError(f"calibration {calibration!r} is not available offline; use 'auto'")
    tokens = zipf_tokens(model.arch.vocab, tuning.n_samples, tuning.seq_len,
                         seed=DEFAULT_SEED if seed is None else seed)
    b = tuning.batch_size
    return [tokens[i:i + b] for i in range(0, tokens.shape[0] - b + 1, b)]


def _rtn_layer(weight: torch.Tensor, scheme: QuantScheme, device) -> QuantizedLayer:
    """Round-to-nearest with nothing learned (reference _round_to_nearest_layers,
    mround/api.py:1877-1937): a searched scheme searches unweighted first."""
    from mround_b200 import kernels
    from mround_b200.core.scale_search import search_scales

    w = weight.to(device).to(torch.bfloat16).contiguous()
    rows, cols = w.shape
    ng = cols // scheme.group_size
    zeros = torch.zeros((rows, cols), dtype=torch.float32, device=device)
    ones = torch.ones((rows, ng), dtype=torch.float32, device=device)
    init = None
    if scheme.scale_init is ScaleInit.SEARCHED:
        init = torch.empty((rows, ng), dtype=torch.float32, device=device)
        search_scales(w, scheme, out=init)
    packed, scales, biases, _ = kernels.pack_mlx(
        w, zeros, ones, ones, bits=scheme.bits, group=scheme.group_size, eps=1e-8,
        symmetric=scheme.symmetry is Symmetry.SYMMETRIC, init_scale=init)
    return QuantizedLayer(packed.cpu(), scales.cpu(), biases.cpu(), scheme, (rows, cols))


def _plan_mixed(model, resolved, average_bits, candidate_bits, *, gradient_source, scoring_samples,
                scoring_seq_len, scoring_batch_size, seed, device, given_plan=None, dist=None):
    from mround_b200.pipeline.scoring import score_widths
    from mround_b200.planner.allocator import allocate_bits
    from mround_b200.planner.sensitivity import (
        SENSITIVITY_SAMPLES,
        SENSITIVITY_SEQ_LEN,
        gradient_source_for,
        mixed_budget_bits,
        score_layer_options,
        scoring_batch_size as batch_rule,
    )

    arch = model.arch
    widths = sorted(set(int(b) for b in candidate_bits))
    shapes = {f"{model.block_name(i)}.{p}": s for i in range(arch.layers)
              for p, s in arch.linear_shapes().items() if s[1] % resolved.group_size == 0}
    if given_plan is not None:
        if set(given_plan) != set(shapes):
            raise SchemeError("plan must name every block layer a scored plan would cover and nothing else")
        overrides = {p: resolved.with_bits(int(b)) for p, b in given_plan.items()}
        return overrides, {"plan": "given", "average_bits": average_bits, "candidate_bits": widths}
    source = gradient_source_for(gradient_source, sum(o * i for o, i in shapes.values()))
    n = scoring_samples or SENSITIVITY_SAMPLES
    s = scoring_seq_len or SENSITIVITY_SEQ_LEN
    bsz = scoring_batch_size or batch_rule(n, s)
    tokens = zipf_tokens(arch.vocab, n, s, seed=DEFAULT_SEED if seed is None else seed)
    batches = [tokens[i:i + bsz] for i in range(0, n - bsz + 1, bsz)]
    scored = score_widths(model, batches, widths, resolved, gradient_source=source, device=device,
                          dist=dist)
    budget = mixed_budget_bits(scored.shapes, average_bits, resolved.group_size)
    options = score_layer_options(scored.scores, scored.shapes, resolved)
    alloc = allocate_bits(options, budget_bits=budget)
    overrides = {p: resolved.with_bits(b) for p, b in alloc.by_layer.items()}
    info = {
        "average_bits": average_bits, "candidate_bits": widths, "gradient_source": source,
        "budget_bits": budget, "total_cost_bits": alloc.total_cost_bits,
        "predicted_loss": alloc.predicted_loss, "achieved_average_bits": alloc.average_bits,
        "assignments": alloc.by_layer, "scoring_seconds": scored.seconds,
        "scoring": {"samples": n, "seq_len": s, "batch_size": bsz},
        "describe": (f"mixed plan: {alloc.average_bits:.3f} bits average over "
                     f"{len(alloc.by_layer)} layers, scored in {scored.seconds:.1f}s ({source})"),
    }
    return overrides, info


def _storage(model: SyntheticModel, quantized: Mapping[str, QuantizedLayer], dense: Mapping[str, torch.Tensor]) -> Storage:
    stored = sum(q.packed.numel() * 4 + q.scales.numel() * 2 + q.biases.numel() * 2
                 for q in quantized.values())
    stored += sum(t.numel() * t.element_size() for t in dense.values())
    weights = sum(q.shape[0] * q.shape[1] for q in quantized.values())
    weights += sum(t.numel() for t in dense.values())
    return Storage(stored, weights)


def _dense_tensors(model: SyntheticModel, quantized: Mapping[str, QuantizedLayer]) -> dict[str, torch.Tensor]:
    arch = model.arch
    dense: dict[str, torch.Tensor] = {}
    if "model.embed_tokens" not in quantized:
        dense["model.embed_tokens.weight"] = model.embed_tokens()
    for i in range(arch.layers):
        params = model.block(i)
        name = model.block_name(i)
        dense[f"{name}.input_layernorm.weight"] = params.input_norm
        dense[f"{name}.post_attention_layernorm.weight"] = params.post_norm
        for path, bias in params.biases.items():
            dense[f"{name}.{path}.bias"] = bias
        for path, w in params.linears.items():
            if f"{name}.{path}" not in quantized:
                dense[f"{name}.{path}.weight"] = w
    dense["model.norm.weight"] = model.final_norm()
    if not arch.tied and "lm_head" not in quantized:
        dense["lm_head.weight"] = model.lm_head()
    return dense


def quantize(model: str | Path | SyntheticModel, *, output_dir: str | Path, bits: int = 4,
             group_size: int = 64, symmetry: Symmetry = Symmetry.SYMMETRIC,
             average_bits: float | None = None, candidate_bits: Sequence[int] = (2, 3, 4),
             sensitivity_gradients: str = "auto", remainder_bits: int | None = None,
             dense_remainder: bool = False, scoring_samples: int | None = None,
             scoring_seq_len: int | None = None, scoring_batch_size: int | None = None,
             scheme: QuantScheme | None = None, tuning: TuningConfig | None = None,
             calibration: str = "auto", export_format: str = "mlx", quantized_inputs: bool = True,
             holdout_batches: int = 0, per_layer_recipe: bool = False,
             plan: Mapping[str, int] | None = None, scale_init: ScaleInit | str | None = None,
             min_block_coverage: float = MIN_BLOCK_COVERAGE, seed: int | None = None,
             memory_budget: int | None = None, memory_check: bool = True,
             progress=print, dist: DistContext | None = None,
             resume_dir: str | Path | None = None) -> QuantizeResult:
    """Quantize ``model`` and write an MLX checkpoint to ``output_dir``.

    ``resume_dir`` (not in the reference): record every finished block there,
    and continue a run that stopped, tuning only the blocks it had not
    finished (:mod:`mround_b200.pipeline.resume`).  A directory written by a
    run with different settings or calibration is refused."""
    if export_format != "mlx":
        raise UnsupportedSchemeError(f"export_format {export_format!r} is not available; use 'mlx'")
    if holdout_batches < 0:
        raise CalibrationError(f"holdout_batches must be zero or more, got {holdout_batches}")
    if plan is not None and average_bits is None:
        raise SchemeError("a plan is a mixed run's allocation and needs average_bits")
    if memory_budget is not None and memory_budget <= 0:
        raise ValueError("memory_budget must be a positive number of bytes")
    resolved, widths = _resolve_scheme(bits=bits, group_size=group_size, symmetry=symmetry,
                                       average_bits=average_bits, candidate_bits=candidate_bits,
                                       remainder_bits=remainder_bits, scheme=scheme,
                                       scale_init=scale_init)
    if plan is not None:
        off = sorted({int(b) for b in plan.values()} - set(int(b) for b in candidate_bits))
        if off:
            raise SchemeError(f"plan widths {off} are not on candidate_bits")
    for width in sorted(widths):
        require_mlx_representable(resolved.with_bits(width))
    tuning = tuning or TuningConfig()
    dist = dist or init_from_env()
    device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else None
    if device is None:
        from mround_b200.exceptions import PlatformError

        raise PlatformError("quantize needs a CUDA device (sm_100); there is no CPU path")
    destination = Path(output_dir)
    bundle = load_model(model)
    arch = bundle.arch
    coverage = sum(o * i for o, i in arch.linear_shapes().values() if i % resolved.group_size == 0)
    if coverage < min_block_coverage * arch.block_weights():
        raise ArchitectureError(f"group size {resolved.group_size} reaches {coverage / arch.block_weights():.1%} "
                                f"of the block weights, below min_block_coverage={min_block_coverage}")
    batches = _calibration(bundle, tuning, seed, calibration)
    overrides, plan_info = None, None
    remainder_scheme = resolved
    if average_bits is not None:
        overrides, plan_info = _plan_mixed(
            bundle, resolved, average_bits, candidate_bits, gradient_source=sensitivity_gradients,
            scoring_samples=scoring_samples, scoring_seq_len=scoring_seq_len,
            scoring_batch_size=scoring_batch_size, seed=seed, device=device, given_plan=plan,
            dist=dist)
        remainder_scheme = resolved.with_bits(_remainder_width(average_bits, candidate_bits,
                                                               remainder_bits))
        plan_info["remainder_bits"] = remainder_scheme.bits
        if progress and "describe" in plan_info:
            progress(f"  {plan_info['describe']}")
    runner = QuantizationRunner(resolved, tuning, progress=(lambda r: progress(r.describe())) if progress else None,
                                quantized_inputs=quantized_inputs, holdout_batches=holdout_batches,
                                per_layer_recipe=per_layer_recipe, dist=dist, device=device)
    resume = None
    if resume_dir is not None:
        fingerprint = run_fingerprint(
            model=bundle.name, arch=arch, scheme=resolved, tuning=tuning, scheme_by_layer=overrides,
            batches=batches, world=dist.world, quantized_inputs=quantized_inputs,
            holdout_batches=holdout_batches, per_layer_recipe=per_layer_recipe,
            calibration=calibration)
        resume = ResumeStore(resume_dir, fingerprint, rank=dist.rank)
        dist.barrier()
    summary, quantized = runner.run(bundle, batches, scheme_by_layer=overrides,
                                    expected_blocks=arch.layers, resume=resume)
    skipped: list[tuple[str, str]] = [s for b in summary.blocks for s in b.skipped]
    t0 = time.perf_counter()
    remainder = {"model.embed_tokens": bundle.embed_tokens()}
    if not arch.tied:
        remainder["lm_head"] = bundle.lm_head()
    for path, w in remainder.items():
        if dense_remainder:
            skipped.append((path, "dense by request"))
        elif w.shape[1] % remainder_scheme.group_size:
            skipped.append((path, f"last dimension {w.shape[1]} is not a multiple of "
                                  f"{remainder_scheme.group_size}"))
        else:
            quantized[path] = _rtn_layer(w, remainder_scheme, device)
    remainder_seconds = time.perf_counter() - t0
    dense = _dense_tensors(bundle, quantized)
    config_path = destination / "mround_run.json"
    if dist.rank == 0:
        t1 = time.perf_counter()
        export_mlx(destination, dense, quantized, bundle.config())
        export_seconds = time.perf_counter() - t1
        storage = _storage(bundle, quantized, dense)
        record = {
            "model": bundle.name,
            "scheme": dataclasses.asdict(resolved),
            "dense_remainder": dense_remainder,
            "per_layer_recipe": per_layer_recipe,
            "quantized_inputs": quantized_inputs,
            "tuning": dataclasses.asdict(tuning),
            "calibration": {"source": "zipf(1.1) synthetic token ids", "n_samples": tuning.n_samples,
                            "seq_len": tuning.seq_len,
                            "seed": DEFAULT_SEED if seed is None else seed,
                            "holdout_batches": holdout_batches},
            "mixed": None if plan_info is None else {k: v for k, v in plan_info.items() if k != "describe"},
            "memory_check": None,
            "time_check": None,
            "device": {"name": torch.cuda.get_device_name(device), "world_size": dist.world},
            "result": {
                "blocks": len(summary.blocks), "reverted": summary.reverted,
                "mean_improvement": summary.mean_improvement,
                "total_seconds": summary.total_seconds,
                "peak_memory_bytes": summary.peak_memory_bytes,
                "memory": summary.memory_record(),
                "timing": {**summary.timing_record(),
                           "after_blocks_seconds": {"remainder": remainder_seconds,
                                                    "export": export_seconds}},
                "bits_per_weight": storage.bits_per_weight,
                "stored_bytes": storage.stored_bytes,
                "skipped": [list(s) for s in skipped],
            },
        }
        config_path.write_text(json.dumps(record, indent=2, default=str), encoding="utf-8")
    else:
        storage = _storage(bundle, quantized, dense)
    dist.barrier()
    return QuantizeResult(output_dir=destination, summary=summary,
                          scheme_by_layer=summary.scheme_by_layer, config_path=config_path,
                          storage=storage, skipped=tuple(sorted(skipped)), mixed=plan_info)


def quantize_round_to_nearest(model: str | Path | SyntheticModel, *, output_dir: str | Path,
                              bits: int = 4, group_size: int = 64,
                              symmetry: Symmetry = Symmetry.SYMMETRIC) -> QuantizeResult:
    """Every eligible module rounded to nearest, nothing learned (reference api.py:841)."""
    scheme = QuantScheme(bits=bits, group_size=group_size, symmetry=symmetry)
    _resolve_scheme(bits=bits, group_size=group_size, symmetry=symmetry, average_bits=None,
                    candidate_bits=(), remainder_bits=None, scheme=scheme, scale_init=None)
    require_mlx_representable(scheme)
    device = torch.device("cuda", torch.cuda.current_device())
    bundle = load_model(model)
    quantized: dict[str, QuantizedLayer] = {}
    skipped = []
    for i in range(bundle.arch.layers):
        params = bundle.block(i)
        for path, w in params.linears.items():
            full = f"{bundle.block_name(i)}.{path}"
            if w.shape[1] % group_size:
                skipped.append((full, f"last dimension {w.shape[1]} is not a multiple of {group_size}"))
            else:
                quantized[full] = _rtn_layer(w, scheme, device)
    for path, w in {"model.embed_tokens": bundle.embed_tokens(),
                    **({} if bundle.arch.tied else {"lm_head": bundle.lm_head()})}.items():
        quantized[path] = _rtn_layer(w, scheme, device)
    dense = _dense_tensors(bundle, quantized)
    destination = Path(output_dir)
    export_mlx(destination, dense, quantized, bundle.config())
    storage = _storage(bundle, quantized, dense)
    config_path = destination / "mround_run.json"
    config_path.write_text(json.dumps({"model": bundle.name, "scheme": dataclasses.asdict(scheme),
                                       "round_to_nearest": True}, indent=2, default=str))
    return QuantizeResult(destination, None, {p: q.scheme for p, q in quantized.items()}, config_path,
                          storage, tuple(skipped))

