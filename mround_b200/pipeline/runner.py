"""Block-by-block quantization on B200: the reference runner's semantics.

Restates ``QuantizationRunner`` (reference mround/pipeline/runner.py:428-953):

- two activation streams: targets from the original block applied to the
  reference stream (written in place), the quantized stream advanced through
  each committed block (``run`` 493-605);
- per block: wrap the linears, score the untuned rounding (mean loss over the
  scoring batches), ``iters`` signed steps cycling ``step % n_batches``,
  score again, revert to the untuned rounding if not improved, commit, and
  advance (``quantize_block`` 607-710, ``_tune`` 790-953);
- the recipe of ``block_recipe`` (389-425): outlier rule and learning rate
  from the run's base width (or per layer);
- ``BlockResult`` / ``RunSummary`` carry the same fields and progress lines.

Device layout: the streams live in HBM as float32 ``(batch_shard, seq, hidden)``
tensors, one per calibration batch; under data parallelism each rank holds its
shard of every batch (``DistContext.shard``).
"""

from __future__ import annotations

import dataclasses
import time
from collections.abc import Callable, Mapping, Sequence
from concurrent.futures import ThreadPoolExecutor
from typing import Any

import torch

from mround_b200.exceptions import ArchitectureError, CalibrationError, ResumeError
from mround_b200.pipeline.block import TUNING_PRECISION, DeviceBlock, Precision
from mround_b200.pipeline.dist import DistContext
from mround_b200.pipeline.model import SyntheticModel
from mround_b200.pipeline.resume import ResumeStore
from mround_b200.pipeline.tuning import BlockTuner, QuantizedLayer
from mround_b200.schemes import DEFAULT_EPS_FP32, QuantScheme, TuningConfig

__all__ = ["BlockResult", "QuantizationRunner", "RunSummary", "block_recipe"]


@dataclasses.dataclass(frozen=True, slots=True)
class BlockResult:
    index: int
    name: str
    initial_loss: float
    final_loss: float
    iterations: int
    seconds: float
    peak_memory_bytes: int
    tuned: tuple[str, ...] = ()
    skipped: tuple[tuple[str, str], ...] = ()
    reverted: bool = False
    generalization_gap: float | None = None
    search_seconds: float = 0.0
    stage_peaks: dict[str, int] = dataclasses.field(default_factory=dict)
    step_seconds: float = 0.0

    @property
    def improvement(self) -> float:
        if self.initial_loss <= 0.0:
            return 0.0
        return 1.0 - (self.final_loss / self.initial_loss)

    def describe(self) -> str:
        note = "  reverted to its untuned rounding" if self.reverted else ""
        if self.stage_peaks:
            stage = max(self.stage_peaks, key=self.stage_peaks.__getitem__)
            note = f"  peak {self.stage_peaks[stage] / 1e9:.2f} GB in {stage}{note}"
        if self.generalization_gap is not None:
            note = f"  gap {self.generalization_gap:+.1%}{note}"
        return (
            f"block {self.index:>3} {self.name:<24} "
            f"loss {self.initial_loss:.4e} to {self.final_loss:.4e} "
            f"({self.improvement:+.1%}) in {self.seconds:.1f}s{note}"
        )


@dataclasses.dataclass(frozen=True, slots=True)
class RunSummary:
    blocks: list[BlockResult]
    total_seconds: float
    peak_memory_bytes: int
    scheme_by_layer: dict[str, QuantScheme]
    before_blocks: dict[str, int] = dataclasses.field(default_factory=dict)
    after_blocks: dict[str, int] = dataclasses.field(default_factory=dict)

    @property
    def mean_improvement(self) -> float:
        if not self.blocks:
            return 0.0
        return sum(b.improvement for b in self.blocks) / len(self.blocks)

    @property
    def reverted(self) -> int:
        return sum(1 for b in self.blocks if b.reverted)

    @property
    def mean_generalization_gap(self) -> float | None:
        gaps = [b.generalization_gap for b in self.blocks if b.generalization_gap is not None]
        return sum(gaps) / len(gaps) if gaps else None

    def stage_peaks(self) -> dict[str, int]:
        peaks = dict(self.before_blocks)
        for block in self.blocks:
            for stage, reached in block.stage_peaks.items():
                peaks[stage] = max(peaks.get(stage, 0), reached)
        for stage, reached in self.after_blocks.items():
            peaks[stage] = max(peaks.get(stage, 0), reached)
        return peaks

    def memory_record(self) -> dict[str, Any]:
        return {
            "peak_bytes": self.peak_memory_bytes,
            "by_stage_bytes": self.stage_peaks(),
            "by_block_bytes": [{"block": b.index, **b.stage_peaks} for b in self.blocks],
        }

    def timing_record(self) -> dict[str, Any]:
        blocks = sum(b.seconds for b in self.blocks)
        return {
            "loop_seconds": self.total_seconds,
            "between_blocks_seconds": self.total_seconds - blocks,
            "by_block": [{"block": b.index, "seconds": b.seconds, "search_seconds": b.search_seconds}
                         for b in self.blocks],
        }

    def describe(self) -> str:
        note = f", {self.reverted} reverted" if self.reverted else ""
        gap = self.mean_generalization_gap
        if gap is not None:
            note = f"{note}, mean gap {gap:+.1%}"
        return (
            f"{len(self.blocks)} blocks tuned in {self.total_seconds:.1f}s, "
            f"mean loss reduction {self.mean_improvement:+.1%}{note}, "
            f"peak memory {self.peak_memory_bytes / 1e9:.2f} GB"
        )


def block_recipe(tuning: TuningConfig, base_bits: int, widths: Mapping[str, int], *,
                 per_layer: bool) -> tuple[bool, dict[str, float]]:
    """Outlier rule and per-layer initial rates (reference runner.py:389-425)."""
    if not per_layer:
        rate = tuning.resolved_lr(base_bits)
        return tuning.resolved_suppress_outliers(base_bits), dict.fromkeys(widths, rate)
    narrowest = min(widths.values(), default=base_bits)
    return tuning.resolved_suppress_outliers(narrowest), {
        name: tuning.resolved_lr(bits) for name, bits in widths.items()
    }


class _Meter:
    """Per-stage peak device memory (reference mround/pipeline/device.py:94-135)."""

    def __init__(self, device) -> None:
        self.device = device
        self.stages: dict[str, int] = {}
        self.peak = 0

    def stage(self, name: str):
        meter = self

        class _Ctx:
            def __enter__(self_inner):
                torch.cuda.reset_peak_memory_stats(meter.device)

            def __exit__(self_inner, *exc):
                reached = torch.cuda.max_memory_allocated(meter.device)
                meter.stages[name] = max(meter.stages.get(name, 0), reached)
                meter.peak = max(meter.peak, reached)
                return False

        return _Ctx()

    def take(self) -> dict[str, int]:
        out, self.stages = self.stages, {}
        return out


class QuantizationRunner:
    """Walks a model block by block on the GPU, quantizing each in turn."""

    def __init__(self, scheme: QuantScheme, tuning: TuningConfig, *,
                 progress: Callable[[BlockResult], None] | None = None,
                 eps: float = DEFAULT_EPS_FP32, quantized_inputs: bool = True,
                 holdout_batches: int = 0, per_layer_recipe: bool = False,
                 precision: Precision | None = None, dist: DistContext | None = None,
                 device: torch.device | str | None = None, keep_codes: bool = False,
                 exchange: str = "auto", gather: str = "codes") -> None:
        """``exchange``: the data-parallel weight-gradient exchange of the
        row-sharded update -- "p2p" (GEMM epilogue stores into the owners'
        memory over NVLink), "copy" (copy engines), "nccl" (reduce-scatter)
        or "auto" (by rank count, as measured); ``gather``: what the ranks
        all-gather after the step -- "codes" (codes and per-group scale /
        zero point) or "operands"; see
        :class:`~mround_b200.pipeline.tuning.BlockTuner`."""
        if holdout_batches < 0:
            raise CalibrationError(f"holdout_batches must be zero or more, got {holdout_batches}")
        self.scheme = scheme
        self.tuning = tuning
        self.progress = progress
        self.eps = eps
        self.quantized_inputs = quantized_inputs
        self.holdout_batches = holdout_batches
        self.per_layer_recipe = per_layer_recipe
        self.precision = precision or TUNING_PRECISION
        self.dist = dist or DistContext()
        self.device = torch.device(device or "cuda")
        self.keep_codes = keep_codes
        self.exchange = exchange
        self.gather = gather

    def _scheme_for(self, path: str, overrides: Mapping[str, QuantScheme] | None) -> QuantScheme:
        if overrides is None:
            return self.scheme
        return overrides.get(path, self.scheme)

    # ------------------------------------------------------------------ entrance
    def entrance(self, model: SyntheticModel, batches: Sequence[Any]) -> list[torch.Tensor]:
        """Block-0 inputs of this rank's shard: the embedding rows, float32.

        The reference captures them by running the model to block 0
        (mround/pipeline/blocks.py:444-533); for an mlx-lm decoder that input is
        the token embedding, widened to float32 (runner.py:531).
        """
        embed = model.embed_tokens().to(self.device)
        out = []
        for batch in batches:
            tokens = torch.as_tensor(batch, dtype=torch.long)
            rows = self.dist.shard(tokens.shape[0])
            ids = tokens[rows].to(self.device)
            out.append(embed[ids].float().contiguous())
        return out

    # ------------------------------------------------------------------ run
    def run(self, model: SyntheticModel, calibration_batches: Sequence[Any], *,
            scheme_by_layer: Mapping[str, QuantScheme] | None = None,
            expected_blocks: int | None = None, blocks: Sequence[int] | None = None,
            resume: ResumeStore | None = None,
            ) -> tuple[RunSummary, dict[str, QuantizedLayer]]:
        """Quantize the model's blocks in order.  With ``resume``, blocks that
        an earlier run with the same fingerprint finished are loaded instead
        of tuned (a leading run of them; the first block without a record and
        every later one are tuned), and each newly tuned block is recorded."""
        started = time.perf_counter()
        meter = _Meter(self.device)
        n_blocks = model.arch.layers
        if expected_blocks is not None and expected_blocks != n_blocks:
            raise ArchitectureError(f"found {n_blocks} blocks but the configuration says {expected_blocks}")
        indices = list(range(n_blocks)) if blocks is None else list(blocks)
        with meter.stage("entrance"):
            reference_stream = self.entrance(model, calibration_batches)
        before_blocks = meter.take()
        quantized_stream = [t.clone() for t in reference_stream] if self.quantized_inputs else None
        resuming = resume is not None
        # The next block's host weights (synthesised or read from the
        # checkpoint) are produced on a worker thread while this block tunes;
        # torch and numpy release the GIL in that work, and an error surfaces
        # when its block is reached, as it would without the prefetch.
        prefetch = ThreadPoolExecutor(max_workers=1, thread_name_prefix="mround-block-prefetch")
        upcoming = prefetch.submit(model.block, indices[0]) if indices else None
        try:
            results, exported, schemes = self._walk(
                model, indices, prefetch, upcoming, meter, reference_stream, quantized_stream,
                scheme_by_layer, resume, resuming)
        finally:
            prefetch.shutdown(wait=True, cancel_futures=True)
        total = time.perf_counter() - started
        return (
            RunSummary(blocks=results, total_seconds=total, peak_memory_bytes=meter.peak,
                       scheme_by_layer=schemes, before_blocks=before_blocks),
            exported,
        )

    def _walk(self, model, indices, prefetch, upcoming, meter, reference_stream,
              quantized_stream, scheme_by_layer, resume, resuming):
        """The block loop of ``run``."""
        results: list[BlockResult] = []
        exported: dict[str, QuantizedLayer] = {}
        schemes: dict[str, QuantScheme] = {}
        for pos, index in enumerate(indices):
            params = upcoming.result()
            if pos + 1 < len(indices):
                upcoming = prefetch.submit(model.block, indices[pos + 1])
            block = DeviceBlock(model.arch, params, self.device)
            del params
            name = model.block_name(index)
            # every rank takes the same decision, even if one sees the file late
            resuming = resuming and self.dist.max_scalar(0.0 if resume.has(index) else 1.0,
                                                         self.device) == 0.0
            with meter.stage("targets"):
                with torch.no_grad():
                    if quantized_stream is not None:
                        for i, x in enumerate(reference_stream):
                            reference_stream[i] = block.forward_fused(x, self.precision, False)[0]
                        targets = reference_stream
                    else:
                        targets = [block.forward_fused(x, self.precision, False)[0]
                                   for x in reference_stream]
            inputs = quantized_stream if quantized_stream is not None else reference_stream
            if resuming:
                result, layers = self._restore_block(block, resume, index)
            else:
                result, layers = self.quantize_block(block, name, inputs, targets,
                                                     scheme_by_layer=scheme_by_layer, meter=meter)
            exported.update(layers)
            for path in layers:
                schemes[path] = self._scheme_for(path, scheme_by_layer)
            with meter.stage("advance"):
                if quantized_stream is not None:
                    with torch.no_grad():
                        for i, x in enumerate(quantized_stream):
                            quantized_stream[i] = block.forward_fused(x, self.precision, False)[0]
            if quantized_stream is None:
                reference_stream = targets
            if not resuming:
                result = dataclasses.replace(result, peak_memory_bytes=meter.peak,
                                             stage_peaks=meter.take())
                if resume is not None:
                    resume.save(index, result, layers,
                                {n: l.wq_hi for n, l in block.layers.items() if l.wq_hi is not l.w})
            else:
                meter.take()
            del block
            results.append(result)
            if self.progress is not None and self.dist.rank == 0:
                self.progress(result)
        return results, exported, schemes

    def _restore_block(self, block: DeviceBlock, resume: ResumeStore,
                       index: int) -> tuple[BlockResult, dict[str, QuantizedLayer]]:
        """A finished block from ``resume``: its committed bf16 weights become
        the block's operands (so the quantized stream advances exactly as it
        did), its stored layers and result are returned as tuned ones."""
        stored = resume.load(index)
        for lname, weight in stored.committed.items():
            if lname not in block.layers:
                raise ResumeError(f"{resume.path(index)} holds a weight {lname!r} this block lacks")
            layer = block.layers[lname]
            if tuple(weight.shape) != tuple(layer.w.shape) or weight.dtype != layer.w.dtype:
                raise ResumeError(f"{resume.path(index)}: {lname} is {tuple(weight.shape)} "
                                  f"{weight.dtype}, the block's is {tuple(layer.w.shape)} {layer.w.dtype}")
            layer.wq_hi, layer.wq_lo, layer.grad = weight.to(self.device), None, None
        f = dict(stored.result)
        f["tuned"] = tuple(f.get("tuned", ()))
        f["skipped"] = tuple(tuple(x) for x in f.get("skipped", ()))
        f["stage_peaks"] = dict(f.get("stage_peaks") or {})
        return BlockResult(**f), ResumeStore.quantized_layers(stored, QuantizedLayer)

    # ------------------------------------------------------------------ block
    def tuner_for(self, block: DeviceBlock, name: str,
                  scheme_by_layer: Mapping[str, QuantScheme] | None = None) -> BlockTuner:
        schemes = {p: self._scheme_for(f"{name}.{p}", scheme_by_layer) for p in block.member_paths()}
        suppress, rates = block_recipe(self.tuning, self.scheme.bits,
                                       {p: s.bits for p, s in schemes.items()},
                                       per_layer=self.per_layer_recipe)
        return BlockTuner(block, schemes, rates, suppress=suppress, eps=self.eps,
                          precision=self.precision, dist=self.dist,
                          pieces=self.tuning.micro_batches, exchange=self.exchange,
                          gather=self.gather)

    def quantize_block(self, block: DeviceBlock, name: str, inputs: list[torch.Tensor],
                       targets: list[torch.Tensor], *,
                       scheme_by_layer: Mapping[str, QuantScheme] | None = None,
                       meter: _Meter | None = None) -> tuple[BlockResult, dict[str, QuantizedLayer]]:
        started = time.perf_counter()
        meter = meter or _Meter(self.device)
        tuner = self.tuner_for(block, name, scheme_by_layer)
        if not tuner.tunables:
            reasons = "; ".join(f"{p}: {why}" for p, why in tuner.skipped)
            raise ArchitectureError(f"nothing in {name!r} can be quantized at this group size. {reasons}")
        with meter.stage("search"):
            search_seconds = tuner.search(inputs)
        outcome = self._tune(tuner, inputs, targets, meter)
        with meter.stage("commit"):
            layers = tuner.commit(self.keep_codes)
        torch.cuda.synchronize(self.device)
        tuner.close()
        exported = {f"{name}.{p}": q for p, q in layers.items()}
        result = BlockResult(
            index=block.index, name=name, initial_loss=outcome["initial"],
            final_loss=outcome["final"], iterations=self.tuning.iters,
            seconds=time.perf_counter() - started, peak_memory_bytes=meter.peak,
            stage_peaks=dict(meter.stages),
            tuned=tuple(sorted(m.path for t in tuner.tunables for m in t.members)),
            skipped=tuple(tuner.skipped), reverted=outcome["reverted"],
            generalization_gap=outcome["gap"], step_seconds=outcome["step_seconds"],
            search_seconds=search_seconds)
        return result, exported

    def _tune(self, tuner: BlockTuner, inputs, targets, meter: _Meter) -> dict[str, Any]:
        n_batches = len(inputs)
        held = min(self.holdout_batches, n_batches - 1)
        tuning_batches = list(range(n_batches - held))
        scoring_batches = list(range(n_batches - held, n_batches)) if held else tuning_batches
        iters = self.tuning.iters
        with meter.stage("score"):
            initial = tuner.mean_loss(inputs, targets, scoring_batches)
            initial_tuning = tuner.mean_loss(inputs, targets, tuning_batches) if held else initial
        torch.cuda.synchronize(self.device)
        t0 = time.perf_counter()
        with meter.stage("tune"):
            for step in range(iters):
                b = tuning_batches[step % len(tuning_batches)]
                tuner.step(inputs[b], targets[b], step, iters)
            torch.cuda.synchronize(self.device)
        step_seconds = time.perf_counter() - t0
        with meter.stage("score"):
            final = tuner.mean_loss(inputs, targets, scoring_batches)
            final_tuning = tuner.mean_loss(inputs, targets, tuning_batches) if held else final
        gap = None
        if held:
            gap = (1.0 - final_tuning / initial_tuning) - (1.0 - final / initial)
        if final >= initial:
            tuner.reset()
            return {"initial": initial, "final": initial, "reverted": True, "gap": gap,
                    "step_seconds": step_seconds}
        return {"initial": initial, "final": final, "reverted": False, "gap": gap,
                "step_seconds": step_seconds}
