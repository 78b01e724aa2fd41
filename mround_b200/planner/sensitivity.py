"""Sensitivity definitions of the mixed-precision planner (host side).

Restates mround/planner/sensitivity.py: the DeltaLoss definition (190-229;
the device computes it with K6), the exact storage cost (232-268), the budget
an average width implies (297-349), option assembly (352-432) and the rule
that picks where scoring gradients come from (125-156).
"""

from __future__ import annotations

from collections.abc import Mapping

import numpy as np

from mround_b200.exceptions import SchemeError
from mround_b200.planner.allocator import LayerOption
from mround_b200.schemes import QuantScheme

__all__ = [
    "GRADIENT_SOURCES",
    "OWN_WIDTH_FROM_WEIGHTS",
    "SENSITIVITY_BATCH_TOKENS",
    "SENSITIVITY_SAMPLES",
    "SENSITIVITY_SEQ_LEN",
    "delta_loss",
    "gradient_source_for",
    "groups_per_row",
    "mixed_budget_bits",
    "score_layer_options",
    "scoring_batch_size",
    "storage_bits",
]

SENSITIVITY_SAMPLES = 128
SENSITIVITY_SEQ_LEN = 1024
SENSITIVITY_BATCH_TOKENS = 2048
OWN_WIDTH_FROM_WEIGHTS = 2_500_000_000
GRADIENT_SOURCES = ("auto", "own_width", "widest")


def gradient_source_for(requested: str, scored_weights: int) -> str:
    if requested not in GRADIENT_SOURCES:
        raise SchemeError(
            "sensitivity_gradients must be one of "
            f"{', '.join(repr(s) for s in GRADIENT_SOURCES)}, got {requested!r}"
        )
    if requested != "auto":
        return requested
    return "own_width" if int(scored_weights) >= OWN_WIDTH_FROM_WEIGHTS else "widest"


def scoring_batch_size(n_samples: int, seq_len: int, *,
                       budget_tokens: int = SENSITIVITY_BATCH_TOKENS) -> int:
    per_batch = max(1, int(budget_tokens) // max(1, int(seq_len)))
    return max(1, min(int(n_samples), per_batch))


def delta_loss(weight, quantized_weight, gradient) -> float:
    """``sum |g * (Q(W) - W)|`` in float64 (the device form is ``kernels.deltaloss``)."""
    w = np.asarray(weight, dtype=np.float64)
    q = np.asarray(quantized_weight, dtype=np.float64)
    g = np.asarray(gradient, dtype=np.float64)
    if not (w.shape == q.shape == g.shape):
        raise ValueError(f"weight {w.shape}, quantized weight {q.shape}, and gradient {g.shape} "
                         "must share one shape")
    return float(np.sum(np.abs(g * (q - w))))


def groups_per_row(in_features: int, group_size: int) -> int:
    if group_size == -1:
        return 1
    if group_size <= 0 or in_features % group_size:
        raise ValueError(f"in_features {in_features} is not a multiple of group size {group_size}; "
                         "this layer stays dense and has no quantized cost")
    return in_features // group_size


def storage_bits(shape: tuple[int, int], bits: int, group_size: int, *, dtype_bits: int = 16) -> int:
    """Packed codes plus one scale and one bias per group."""
    out_features, in_features = shape
    if out_features <= 0 or in_features <= 0:
        raise ValueError(f"shape must be positive, got {shape}")
    groups = out_features * groups_per_row(in_features, group_size)
    return out_features * in_features * bits + 2 * groups * dtype_bits


def mixed_budget_bits(shapes: Mapping[str, tuple[int, int]], average_bits: float, group_size: int,
                      *, dtype_bits: int = 16) -> int:
    """Element count times the average, plus the exact metadata cost."""
    if not shapes:
        raise ValueError("no layers to budget over")
    if average_bits <= 0:
        raise ValueError(f"average_bits must be positive, got {average_bits}")
    elements = 0
    metadata = 0
    for name, (o, i) in shapes.items():
        if o <= 0 or i <= 0:
            raise ValueError(f"layer {name!r} with shape {(o, i)} cannot be grouped")
        try:
            groups = groups_per_row(i, group_size)
        except ValueError as exc:
            raise ValueError(f"layer {name!r} with shape {(o, i)} cannot be grouped") from exc
        elements += o * i
        metadata += 2 * o * groups * dtype_bits
    return int(elements * average_bits) + metadata


def score_layer_options(scores: Mapping[str, Mapping[int, float]],
                        shapes: Mapping[str, tuple[int, int]], base_scheme: QuantScheme, *,
                        dtype_bits: int = 16) -> dict[str, list[LayerOption]]:
    if set(scores) != set(shapes):
        raise ValueError(
            "scores and shapes must cover the same layers; "
            f"only scored: {sorted(set(scores) - set(shapes))}, "
            f"only shaped: {sorted(set(shapes) - set(scores))}"
        )
    if not scores:
        raise ValueError("no layers to score")
    widths: set[int] | None = None
    for name, per in scores.items():
        if widths is None:
            widths = set(per)
            if not widths:
                raise ValueError(f"layer {name!r} has no scored widths")
        elif set(per) != widths:
            raise ValueError(f"layer {name!r} is scored at widths {sorted(per)} but others at "
                             f"{sorted(widths)}; every layer must come from the same scoring passes")
    options: dict[str, list[LayerOption]] = {}
    for name, per in scores.items():
        cands = []
        for width in sorted(per):
            score = per[width]
            if not np.isfinite(score) or score < 0.0:
                raise ValueError(f"layer {name!r} at {width} bits has invalid score {score!r}")
            o, i = shapes[name]
            cands.append(LayerOption(bits=width,
                                     cost_bits=storage_bits(shapes[name], width,
                                                            base_scheme.group_size,
                                                            dtype_bits=dtype_bits),
                                     delta_loss=score, elements=o * i))
        options[name] = cands
    return options
