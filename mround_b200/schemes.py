"""Quantization schemes and the tuning recipe.

These two frozen dataclasses are the drop-in surface shared with MRound: same
field names, defaults, validation and derived properties as the reference's
``mround/schemes.py:90-337`` (``QuantScheme`` 90-211, ``TuningConfig``
214-337), restated here so that a caller constructing either object gets the
same answers and the same refusals.  Nothing here knows about devices.
"""

from __future__ import annotations

import dataclasses
from enum import StrEnum
from typing import Self

from mround_b200.exceptions import SchemeError

__all__ = [
    "DEFAULT_EPS_FP32",
    "DEFAULT_EPS_LOW_PRECISION",
    "LONG_BUDGET_ITERS",
    "LOW_BIT_THRESHOLD",
    "SUPPORTED_BITS",
    "QuantScheme",
    "ScaleInit",
    "Symmetry",
    "TuningConfig",
]

#: Widths the uint32 packing handles (reference ``schemes.py:39``).
SUPPORTED_BITS: frozenset[int] = frozenset({2, 3, 4, 5, 6, 7, 8})

#: Below this width the outlier rule switches on by default and, at long
#: budgets, the learning-rate constant doubles (reference ``schemes.py:46``).
LOW_BIT_THRESHOLD: int = 4

#: Step budget from which narrow widths start at twice the rate
#: (reference ``schemes.py:52``).
LONG_BUDGET_ITERS: int = 1000

#: Scale epsilon guarding all-zero groups (reference ``schemes.py:55-56``).
DEFAULT_EPS_FP32: float = 1e-8
DEFAULT_EPS_LOW_PRECISION: float = 1e-5


class Symmetry(StrEnum):
    """Signed (``sym``) or unsigned-with-zero-point (``asym``) code range."""

    SYMMETRIC = "sym"
    ASYMMETRIC = "asym"


class ScaleInit(StrEnum):
    """Where the per-group scale starts: observed extremes, or the v2 search."""

    OBSERVED_RANGE = "observed_range"
    SEARCHED = "searched"


@dataclasses.dataclass(frozen=True, slots=True)
class QuantScheme:
    """Target representation of one layer's weights.

    Attributes:
        bits: Code width, one of :data:`SUPPORTED_BITS`.
        group_size: Weights per scale along the input axis; ``-1`` is one
            group per output channel.
        symmetry: Code range.
        scale_init: Scale parameterization.
    """

    bits: int = 4
    group_size: int = 64
    symmetry: Symmetry = Symmetry.SYMMETRIC
    scale_init: ScaleInit = ScaleInit.OBSERVED_RANGE

    def __post_init__(self) -> None:
        # Strings are coerced to the enum members because every consumer
        # compares with ``is``.
        object.__setattr__(self, "symmetry", Symmetry(self.symmetry))
        object.__setattr__(self, "scale_init", ScaleInit(self.scale_init))
        if self.bits not in SUPPORTED_BITS:
            allowed = ", ".join(str(b) for b in sorted(SUPPORTED_BITS))
            raise SchemeError(f"bits must be one of {{{allowed}}}, got {self.bits}")
        if self.group_size != -1 and self.group_size <= 0:
            raise SchemeError(
                f"group_size must be positive or -1 (per-channel), got {self.group_size}"
            )
        if self.scale_init is ScaleInit.SEARCHED and self.symmetry is not Symmetry.SYMMETRIC:
            raise SchemeError(
                "the searched scale initialization is defined for symmetric schemes only"
            )

    @property
    def is_per_channel(self) -> bool:
        """True when one scale covers a whole output row."""
        return self.group_size == -1

    @property
    def packs_evenly(self) -> bool:
        """True when codes tile a 32-bit word (2, 4, 8 bits)."""
        return 32 % self.bits == 0

    @property
    def code_range(self) -> tuple[int, int]:
        """Inclusive integer code range before any storage offset."""
        if self.symmetry is Symmetry.SYMMETRIC:
            half = 1 << (self.bits - 1)
            return (-half, half - 1)
        return (0, (1 << self.bits) - 1)

    @property
    def coefficient_bounds(self) -> tuple[float, float]:
        """Projection interval of the clipping coefficients alpha and beta."""
        if self.scale_init is ScaleInit.SEARCHED:
            return (0.5, 1.5)
        return (0.1, 1.0)

    def groups_per_row(self, in_features: int) -> int:
        """Scales per output row; refuses an input width that is not whole groups."""
        if self.is_per_channel:
            return 1
        if in_features % self.group_size:
            raise SchemeError(
                f"in_features={in_features} is not divisible by group_size={self.group_size}"
            )
        return in_features // self.group_size

    def with_bits(self, bits: int) -> Self:
        """The same scheme at another width."""
        return dataclasses.replace(self, bits=bits)


@dataclasses.dataclass(frozen=True, slots=True)
class TuningConfig:
    """The signSGD recipe (standard recipe: 200 steps, batch 8, 128 x 2048).

    Attributes mirror the reference one for one; ``minmax_lr`` and
    ``gradient_accumulate_steps`` are refused unless left at their inert
    values, as the reference refuses them.
    """

    iters: int = 200
    batch_size: int = 8
    n_samples: int = 128
    seq_len: int = 2048
    lr: float | None = None
    minmax_lr: float | None = None
    gradient_accumulate_steps: int = 1
    suppress_outliers: bool | None = None
    micro_batches: int = 1

    def __post_init__(self) -> None:
        if self.iters <= 0:
            raise SchemeError(f"iters must be positive, got {self.iters}")
        if self.batch_size <= 0:
            raise SchemeError(f"batch_size must be positive, got {self.batch_size}")
        if self.n_samples < self.batch_size:
            raise SchemeError(
                f"n_samples={self.n_samples} is smaller than batch_size={self.batch_size}"
            )
        if self.minmax_lr is not None:
            raise SchemeError(
                "minmax_lr is not implemented: the clipping coefficients share lr"
            )
        if self.gradient_accumulate_steps != 1:
            raise SchemeError(
                "gradient_accumulate_steps other than 1 is not implemented, got "
                f"{self.gradient_accumulate_steps}"
            )
        if not 1 <= self.micro_batches <= self.batch_size:
            raise SchemeError(
                f"micro_batches must be between 1 and batch_size={self.batch_size}, "
                f"got {self.micro_batches}"
            )

    def resolved_lr(self, bits: int) -> float:
        """Initial rate: the explicit ``lr`` or ``c / iters`` (c = 2 only for
        narrow widths at budgets of 1000 steps or more)."""
        if self.lr is not None:
            return self.lr
        doubled = bits < LOW_BIT_THRESHOLD and self.iters >= LONG_BUDGET_ITERS
        return (2.0 if doubled else 1.0) / self.iters

    def resolved_minmax_lr(self, bits: int) -> float:
        """Rate of the clipping coefficients (always the main rate)."""
        if self.minmax_lr is not None:
            return self.minmax_lr
        return self.resolved_lr(bits)

    def resolved_suppress_outliers(self, bits: int) -> bool:
        """Outlier rule: explicit setting, else on below 4 bits."""
        if self.suppress_outliers is not None:
            return self.suppress_outliers
        return bits < LOW_BIT_THRESHOLD
