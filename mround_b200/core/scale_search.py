"""The v2 candidate scale grid search on the device (K8).

Same entry point and candidate family as the reference's
``mround/core/scale_search.py:73-126`` (NumPy oracle
``mround/reference/scale_search.py:78-211``): per group the signed
largest-magnitude element is mapped onto ``-eff`` for ``eff`` in
``[nmax] + [nmax - step * i for i in -half..half, i != 0]`` and the first
candidate with the strictly smallest (importance-weighted) squared
reconstruction error is kept.  ``SearchGrid.steps`` is the reference's table:
180 candidates at step 0.01 around ``nmax = 2`` for 2 bits, otherwise
``step = 2 * nmax * ratio / 200`` and ``half = int(nmax * ratio / step)``.

The whole matrix is one launch: every group's search is independent and held
in registers, so there is no candidate chunking or row slicing to bound
memory.  Losses accumulate in float32, as the reference's MLX port does.
"""

from __future__ import annotations

import dataclasses

import torch

from mround_b200 import kernels
from mround_b200.exceptions import SchemeError
from mround_b200.schemes import QuantScheme, Symmetry

__all__ = ["SearchGrid", "candidates", "search_scales"]

_TWO_BIT_STEP = 0.01
_TWO_BIT_HALF_COUNT = 90
_GRID = 200


@dataclasses.dataclass(frozen=True, slots=True)
class SearchGrid:
    """The candidate family as perturbations of the effective code range.

    ``ratio`` is the span as a fraction of ``nmax``
    (reference ``mround/reference/scale_search.py:78-105``).
    """

    ratio: float = 0.75

    def steps(self, bits: int) -> tuple[float, int]:
        """``(step, half_count)`` for ``bits``."""
        if bits == 2:
            return _TWO_BIT_STEP, _TWO_BIT_HALF_COUNT
        nmax = float(2 ** (bits - 1))
        span = nmax * self.ratio
        step = span / _GRID * 2
        return step, int(span / step)


def candidates(bits: int, grid: SearchGrid | None = None) -> list[float]:
    """Effective ranges in evaluation order, the anchor ``2**(bits-1)`` first."""
    nmax = float(2 ** (bits - 1))
    step, half = (grid or SearchGrid()).steps(bits)
    return [nmax] + [nmax - step * i for i in range(-half, half + 1) if i != 0]


def search_scales(weight: torch.Tensor, scheme: QuantScheme, *,
                  importance: torch.Tensor | None = None, grid: SearchGrid | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """One signed scale per group, ``(n_groups, 1)`` float32, row-major groups.

    ``weight`` is the bf16 ``(out_features, in_features)`` matrix on the GPU;
    ``importance`` a per-input-channel float32 weighting (only relative values
    matter).  An all-zero group yields 0, which the quantizer clamps to eps.
    ``out`` (float32, ``(rows, in_features // group)``) receives the result
    when given.

    Raises:
        SchemeError: the scheme is not symmetric, or the weight does not group.
    """
    if scheme.symmetry is not Symmetry.SYMMETRIC:
        raise SchemeError("the searched initialization is defined for symmetric schemes only")
    if weight.dim() != 2 or weight.shape[-1] % scheme.group_size:
        raise SchemeError(
            f"search expects a 2-D weight whose last dimension is a multiple of "
            f"group_size={scheme.group_size}, got shape {tuple(weight.shape)}")
    if importance is not None:
        importance = importance.to(device=weight.device, dtype=torch.float32).reshape(-1).contiguous()
        if importance.numel() != weight.shape[-1]:
            raise SchemeError(f"importance has {importance.numel()} channels but the weight has "
                              f"{weight.shape[-1]} input features")
    w = weight.to(torch.bfloat16).contiguous()
    res = kernels.scale_search(w, bits=scheme.bits, group=scheme.group_size,
                               candidates=candidates(scheme.bits, grid), importance=importance,
                               out=out)
    return res.reshape(-1, 1) if out is None else res
