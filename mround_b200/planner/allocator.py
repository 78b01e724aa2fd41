"""Exact mixed-precision bit allocation (multiple-choice knapsack), on the host.

Restates ``allocate_bits`` (reference mround/planner/allocator.py:98-194):
dynamic programming over exact integer cumulative costs, Pareto pruning after
each layer, states above the budget dropped, final choice the minimum
``(loss, cost)``.  The plan must be identical to the reference's, including
how ties are broken, so the iteration order follows it: layers in the given
order, options in their given order, a state replaced only by a strictly
smaller loss, pruning in ascending cost keeping strictly decreasing losses.
"""

from __future__ import annotations

import dataclasses
import math

__all__ = ["Allocation", "LayerOption", "allocate_bits"]


@dataclasses.dataclass(frozen=True, slots=True)
class LayerOption:
    bits: int
    cost_bits: int
    delta_loss: float
    elements: int | None = None

    def __post_init__(self) -> None:
        if self.cost_bits < 0:
            raise ValueError(f"cost_bits must be non-negative, got {self.cost_bits}")
        if not math.isfinite(self.delta_loss) or self.delta_loss < 0.0:
            raise ValueError(f"delta_loss must be finite and non-negative, got {self.delta_loss}")
        if self.elements is not None and self.elements <= 0:
            raise ValueError(f"elements must be positive when given, got {self.elements}")


@dataclasses.dataclass(frozen=True, slots=True)
class Allocation:
    by_layer: dict[str, int]
    total_cost_bits: int
    predicted_loss: float
    average_bits: float


def allocate_bits(options: dict[str, list[LayerOption]], *, budget_bits: int,
                  max_states: int | None = None) -> Allocation:
    """One width per layer minimising summed predicted loss under ``budget_bits``."""
    if not options:
        raise ValueError("no layers to allocate")
    for name, cands in options.items():
        if not cands:
            raise ValueError(f"layer {name!r} has no candidate bit widths")
    if max_states is not None and max_states < 1:
        raise ValueError(f"max_states must be positive or None, got {max_states}")
    names = list(options)
    cheapest = sum(min(o.cost_bits for o in options[n]) for n in names)
    if cheapest > budget_bits:
        raise ValueError(
            f"budget of {budget_bits} bits is infeasible: the cheapest possible allocation "
            f"costs {cheapest} bits"
        )
    # cost -> (loss, widths chosen so far)
    states: dict[int, tuple[float, tuple[int, ...]]] = {0: (0.0, ())}
    for name in names:
        grown: dict[int, tuple[float, tuple[int, ...]]] = {}
        for cost, (loss, chosen) in states.items():
            for opt in options[name]:
                c = cost + opt.cost_bits
                if c > budget_bits:
                    continue
                l_new = loss + opt.delta_loss
                have = grown.get(c)
                if have is None or l_new < have[0]:
                    grown[c] = (l_new, (*chosen, opt.bits))
        if not grown:
            raise ValueError(f"no feasible allocation remains after layer {name!r}")
        states = _pareto(grown)
        if max_states is not None:
            states = _subsample(states, max_states)
    _, (best_loss, best) = min(states.items(), key=lambda kv: (kv[1][0], kv[0]))
    by_layer = dict(zip(names, best, strict=True))
    total = sum(next(o.cost_bits for o in options[n] if o.bits == by_layer[n]) for n in names)
    return Allocation(by_layer, total, best_loss, _average(options, by_layer))


def _pareto(states):
    kept, floor = {}, math.inf
    for cost in sorted(states):
        loss, chosen = states[cost]
        if loss < floor:
            kept[cost] = (loss, chosen)
            floor = loss
    return kept


def _subsample(states, max_states):
    if len(states) <= max_states:
        return states
    costs = sorted(states)
    if max_states == 1:
        picked = [costs[0]]
    else:
        step = (len(costs) - 1) / (max_states - 1)
        picked = sorted({costs[round(i * step)] for i in range(max_states)})
    return {c: states[c] for c in picked}


def _average(options, by_layer) -> float:
    bits_sum = 0.0
    elems = 0.0
    for name, bits in by_layer.items():
        opt = next(o for o in options[name] if o.bits == bits)
        if opt.elements is not None:
            e = float(opt.elements)
            bits_sum += bits * e
        else:
            e = opt.cost_bits / bits if bits else 0.0
            bits_sum += opt.cost_bits
        elems += e
    return bits_sum / elems if elems else 0.0
