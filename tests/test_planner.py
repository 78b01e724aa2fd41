"""Planner: the exact allocator reproduces the reference's plans (golden), and
the sensitivity definitions hold their documented properties (reference
tests/unit/test_allocator.py:90-231, tests/unit/test_sensitivity.py:42-237)."""

from __future__ import annotations

import itertools
import json

import numpy as np
import pytest

from mround_b200.planner.allocator import LayerOption, allocate_bits
from mround_b200.planner.sensitivity import (
    delta_loss,
    gradient_source_for,
    mixed_budget_bits,
    score_layer_options,
    scoring_batch_size,
    storage_bits,
)
from mround_b200.schemes import QuantScheme
from tests.conftest import GOLDEN

CASES = json.loads((GOLDEN / "allocations.json").read_text())


@pytest.mark.parametrize("case", range(len(CASES)))
def test_identical_plan_to_reference(case):
    c = CASES[case]
    shapes = {k: tuple(v) for k, v in c["shapes"].items()}
    scores = {k: {int(b): s for b, s in v.items()} for k, v in c["scores"].items()}
    scheme = QuantScheme(bits=4, group_size=c["group_size"], symmetry="asym")
    budget = mixed_budget_bits(shapes, c["average_bits"], c["group_size"])
    assert budget == c["budget_bits"]
    alloc = allocate_bits(score_layer_options(scores, shapes, scheme), budget_bits=budget)
    assert alloc.by_layer == c["by_layer"]
    assert alloc.total_cost_bits == c["total_cost_bits"]
    assert alloc.predicted_loss == c["predicted_loss"]
    assert alloc.average_bits == c["average"]


def test_exact_against_exhaustive_search():
    rng = np.random.default_rng(0)
    for _ in range(20):
        n = 6
        options = {f"l{i}": [LayerOption(b, int(rng.integers(100, 400)) * b, float(rng.random() * (5 - b)))
                             for b in (2, 3, 4)] for i in range(n)}
        budget = int(sum(min(o.cost_bits for o in opts) for opts in options.values()) * 1.4)
        best = None
        for combo in itertools.product(*[options[f"l{i}"] for i in range(n)]):
            cost = sum(o.cost_bits for o in combo)
            if cost <= budget:
                loss = sum(o.delta_loss for o in combo)
                if best is None or loss < best - 1e-12:
                    best = loss
        got = allocate_bits(options, budget_bits=budget)
        assert got.predicted_loss == pytest.approx(best, abs=1e-9)
        assert got.total_cost_bits <= budget


def test_infeasible_budget_is_refused():
    opts = {"a": [LayerOption(2, 100, 1.0)]}
    with pytest.raises(ValueError, match="infeasible"):
        allocate_bits(opts, budget_bits=99)


def test_integer_average_budget_equals_uniform_storage():
    shapes = {"a": (64, 128), "b": (32, 192)}
    for bits in (2, 3, 4):
        assert mixed_budget_bits(shapes, bits, 64) == sum(storage_bits(s, bits, 64) for s in shapes.values())


def test_delta_loss_hand_computed():
    w = np.array([[1.0, -2.0]])
    q = np.array([[1.5, -1.0]])
    g = np.array([[2.0, -3.0]])
    assert delta_loss(w, q, g) == 2.0 * 0.5 + 3.0 * 1.0


def test_gradient_source_rule():
    assert gradient_source_for("auto", 2_775_000_000) == "own_width"
    assert gradient_source_for("auto", 358_000_000) == "widest"
    assert gradient_source_for("widest", 10**10) == "widest"
    with pytest.raises(ValueError):
        gradient_source_for("bogus", 1)


def test_scoring_batch_size():
    assert scoring_batch_size(128, 1024) == 2
    assert scoring_batch_size(128, 2048) == 1
    assert scoring_batch_size(1, 16) == 1
