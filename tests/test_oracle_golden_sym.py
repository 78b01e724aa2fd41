"""The float32 oracle's symmetric, searched and scale-search paths against the
reference NumPy oracle's golden vectors.

Tolerances are the reference's own for a float32 implementation against its
float64 oracle (``tests/unit/test_mlx_parity.py``): scales and reconstructions
2e-5, fewer than 0.1 % of codes differing, gradients 1e-3 max-normalised; the
scale search must pick the same scale in at least 98 % of groups (95 % under
importance weighting, lines 615-670) and, where it does not, reconstruct no
worse.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import quant_fp32, scale_search
from tests.conftest import relative_error

FLOAT32_TOL = 2e-5
GRAD_TOL = 1e-3

SYM_CASES = [f"s{i}_b{b}_g{g}" for i in ("o", "s") for b in (2, 3, 4, 8) for g in (32, 64, 128)]
SEARCH_CASES = [f"srch_b{b}_g{g}" for b in (2, 3, 4, 8) for g in (32, 64)]


def _sym(golden, key):
    bits = int(key.split("_")[1][1:])
    group = int(key.split("_")[2][1:])
    c = {n: golden[f"{key}_{n}"] for n in ("w", "v", "alpha", "beta", "gq", "qdq", "codes",
                                           "scale", "gv", "galpha", "gbeta")}
    c["init"] = golden.get(f"{key}_init")
    return bits, group, c


@pytest.mark.parametrize("key", SYM_CASES)
def test_sym_forward_matches_reference(golden, key):
    bits, group, c = _sym(golden, key)
    qdq, codes, scale, zp = quant_fp32.fake_quantize(
        c["w"], c["v"], c["alpha"], c["beta"], bits, group, symmetric=True, init_scale=c["init"])
    assert zp is None
    assert relative_error(scale, c["scale"]) < FLOAT32_TOL
    half = 1 << (bits - 1)
    assert codes.min() >= -half and codes.max() <= half - 1
    differing = float(np.mean(codes != c["codes"]))
    assert differing < 0.001, f"{differing:.3%} of codes differ"
    same = codes == c["codes"]
    assert relative_error(np.where(same, qdq, 0.0), np.where(same, c["qdq"], 0.0)) < FLOAT32_TOL


@pytest.mark.parametrize("key", SYM_CASES)
def test_sym_gradients_match_reference(golden, key):
    bits, group, c = _sym(golden, key)
    gv, ga, gb = quant_fp32.ste_grads(c["w"], c["v"], c["alpha"], c["beta"], c["gq"], bits, group,
                                      symmetric=True, init_scale=c["init"])
    for name, got, want in (("v", gv, c["gv"]), ("alpha", ga, c["galpha"]), ("beta", gb, c["gbeta"])):
        assert relative_error(got, want) < GRAD_TOL, f"{name}: {relative_error(got, want):.2e}"
    if c["init"] is not None:
        assert not ga.any(), "alpha is inert under a searched scale"
    else:
        # only the dominant side's coefficient receives gradient
        assert not (ga.astype(bool) & gb.astype(bool)).any()


def test_sym_dominant_extreme_reconstructs_exactly():
    # positive side dominates -> negative scale; the extreme lands on -2^(b-1)
    w = np.array([[0.02, -0.01, 0.005, 0.0]], np.float32)
    ones = np.ones((1, 1), np.float32)
    qdq, codes, scale, _ = quant_fp32.fake_quantize(w, np.zeros_like(w), ones, ones, 2, 4,
                                                    symmetric=True)
    assert scale[0, 0] < 0 and codes[0, 0] == -2 and qdq[0, 0] == w[0, 0]


def test_sym_all_zero_group_positive_eps():
    w = np.zeros((1, 8), np.float32)
    ones = np.ones((1, 1), np.float32)
    _, _, scale, _ = quant_fp32.fake_quantize(w, np.zeros_like(w), ones, ones, 4, 8, symmetric=True)
    assert scale[0, 0] == np.float32(1e-8)


@pytest.mark.parametrize("bits,step,half", [(2, 0.01, 90), (3, 0.03, 100), (4, 0.06, 100),
                                            (5, 0.12, 100), (8, 0.96, 100)])
def test_grid_matches_reference_table(bits, step, half):
    got_step, got_half = scale_search.grid_steps(bits)
    assert got_step == pytest.approx(step, abs=1e-12) and got_half == half
    assert len(scale_search.candidates(bits)) == 2 * half + 1
    assert scale_search.grid_steps(4, 0.9)[1] == 99


def _choice_agrees(got, want, w, bits, group, tol_frac):
    same = np.isclose(got, want, rtol=1e-5, atol=1e-8)
    assert same.mean() >= tol_frac, f"only {same.mean():.1%} of groups chose the same scale"
    nmax = float(2 ** (bits - 1))
    grouped = np.asarray(w, np.float64).reshape(-1, group)
    for row in np.flatnonzero(~same.ravel()):
        losses = []
        for s in (float(got.ravel()[row]), float(want.ravel()[row])):
            inv = 0.0 if s == 0 else 1.0 / s
            codes = np.clip(np.rint(inv * grouped[row]), -nmax, nmax - 1)
            losses.append(float(np.sum((s * codes - grouped[row]) ** 2)))
        assert losses[0] <= losses[1] * (1 + 1e-4), (row, losses)


@pytest.mark.parametrize("key", SEARCH_CASES)
def test_search_f64_matches_reference_exactly(golden, key):
    bits, group = int(key.split("_")[1][1:]), int(key.split("_")[2][1:])
    got = scale_search.search_scales_f64(golden[f"{key}_w"], bits, group)
    assert np.array_equal(got, golden[f"{key}_scale"])


@pytest.mark.parametrize("key", SEARCH_CASES)
def test_search_f32_matches_reference(golden, key):
    bits, group = int(key.split("_")[1][1:]), int(key.split("_")[2][1:])
    got = scale_search.search_scales_f32(golden[f"{key}_w"], bits, group)
    _choice_agrees(got, golden[f"{key}_scale"], golden[f"{key}_w"], bits, group, 0.98)


def test_search_importance_matches_reference(golden):
    w, imp = golden["srch_imp_w"], golden["srch_imp_importance"]
    want = golden["srch_imp_scale"]
    assert np.allclose(scale_search.search_scales_f64(w, 3, 16, imp.astype(np.float64)), want,
                       rtol=1e-12, atol=0)
    got = scale_search.search_scales_f32(w, 3, 16, imp)
    assert np.isclose(got, want, rtol=1e-5, atol=1e-8).mean() >= 0.95


@pytest.mark.parametrize("bits", [2, 4])
def test_search_edges(golden, bits):
    w = golden["srch_edge_w"]
    want = golden[f"srch_edge_b{bits}_scale"]
    got = scale_search.search_scales_f32(w, bits, 16)
    assert want[0, 0] == 0.0 and got[0, 0] == 0.0, "an all-zero group returns scale 0"
    assert np.sign(got[2, 0]) == np.sign(want[2, 0]) < 0, "first of a |max| tie anchors"
    assert np.allclose(got, want, rtol=1e-5, atol=1e-8)
