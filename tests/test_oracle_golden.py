"""The float32 oracle against the reference NumPy oracle's golden vectors.

Tolerances are the reference's own for a float32 implementation against its
float64 oracle (``tests/unit/test_mlx_parity.py``): 2e-5 on scales and
reconstructions (line 58), zero points exactly (175-193), fewer than 0.1 % of
codes differing (213-234), gradients within 1e-3 max-normalised (264-311).
Packing is bit-exact; the allocation is identical.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from oracle import deltaloss, losses_fp32, packing, quant_fp32
from tests.conftest import GOLDEN, relative_error

FLOAT32_TOL = 2e-5
GRAD_TOL = 1e-3

CASES = [f"q_b{b}_g{g}" for b in (2, 3, 4, 8) for g in (32, 64, 128)]


def _case(golden, key):
    bits = int(key.split("_")[1][1:])
    group = int(key.split("_")[2][1:])
    return bits, group, {n: golden[f"{key}_{n}"] for n in
                         ("w", "v", "alpha", "beta", "gq", "qdq", "codes", "scale", "zp",
                          "gv", "galpha", "gbeta")}


@pytest.mark.parametrize("key", CASES)
def test_forward_matches_reference(golden, key):
    bits, group, c = _case(golden, key)
    qdq, codes, scale, zp = quant_fp32.fake_quantize(c["w"], c["v"], c["alpha"], c["beta"], bits, group)
    assert relative_error(scale, c["scale"]) < FLOAT32_TOL
    assert np.array_equal(zp, c["zp"]), "zero points must match exactly"
    differing = float(np.mean(codes != c["codes"]))
    assert differing < 0.001, f"{differing:.3%} of codes differ"
    same = codes == c["codes"]
    assert relative_error(np.where(same, qdq, 0.0), np.where(same, c["qdq"], 0.0)) < FLOAT32_TOL


@pytest.mark.parametrize("key", CASES)
def test_gradients_match_reference(golden, key):
    bits, group, c = _case(golden, key)
    gv, ga, gb = quant_fp32.ste_grads(c["w"], c["v"], c["alpha"], c["beta"], c["gq"], bits, group)
    for name, got, want in (("v", gv, c["gv"]), ("alpha", ga, c["galpha"]), ("beta", gb, c["gbeta"])):
        assert relative_error(got, want) < GRAD_TOL, f"{name}: {relative_error(got, want):.2e}"


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_edge_groups(golden, bits):
    w = golden[f"edge_b{bits}_w"]
    ones = np.ones((w.shape[0], 1), np.float32)
    qdq, codes, scale, zp = quant_fp32.fake_quantize(w, np.zeros_like(w), ones, ones, bits, 4)
    assert np.array_equal(codes, golden[f"edge_b{bits}_codes"])
    assert np.array_equal(zp, golden[f"edge_b{bits}_zp"])
    assert relative_error(qdq, golden[f"edge_b{bits}_qdq"]) < FLOAT32_TOL
    assert ((zp >= 0) & (zp <= (1 << bits) - 1)).all(), "asymmetric zero point must be representable"
    gv, ga, gb = quant_fp32.ste_grads(w, np.zeros_like(w), ones, ones, np.ones_like(w), bits, 4)
    assert relative_error(gv, golden[f"edge_b{bits}_gv"]) < GRAD_TOL
    assert relative_error(ga, golden[f"edge_b{bits}_galpha"]) < GRAD_TOL
    assert relative_error(gb, golden[f"edge_b{bits}_gbeta"]) < GRAD_TOL


def test_all_zero_group_uses_eps(golden):
    w = golden["edge_b2_w"]
    ones = np.ones((w.shape[0], 1), np.float32)
    _, _, scale, _ = quant_fp32.fake_quantize(w, np.zeros_like(w), ones, ones, 2, 4)
    assert scale[3] == np.float32(1e-8)


def test_ties_round_to_even():
    # 0.5 -> 0, 1.5 -> 2, 2.5 -> 2 (reference tests/unit/test_reference_quantize.py:44-54)
    w = np.array([[0.0, 0.5, 1.5, 2.5, 3.0]], np.float32)
    ones = np.ones((1, 1), np.float32)
    # scale = 3/3 = 1 at 2 bits, zp = 0 -> codes are rint(w)
    _, codes, scale, zp = quant_fp32.fake_quantize(w, np.zeros_like(w), ones, ones, 2, -1)
    assert scale[0, 0] == 1.0 and zp[0, 0] == 0.0
    assert codes.tolist() == [[0.0, 0.0, 2.0, 2.0, 3.0]]


def test_optimizer_matches_reference(golden):
    v, a, b = golden["opt_v0"], golden["opt_a0"], golden["opt_b0"]
    lr0, iters = float(golden["opt_lr0"]), int(golden["opt_iters"])
    for step in range(iters):
        lr = quant_fp32.lr_at(lr0, iters, step)
        v, a, b = quant_fp32.signsgd_step(
            v, a, b, golden[f"opt_gv{step}"], golden[f"opt_ga{step}"], golden[f"opt_gb{step}"],
            lr, 0.1, 1.0)
    # float32 parameters against float64 arithmetic: one rounding per step
    assert np.abs(v - golden["opt_v5"]).max() < 1e-6
    assert np.abs(a - golden["opt_a5"]).max() < 1e-6
    assert np.abs(b - golden["opt_b5"]).max() < 1e-6
    assert np.abs(v).max() <= 0.5


@pytest.mark.parametrize("name", ["small", "mid"])
def test_losses_match_reference(golden, name):
    pred, tgt = golden[f"loss_{name}_pred"], golden[f"loss_{name}_tgt"]
    loss, grad, thr = losses_fp32.loss_and_grad(pred, tgt, suppress=True)
    assert loss == pytest.approx(float(golden[f"loss_{name}_outlier"]), rel=1e-6)
    assert relative_error(grad, golden[f"loss_{name}_outlier_grad"]) < 1e-6
    r = np.abs(pred - tgt)
    assert int((r >= thr).sum()) == losses_fp32.outlier_k(r.size)
    loss, grad, _ = losses_fp32.loss_and_grad(pred, tgt, suppress=False)
    assert loss == pytest.approx(float(golden[f"loss_{name}_mse"]), rel=1e-6)
    assert relative_error(grad, golden[f"loss_{name}_mse_grad"]) < 1e-6


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 7, 8])
def test_packing_matches_reference(golden, bits):
    codes = golden[f"pack_b{bits}_codes"]
    words = packing.pack_codes(codes, bits)
    assert np.array_equal(words, golden[f"pack_b{bits}_words"])
    assert np.array_equal(packing.unpack_codes(words, codes.shape[1], bits), codes)


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("group", [32, 64])
def test_deltaloss_matches_reference(golden, bits, group):
    got = deltaloss.delta_loss(golden["dl_w"], golden["dl_g"], bits, group)
    assert got == pytest.approx(float(golden[f"dl_b{bits}_g{group}"]), rel=1e-5)


def test_affine_form():
    scale = np.array([0.0123, 1e-8, 0.5], np.float32)
    zp = np.array([3.0, 0.0, 255.0], np.float32)
    s_bits, b_bits = packing.to_affine(scale, zp)
    s = packing.bf16_to_f32(s_bits)
    assert np.array_equal(s, packing.bf16_to_f32(packing.bf16_bits(scale)))
    assert packing.bf16_to_f32(b_bits)[2] == -(s[2] * 255.0)


def test_allocations_fixture_loads():
    cases = json.loads((GOLDEN / "allocations.json").read_text())
    assert len(cases) == 6 and all(c["by_layer"] for c in cases)
