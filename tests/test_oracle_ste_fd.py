"""The oracle's straight-through gradients against central finite differences.

An analytic pin, independent of the reference's golden vectors (the reference
pins its NumPy gradients the same way, ``tests/unit/test_reference_quantize.py``
finite differences of a surrogate).  At a point (V0, alpha0, beta0) the
straight-through backward is the exact gradient of a *frozen surrogate*: the
same forward with every integer decision held at its value at the point --
each element's rounding offset rint(x) - x, the zero point's rounding offset,
the clamp mask (inclusive) and the clamped codes outside it.  The surrogate is
smooth in (V, alpha, beta), so float64 central differences of
sum(g * qdq_surrogate) must equal ``oracle.quant_fp32.ste_grads`` for the
asymmetric, symmetric observed-range and searched schemes.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import quant_fp32 as Q

ROWS, COLS, GROUP, H = 4, 128, 32, 1e-6


def _point(seed, symmetric, searched):
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, (ROWS, COLS)).astype(np.float32)
    w[rng.random((ROWS, COLS)) < 0.02] *= 8.0
    v = rng.uniform(-0.3, 0.3, (ROWS, COLS)).astype(np.float32)
    ng = COLS // GROUP
    a = rng.uniform(0.6, 1.0, (ROWS, ng)).astype(np.float32)
    b = rng.uniform(0.6, 1.0, (ROWS, ng)).astype(np.float32)
    g = rng.normal(0.0, 1.0, (ROWS, COLS)).astype(np.float32)
    init = rng.uniform(0.002, 0.01, (ROWS, ng)).astype(np.float32) if searched else None
    return w, v, a, b, g, init


def _surrogate(w, g, bits, symmetric, init, frozen):
    """sum(g * qdq) with the integer decisions of ``frozen`` (float64)."""
    wg = Q.group_view(w.astype(np.float64), GROUP)
    gg = Q.group_view(g.astype(np.float64), GROUP)
    p = frozen

    def value(v, a, b):
        vg = v.reshape(wg.shape)
        a3, b3 = a[..., None], b[..., None]
        if not symmetric and init is None:
            maxq = float((1 << bits) - 1)
            s = (p["wmax_raw"] * a3 - p["wmin_raw"] * b3) / maxq
            zp = -(p["wmin_raw"] * b3) / s + p["dz"]
            x = wg / s + vg + p["dr"] + zp
            c = np.where(p["inside"], x, p["codes"])
            return float((gg * s * (c - zp)).sum())
        maxq = float(1 << (bits - 1))
        if init is not None:
            s = init[..., None].astype(np.float64) * b3
        else:
            s = np.where(p["pos"], -(p["wmax_raw"] * a3), -(p["wmin_raw"] * b3)) / maxq
        x = wg / s + vg + p["dr"]
        c = np.where(p["inside"], x, p["codes"])
        return float((gg * s * c).sum())

    return value


def _frozen(w, v, a, b, bits, symmetric, init):
    p = Q._forward_parts(w, v, a, b, bits, GROUP, 1e-8, symmetric, init)
    wg = p["grouped"].astype(np.float64)
    s = p["scale"].astype(np.float64)
    raw = wg / s + v.reshape(wg.shape).astype(np.float64)
    out = {"wmax_raw": p["wmax_raw"].astype(np.float64),
           "wmin_raw": p["wmin_raw"].astype(np.float64),
           "codes": p["codes"].astype(np.float64)}
    maxq = float(p["maxq"])
    if p["symmetric"]:
        out["dr"] = np.rint(raw) - raw
        out["inside"] = (p["x"] >= -maxq) & (p["x"] <= maxq - 1.0)
        out["pos"] = p["pos"]
    else:
        zp = p["zp"].astype(np.float64)
        out["dz"] = zp - (-p["w_min"].astype(np.float64) / s)
        out["dr"] = np.rint(raw) - raw
        out["inside"] = (p["x"] >= 0) & (p["x"] <= maxq)
    return out


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("kind", ["asym", "sym", "searched"])
def test_ste_gradients_equal_frozen_surrogate_differences(bits, kind):
    symmetric, searched = kind != "asym", kind == "searched"
    w, v, a, b, g, init = _point(bits * 10 + len(kind), symmetric, searched)
    gv, ga, gb = Q.ste_grads(w, v, a, b, g, bits, GROUP, symmetric=symmetric, init_scale=init)
    f = _surrogate(w, g, bits, symmetric, init, _frozen(w, v, a, b, bits, symmetric, init))
    v64, a64, b64 = v.astype(np.float64), a.astype(np.float64), b.astype(np.float64)

    def central(which, idx):
        args = [v64.copy(), a64.copy(), b64.copy()]
        args[which][idx] += H
        up = f(*args)
        args[which][idx] -= 2 * H
        down = f(*args)
        return (up - down) / (2 * H)

    rng = np.random.default_rng(bits)
    picks = [(int(r), int(c)) for r, c in zip(rng.integers(0, ROWS, 24), rng.integers(0, COLS, 24))]
    fd_v = np.array([central(0, ix) for ix in picks])
    want_v = np.array([gv[ix] for ix in picks], dtype=np.float64)
    assert np.allclose(fd_v, want_v, rtol=1e-5, atol=1e-6 * np.abs(want_v).max())
    fd_a = np.array([[central(1, (r, j)) for j in range(COLS // GROUP)] for r in range(ROWS)])
    fd_b = np.array([[central(2, (r, j)) for j in range(COLS // GROUP)] for r in range(ROWS)])
    scale_a = max(np.abs(ga).max(), 1e-12)
    scale_b = max(np.abs(gb).max(), 1e-12)
    assert np.abs(fd_a - ga).max() <= 1e-5 * scale_a, (fd_a, ga)
    assert np.abs(fd_b - gb).max() <= 1e-5 * scale_b, (fd_b, gb)
    if searched:
        assert np.all(ga == 0.0), "alpha is inert under the searched scale"
