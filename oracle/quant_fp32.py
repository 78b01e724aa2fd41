"""Float32 restatement of MRound's fake quantization. TEST ORACLE ONLY.

Asymmetric, symmetric observed-range and searched (symmetric, scale from the
v2 grid search times beta) schemes.  The asymmetric path is described below;
the symmetric and searched paths follow ``symmetric_scale`` /
``_clamp_magnitude`` and the searched branch of ``fake_quantize``
(reference ``mround/core/quantizer.py:216-251, 319-339``).

Follows the operation order of the MLX implementation, which computes in
float32 (reference ``mround/core/quantizer.py``):

- extremes with zero forced in, times the clipping coefficients
  (``_clipped_extremes`` 185-195);
- ``scale = max((w_max - w_min) / maxq, eps)``, ``zp = rint(-w_min / scale)``
  (``asymmetric_scale`` 254-266, ties to even as ``round_half_to_even`` 84-107);
- ``codes = clip(rint(W / scale + v) + zp, 0, maxq)``, ``qdq = scale * (codes - zp)``
  (``fake_quantize`` 341-347, ``quantize_codes`` 395-398).

The backward is the chain MLX autodiff builds through ``round_ste`` (identity),
``clip_ste`` (gradient passes where ``0 <= x <= maxq``, inclusive,
``quantizer.py:119-149``) and the zero point's own straight-through rounding.
Written out per group, with ``inside`` the clamp mask and ``g`` the gradient on
the reconstruction, it is the hand derivation of
``mround/reference/quantize.py:488-520``:

    gV     = g * scale * inside
    gscale = sum g * [(codes - zp) + (inside * (w_min - W) - w_min) / scale]
    galpha = gscale * w_max_raw / maxq
    gbeta  = gscale * (-w_min_raw / maxq) + sum g * (1 - inside) * w_min_raw

The forward (codes, masks, scale, zero point) is evaluated in float32 so the
integer decisions are the ones a float32 implementation makes; the gradient
arithmetic and its group sums are carried in float64 so that the oracle is the
most accurate statement of the float32 path's gradient.

``signsgd_step`` restates ``SignSGD.apply`` + ``project_params``
(``mround/core/signsgd.py:76-85, 125-145``; ``mround/core/quantizer.py:430-446``):
``p <- clip(p - float32(lr) * sign(g), lo, hi)`` with V bounded by 0.5.

Sign of zero: a group whose minimum is exactly zero or positive gets
``w_min_raw = +0.0``, which makes ``zp = -0.0`` (``rint(-0/s)``); the CUDA
kernel makes the same choice, so the bf16 bias ``-scales * zp`` agrees to the bit.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "V_BOUND",
    "fake_quantize",
    "group_view",
    "lr_at",
    "signsgd_step",
    "ste_grads",
]

V_BOUND = np.float32(0.5)
F32 = np.float32


def group_view(x: np.ndarray, group: int) -> np.ndarray:
    """(rows, cols) -> (rows, cols // group, group); group -1 is the whole row."""
    rows, cols = x.shape
    g = cols if group == -1 else group
    if cols % g:
        raise ValueError(f"cols={cols} is not a multiple of group={g}")
    return x.reshape(rows, cols // g, g)


def _forward_parts(w, v, alpha, beta, bits, group, eps, symmetric=False, init_scale=None):
    w = np.asarray(w, dtype=F32)
    grouped = group_view(w, group)
    vg = np.asarray(v, dtype=F32).reshape(grouped.shape)
    a = np.asarray(alpha, dtype=F32).reshape(grouped.shape[0], grouped.shape[1], 1)
    b = np.asarray(beta, dtype=F32).reshape(grouped.shape[0], grouped.shape[1], 1)
    if symmetric or init_scale is not None:
        return _forward_parts_sym(grouped, vg, a, b, bits, eps, init_scale)
    maxq = F32((1 << bits) - 1)
    gmax = grouped.max(axis=-1, keepdims=True)
    gmin = grouped.min(axis=-1, keepdims=True)
    wmax_raw = np.where(gmax > 0, gmax, F32(0.0)).astype(F32)
    wmin_raw = np.where(gmin < 0, gmin, F32(0.0)).astype(F32)
    w_max = (wmax_raw * a).astype(F32)
    w_min = (wmin_raw * b).astype(F32)
    span = ((w_max - w_min) / maxq).astype(F32)
    scale = np.maximum(span, F32(eps)).astype(F32)
    zp = np.rint((-w_min) / scale).astype(F32)
    raw = (grouped / scale + vg).astype(F32)
    x = (np.rint(raw) + zp).astype(F32)
    codes = np.clip(x, F32(0.0), maxq).astype(F32)
    qdq = (scale * (codes - zp)).astype(F32)
    return dict(
        grouped=grouped, maxq=maxq, wmax_raw=wmax_raw, wmin_raw=wmin_raw,
        w_max=w_max, w_min=w_min, span=span, scale=scale, zp=zp, x=x,
        codes=codes, qdq=qdq, symmetric=False,
    )


def _clamp_magnitude(s, eps):
    """``sign(s) * max(|s|, eps)`` with sign(0) = +1 (reference quantizer.py:216-225)."""
    sign = np.sign(s).astype(F32)
    sign = np.where(sign == 0, F32(1.0), sign).astype(F32)
    return (sign * np.maximum(np.abs(s), F32(eps))).astype(F32)


def _forward_parts_sym(grouped, vg, a, b, bits, eps, init_scale):
    """Symmetric observed-range scale (reference ``symmetric_scale``
    quantizer.py:228-251) or the searched scale times beta (``fake_quantize``
    searched branch, quantizer.py:319-331); codes in [-2^(b-1), 2^(b-1) - 1]."""
    maxq = F32(1 << (bits - 1))
    gmax = grouped.max(axis=-1, keepdims=True)
    gmin = grouped.min(axis=-1, keepdims=True)
    wmax_raw = np.where(gmax > 0, gmax, F32(0.0)).astype(F32)
    wmin_raw = np.where(gmin < 0, gmin, F32(0.0)).astype(F32)
    if init_scale is None:
        w_max = (wmax_raw * a).astype(F32)
        w_min = (wmin_raw * b).astype(F32)
        neg_mag = (-w_min).astype(F32)
        pos = w_max >= neg_mag
        dominant = np.where(pos, w_max, neg_mag).astype(F32)
        signed = np.where(pos, -dominant, dominant).astype(F32)
        s = (signed / maxq).astype(F32)
        base = None
    else:
        base = np.asarray(init_scale, dtype=F32).reshape(b.shape)
        s = (base * b).astype(F32)
        pos = np.zeros(b.shape, dtype=bool)
    scale = _clamp_magnitude(s, eps)
    raw = (grouped / scale + vg).astype(F32)
    x = np.rint(raw).astype(F32)
    codes = np.clip(x, -maxq, maxq - F32(1.0)).astype(F32)
    qdq = (scale * codes).astype(F32)
    return dict(
        grouped=grouped, maxq=maxq, wmax_raw=wmax_raw, wmin_raw=wmin_raw, pos=pos,
        span=np.abs(s).astype(F32), scale=scale, zp=None, x=x, codes=codes, qdq=qdq,
        symmetric=True, base=base,
    )


def fake_quantize(w, v, alpha, beta, bits, group, eps=1e-8, *, symmetric=False, init_scale=None):
    """Return ``(qdq, codes, scale, zp)``.

    ``qdq`` is (rows, cols) float32; ``codes`` (rows, cols) float32 integers in
    ``[0, 2**bits - 1]`` (asymmetric) or ``[-2**(bits-1), 2**(bits-1) - 1]``
    (symmetric, and searched when ``init_scale`` is given); ``scale`` and ``zp``
    (rows, n_groups) float32, ``zp`` None for symmetric schemes.
    """
    p = _forward_parts(w, v, alpha, beta, bits, group, eps, symmetric, init_scale)
    rows, cols = np.asarray(w).shape
    return (
        p["qdq"].reshape(rows, cols),
        p["codes"].reshape(rows, cols),
        p["scale"][..., 0],
        None if p["zp"] is None else p["zp"][..., 0],
    )


def ste_grads(w, v, alpha, beta, gq, bits, group, eps=1e-8, *, symmetric=False, init_scale=None):
    """Gradients of the loss w.r.t. ``(v, alpha, beta)`` given ``gq = dL/dqdq``.

    Returns ``(gV (rows, cols) float32, galpha, gbeta (rows, n_groups) float64)``.
    """
    p = _forward_parts(w, v, alpha, beta, bits, group, eps, symmetric, init_scale)
    if p["symmetric"]:
        return _ste_grads_sym(p, w, gq, group, eps)
    g = group_view(np.asarray(gq, dtype=F32), group).astype(np.float64)
    scale = p["scale"].astype(np.float64)
    inside = ((p["x"] >= 0) & (p["x"] <= p["maxq"])).astype(np.float64)
    codes = p["codes"].astype(np.float64)
    zp = p["zp"].astype(np.float64)
    w_min = p["w_min"].astype(np.float64)
    grouped = p["grouped"].astype(np.float64)

    gv32 = (np.asarray(gq, dtype=F32).reshape(g.shape) * p["scale"]).astype(F32)
    gv32 = (gv32 * inside.astype(F32)).astype(F32)

    d_scale = (codes - zp) + (inside * (w_min - grouped) - w_min) / scale
    gscale = (g * d_scale).sum(axis=-1, keepdims=True)
    # The eps floor on the scale removes its dependence on the coefficients.
    live = (p["span"] > F32(eps)).astype(np.float64)
    gscale_pre = gscale * live
    maxq = float(p["maxq"])
    direct = (g * (1.0 - inside)).sum(axis=-1, keepdims=True)
    galpha = gscale_pre / maxq * p["wmax_raw"].astype(np.float64)
    gbeta = (direct - gscale_pre / maxq) * p["wmin_raw"].astype(np.float64)
    rows, cols = np.asarray(w).shape
    return gv32.reshape(rows, cols), galpha[..., 0], gbeta[..., 0]


def _ste_grads_sym(p, w, gq, group, eps):
    """Symmetric and searched branches of the straight-through backward
    (reference ``mround/reference/quantize.py:370-397, 465-486``):

        gV     = g * scale * inside
        gscale = sum g * (codes - inside * W / scale)
        observed: galpha = gscale * (-w_max_raw / maxq) where the positive side
                  dominates, else 0; gbeta = gscale * (-w_min_raw / maxq) where
                  the negative side dominates, else 0
        searched: galpha = 0; gbeta = gscale * init_scale

    ``gscale`` is zeroed where the eps floor holds the scale (``|s| <= eps``),
    as the autodiff of ``max(|s|, eps)`` does.
    """
    g = group_view(np.asarray(gq, dtype=F32), group).astype(np.float64)
    maxq = float(p["maxq"])
    inside = ((p["x"] >= -maxq) & (p["x"] <= maxq - 1.0)).astype(np.float64)
    scale = p["scale"].astype(np.float64)
    codes = p["codes"].astype(np.float64)
    grouped = p["grouped"].astype(np.float64)
    gv32 = (np.asarray(gq, dtype=F32).reshape(g.shape) * p["scale"]).astype(F32)
    gv32 = (gv32 * inside.astype(F32)).astype(F32)
    gscale = (g * (codes - inside * grouped / scale)).sum(axis=-1, keepdims=True)
    gscale = gscale * (p["span"] > F32(eps)).astype(np.float64)
    if p["base"] is not None:
        galpha = np.zeros_like(gscale)
        gbeta = gscale * p["base"].astype(np.float64)
    else:
        pos = p["pos"]
        galpha = np.where(pos, gscale * (-p["wmax_raw"].astype(np.float64) / maxq), 0.0)
        gbeta = np.where(pos, 0.0, gscale * (-p["wmin_raw"].astype(np.float64) / maxq))
    rows, cols = np.asarray(w).shape
    return gv32.reshape(rows, cols), galpha[..., 0], gbeta[..., 0]


def lr_at(lr0: float, iters: int, step: int) -> float:
    """LinearDecay (reference ``mround/core/signsgd.py:36-62``)."""
    if step >= iters:
        return 0.0
    return lr0 * (1.0 - step / iters)


def signsgd_step(v, alpha, beta, gv, galpha, gbeta, lr, lo, hi):
    """One signed step plus projection, float32, returning new arrays."""
    lr32 = F32(lr)
    sv = np.sign(np.asarray(gv, dtype=np.float64)).astype(F32)
    sa = np.sign(np.asarray(galpha, dtype=np.float64)).astype(F32)
    sb = np.sign(np.asarray(gbeta, dtype=np.float64)).astype(F32)
    v_new = np.clip((np.asarray(v, F32) - lr32 * sv).astype(F32), -V_BOUND, V_BOUND)
    a_new = np.clip((np.asarray(alpha, F32) - lr32 * sa).astype(F32), F32(lo), F32(hi))
    b_new = np.clip((np.asarray(beta, F32) - lr32 * sb).astype(F32), F32(lo), F32(hi))
    return v_new.astype(F32), a_new.astype(F32), b_new.astype(F32)
