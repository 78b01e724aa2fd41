"""The v2 candidate scale grid search. TEST ORACLE ONLY.

Restates the reference's search (``mround/reference/scale_search.py:78-211``,
MLX port ``mround/core/scale_search.py:73-187``): per group, the signed
largest-magnitude element (first on ties) is the anchor; candidate ``c`` maps
it onto ``-eff_c`` with ``eff_c = nmax - step * i``,

    inverse = -eff_c * (1 / anchor)            (0 when the anchor is 0)
    codes   = clip(rint(inverse * w), -nmax, nmax - 1)
    scale   = 1 / inverse                      (0 when inverse is 0)
    loss    = sum (scale * codes - w)^2 [* importance]

and the kept scale is the first candidate with the strictly smallest loss,
the anchor ``eff = nmax`` first and then ``i = -half .. half`` without 0.

Two evaluations of the same algorithm:

- ``search_scales_f64``: float64 throughout, the reference NumPy oracle's
  arithmetic (pinned to its outputs by ``tests/golden``);
- ``search_scales_f32``: float32, in the operation order of the CUDA kernel:
  each run of 8 consecutive elements of a group is summed left to right from
  zero, and the runs' partial sums are combined by a butterfly (pairs, then
  pairs of pairs, ...).  With the same summation order the device result is
  bit-identical to this one.
"""

from __future__ import annotations

import numpy as np

__all__ = ["candidates", "grid_steps", "search_scales_f32", "search_scales_f64"]

F32 = np.float32

# The 2-bit window and the grid size, from the reference's SearchGrid
# (mround/reference/scale_search.py:62-105).
_TWO_BIT_STEP = 0.01
_TWO_BIT_HALF_COUNT = 90
_GRID = 200


def grid_steps(bits: int, ratio: float = 0.75) -> tuple[float, int]:
    """``(step, half_count)`` of the candidate family at ``bits``."""
    if bits == 2:
        return _TWO_BIT_STEP, _TWO_BIT_HALF_COUNT
    nmax = float(2 ** (bits - 1))
    span = nmax * ratio
    step = span / _GRID * 2
    return step, int(span / step)


def candidates(bits: int, ratio: float = 0.75) -> np.ndarray:
    """Effective ranges in evaluation order, as float32 (anchor first)."""
    nmax = float(2 ** (bits - 1))
    step, half = grid_steps(bits, ratio)
    vals = [nmax] + [nmax - step * i for i in range(-half, half + 1) if i != 0]
    return np.array(vals, dtype=np.float64).astype(F32)


def _grouped(weight: np.ndarray, group: int) -> np.ndarray:
    w = np.asarray(weight)
    if w.ndim != 2 or w.shape[1] % group:
        raise ValueError(f"weight {w.shape} does not group by {group}")
    return w.reshape(-1, group)


def _anchor(grouped: np.ndarray) -> np.ndarray:
    idx = np.argmax(np.abs(grouped), axis=-1)[:, None]
    return np.take_along_axis(grouped, idx, axis=-1)


def _qw(importance, weight_shape, group, dtype):
    if importance is None:
        return None
    flat = np.asarray(importance, dtype=dtype).reshape(-1)
    if flat.size != weight_shape[1]:
        raise ValueError("importance does not match the input width")
    return np.tile(flat, weight_shape[0]).reshape(-1, group)


def search_scales_f64(weight, bits: int, group: int, importance=None, ratio: float = 0.75):
    """Float64 search; returns (n_groups, 1) float64 signed scales."""
    grouped = _grouped(np.asarray(weight, dtype=np.float64), group)
    qw = _qw(importance, np.shape(weight), group, np.float64)
    nmax = float(2 ** (bits - 1))
    gm = _anchor(grouped)
    rg = np.zeros_like(gm)
    np.divide(1.0, gm, out=rg, where=gm != 0)

    def evaluate(eff: float):
        inv = -eff * rg
        codes = np.clip(np.rint(inv * grouped), -nmax, nmax - 1.0)
        sc = np.zeros_like(inv)
        np.divide(1.0, inv, out=sc, where=inv != 0)
        r = (sc * codes - grouped) ** 2
        if qw is not None:
            r = r * qw
        return sc, r.sum(axis=-1, keepdims=True)

    best_s, best_l = evaluate(nmax)
    step, half = grid_steps(bits, ratio)
    for i in range(-half, half + 1):
        if i == 0:
            continue
        s, l = evaluate(nmax - step * i)
        better = l < best_l
        best_s = np.where(better, s, best_s)
        best_l = np.where(better, l, best_l)
    return best_s


def _device_sum(sq: np.ndarray, group: int) -> np.ndarray:
    """Per-group float32 sum in the kernel's order (8-element runs, butterfly)."""
    lanes = group // 8
    runs = sq.reshape(sq.shape[0], lanes, 8)
    acc = np.zeros(runs.shape[:2], dtype=F32)
    for i in range(8):
        acc = (acc + runs[:, :, i]).astype(F32)
    off = 1
    while off < lanes:
        partner = np.arange(lanes) ^ off
        acc = (acc + acc[:, partner]).astype(F32)
        off <<= 1
    return acc[:, :1]


def search_scales_f32(weight, bits: int, group: int, importance=None, ratio: float = 0.75):
    """Float32 search in the device's operation order; (n_groups, 1) float32."""
    if group % 8:
        raise ValueError("the device search takes groups of a multiple of 8")
    grouped = _grouped(np.asarray(weight, dtype=F32), group)
    qw = _qw(importance, np.shape(weight), group, F32)
    nmax = F32(2 ** (bits - 1))
    gm = _anchor(grouped)
    with np.errstate(divide="ignore"):
        rg = np.where(gm != 0, (F32(1.0) / gm).astype(F32), F32(0.0)).astype(F32)
    best_s = best_l = None
    for eff in candidates(bits, ratio):
        inv = ((-eff) * rg).astype(F32)
        codes = np.clip(np.rint((inv * grouped).astype(F32)), -nmax, nmax - F32(1.0)).astype(F32)
        with np.errstate(divide="ignore"):
            sc = np.where(inv != 0, (F32(1.0) / inv).astype(F32), F32(0.0)).astype(F32)
        r = ((sc * codes).astype(F32) - grouped).astype(F32)
        sq = (r * r).astype(F32)
        if qw is not None:
            sq = (sq * qw).astype(F32)
        loss = _device_sum(sq, group)
        if best_s is None:
            best_s, best_l = sc, loss
        else:
            better = loss < best_l
            best_s = np.where(better, sc, best_s).astype(F32)
            best_l = np.where(better, loss, best_l).astype(F32)
    return best_s
