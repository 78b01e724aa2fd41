"""Block reconstruction losses, float32 residuals. TEST ORACLE ONLY.

Restates the MLX losses (reference ``mround/core/losses.py``):

- ``reconstruction_loss`` 42-56: ``mean(r * r)``, ``r = pred - target`` in float32;
- ``outlier_threshold`` 96-107: the k-th largest ``|r|`` over the flattened
  batch, ``k = max(1, int(n * 0.001))``;
- ``outlier_suppressed_loss`` 59-93: errors with ``|r| >= threshold`` are zeroed
  (strict comparison, so ties at the threshold are all excluded) and the sum is
  divided by the full count ``n``;
- ``piece_loss`` 110-130: a piece's share, divided by the whole batch's count.

Sums are carried in float64; the gradient ``2 * r * keep / n`` is float32.
"""

from __future__ import annotations

import numpy as np

__all__ = ["OUTLIER_FRACTION", "outlier_k", "outlier_threshold", "loss_and_grad"]

OUTLIER_FRACTION = 0.001


def outlier_k(n: int, fraction: float = OUTLIER_FRACTION) -> int:
    """Number of elements at or above the threshold (``losses.py:106``)."""
    return max(1, int(n * fraction))


def outlier_threshold(residual: np.ndarray, fraction: float = OUTLIER_FRACTION) -> np.float32:
    """k-th largest |r| of the flattened residual (``losses.py:105-107``)."""
    flat = np.abs(np.asarray(residual, dtype=np.float32)).reshape(-1)
    n = flat.size
    k = outlier_k(n, fraction)
    return np.float32(np.partition(flat, n - k)[n - k])


def loss_and_grad(pred, target, *, suppress: bool, elements: int | None = None,
                  threshold: np.float32 | None = None):
    """Return ``(loss float64, dL/dpred float32, threshold or None)``.

    ``elements`` is the divisor (the whole batch's count for a piece);
    ``threshold`` given means the piece form of the outlier rule.
    """
    r = (np.asarray(pred, dtype=np.float32) - np.asarray(target, dtype=np.float32)).astype(np.float32)
    n = r.size if elements is None else int(elements)
    thr = None
    if suppress:
        thr = outlier_threshold(r) if threshold is None else np.float32(threshold)
        keep = (np.abs(r) < thr)
        kept = np.where(keep, r, np.float32(0.0)).astype(np.float32)
    else:
        kept = r
    loss = float(np.sum(kept.astype(np.float64) ** 2) / n)
    grad = (np.float32(2.0) * kept / np.float32(n)).astype(np.float32)
    return loss, grad, thr


def radix_digit_hist(residual: np.ndarray, pass_index: int, prefix: int, mask: int) -> np.ndarray:
    """Histogram of one radix digit of |r|'s bit pattern among keys matching the
    prefix -- the same digit layout as the device selection ([21,31), [10,21), [0,10))."""
    keys = np.abs(np.asarray(residual, np.float32)).reshape(-1).view(np.uint32) & np.uint32(0x7FFFFFFF)
    shift = (21, 10, 0)[pass_index]
    dmask = (0x3FF, 0x7FF, 0x3FF)[pass_index]
    sel = keys[(keys & np.uint32(mask)) == np.uint32(prefix)]
    return np.bincount(((sel >> np.uint32(shift)) & np.uint32(dmask)).astype(np.int64),
                       minlength=2048).astype(np.int64)


def radix_select_step(hist: np.ndarray, k_left: int, pass_index: int, prefix: int, mask: int):
    """Pick the digit holding the k_left-th largest; returns (prefix, mask, k_left)."""
    shift = (21, 10, 0)[pass_index]
    dmask = (0x3FF, 0x7FF, 0x3FF)[pass_index]
    above = 0
    for b in range(dmask, -1, -1):
        if above + int(hist[b]) >= k_left:
            return prefix | (b << shift), mask | (dmask << shift), k_left - above
        above += int(hist[b])
    raise ValueError("k exceeds the candidate count")
