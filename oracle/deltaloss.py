"""DeltaLoss sensitivity score. TEST ORACLE ONLY.

``sum |g * (Q_b(W) - W)|`` in float64 (reference
``mround/planner/sensitivity.py:190-229``), where ``Q_b`` is round-to-nearest
at width ``b``: the quantizer with ``v = 0`` and unit clipping coefficients
(``mround/pipeline/scoring.py:213-221``, the perturbation of line 262).
"""

from __future__ import annotations

import numpy as np

from oracle.quant_fp32 import fake_quantize

__all__ = ["delta_loss", "rtn"]


def rtn(w: np.ndarray, bits: int, group: int, eps: float = 1e-8, *, symmetric: bool = False,
        init_scale=None) -> np.ndarray:
    """Round-to-nearest quantize-dequantize, float32 (any scheme; a searched
    scheme passes its grid as ``init_scale``)."""
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    ng = 1 if group == -1 else cols // group
    ones = np.ones((rows, ng), np.float32)
    qdq, _, _, _ = fake_quantize(w, np.zeros_like(w), ones, ones, bits, group, eps,
                                 symmetric=symmetric, init_scale=init_scale)
    return qdq


def delta_loss(w: np.ndarray, g: np.ndarray, bits: int, group: int, eps: float = 1e-8, *,
               symmetric: bool = False, init_scale=None) -> float:
    """Score of one layer at one width, accumulated in float64."""
    q = rtn(w, bits, group, eps, symmetric=symmetric, init_scale=init_scale).astype(np.float64)
    return float(np.sum(np.abs(np.asarray(g, np.float64) * (q - np.asarray(w, np.float64)))))
