"""Device quantizer with the reference's function names and parameter layout.

Mirrors ``mround/core/quantizer.py`` for asymmetric observed-range schemes on
CUDA tensors: ``init_params`` (414-427), ``fake_quantize`` (287-347),
``quantize_codes`` (350-398), ``dequantize`` (401-411), ``project_params``
(430-446).  Parameters are a dict ``{"v", "alpha", "beta"}`` as in the
reference, in its grouped shapes ``(rows, n_groups, group)`` /
``(rows, n_groups, 1)`` (views of contiguous float32 storage).  The arithmetic
is the K1/K5 kernels'; there is no CPU path.  Symmetric and searched schemes
are refused with :class:`UnsupportedSchemeError` (the device path covers the
asymmetric observed-range scheme of every benchmark configuration).
"""

from __future__ import annotations

import torch

from mround_b200 import kernels
from mround_b200.exceptions import SchemeError, UnsupportedSchemeError
from mround_b200.schemes import DEFAULT_EPS_FP32, QuantScheme, ScaleInit, Symmetry

__all__ = [
    "V_BOUND",
    "dequantize",
    "fake_quantize",
    "init_params",
    "project_params",
    "quantize_codes",
    "require_device_scheme",
]

V_BOUND = 0.5

Params = dict[str, torch.Tensor]


def require_device_scheme(scheme: QuantScheme, in_features: int) -> int:
    """Group size the device kernels will use; refuses what they do not cover."""
    if scheme.symmetry is not Symmetry.ASYMMETRIC or scheme.scale_init is not ScaleInit.OBSERVED_RANGE:
        raise UnsupportedSchemeError(
            f"the B200 path implements asymmetric observed-range schemes; got {scheme.symmetry.value}"
            f"/{scheme.scale_init.value}"
        )
    group = in_features if scheme.is_per_channel else scheme.group_size
    if group not in kernels.DEVICE_GROUPS:
        raise UnsupportedSchemeError(
            f"group size {group} is not one of the device group sizes {kernels.DEVICE_GROUPS}"
        )
    if in_features % group:
        raise SchemeError(f"in_features={in_features} is not divisible by group_size={group}")
    return group


def _flat(params: Params, rows: int, cols: int, group: int):
    v = params["v"].reshape(rows, cols)
    a = params["alpha"].reshape(rows, cols // group)
    b = params["beta"].reshape(rows, cols // group)
    return v.contiguous(), a.contiguous(), b.contiguous()


def _unit_params(weight: torch.Tensor, group: int) -> Params:
    rows, cols = weight.shape
    ng = cols // group
    return {
        "v": torch.zeros((rows, ng, group), dtype=torch.float32, device=weight.device),
        "alpha": torch.ones((rows, ng, 1), dtype=torch.float32, device=weight.device),
        "beta": torch.ones((rows, ng, 1), dtype=torch.float32, device=weight.device),
    }


def init_params(weight: torch.Tensor, scheme: QuantScheme) -> Params:
    """Zero perturbation and unit coefficients: the start is round-to-nearest."""
    group = require_device_scheme(scheme, weight.shape[1])
    return _unit_params(weight, group)


def fake_quantize(weight: torch.Tensor, params: Params | None, scheme: QuantScheme, *,
                  eps: float = DEFAULT_EPS_FP32) -> torch.Tensor:
    """Quantize-dequantize ``weight`` (bf16, (out, in)); returns float32 (out, in)."""
    rows, cols = weight.shape
    group = require_device_scheme(scheme, cols)
    params = params if params is not None else _unit_params(weight, group)
    v, a, b = _flat(params, rows, cols, group)
    out = torch.empty((rows, cols), dtype=torch.float32, device=weight.device)
    kernels.fq_forward(weight.to(torch.bfloat16).contiguous(), v, a, b, bits=scheme.bits,
                       group=group, eps=eps, wq_f32=out)
    return out


def quantize_codes(weight: torch.Tensor, params: Params | None, scheme: QuantScheme, *,
                   eps: float = DEFAULT_EPS_FP32):
    """``(codes, scale, zero_point)`` grouped as the reference returns them.

    ``codes`` are uint8 (rows, n_groups, group) -- already the narrowed form
    of ``narrow_codes`` -- and ``scale``/``zero_point`` float32 (rows, n_groups, 1).
    """
    rows, cols = weight.shape
    group = require_device_scheme(scheme, cols)
    params = params if params is not None else _unit_params(weight, group)
    v, a, b = _flat(params, rows, cols, group)
    w = weight.to(torch.bfloat16).contiguous()
    scale = torch.empty((rows, cols // group), dtype=torch.float32, device=weight.device)
    zp = torch.empty_like(scale)
    kernels.fq_forward(w, v, a, b, bits=scheme.bits, group=group, eps=eps, scale=scale, zp=zp)
    bits = scheme.bits
    packable = (cols % (32 // bits) == 0) if 32 % bits == 0 else (cols % 32 == 0)
    if not packable:
        raise SchemeError(f"in_features={cols} does not tile {bits}-bit words")
    _, _, _, codes = kernels.pack_mlx(w, v, a, b, bits=bits, group=group, eps=eps, want_codes=True)
    ng = cols // group
    return codes.view(rows, ng, group), scale.view(rows, ng, 1), zp.view(rows, ng, 1)


def dequantize(codes: torch.Tensor, scale: torch.Tensor, zero_point: torch.Tensor,
               shape: tuple[int, int], scheme: QuantScheme) -> torch.Tensor:
    """``scale * (codes - zero_point)`` in float32, ungrouped."""
    out = scale.float() * (codes.float() - zero_point.float())
    return out.reshape(shape)


def project_params(params: Params, scheme: QuantScheme) -> Params:
    """Clip into the permitted ranges; returns a new mapping."""
    lo, hi = scheme.coefficient_bounds
    return {
        "v": params["v"].clamp(-V_BOUND, V_BOUND),
        "alpha": params["alpha"].clamp(lo, hi),
        "beta": params["beta"].clamp(lo, hi),
    }
