"""Device quantizer with the reference's function names and parameter layout.

Mirrors ``mround/core/quantizer.py`` on CUDA tensors for every scheme it
defines -- asymmetric and symmetric observed-range, and the searched (v2)
symmetric scale: ``init_params`` (414-427), ``fake_quantize`` (287-347),
``quantize_codes`` (350-398), ``dequantize`` (401-411), ``project_params``
(430-446).  Parameters are a dict ``{"v", "alpha", "beta"}`` as in the
reference, in its grouped shapes ``(rows, n_groups, group)`` /
``(rows, n_groups, 1)`` (views of contiguous float32 storage); a searched
scheme takes ``init_scale`` from :func:`mround_b200.core.scale_search.search_scales`
and refuses to run without it, as the reference does (``_check_init_scale``
196-213).  The arithmetic is the K1/K5 kernels'; there is no CPU path.
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
    group = in_features if scheme.is_per_channel else scheme.group_size
    if group not in kernels.DEVICE_GROUPS:
        raise UnsupportedSchemeError(
            f"group size {group} is not one of the device group sizes {kernels.DEVICE_GROUPS}"
        )
    if in_features % group:
        raise SchemeError(f"in_features={in_features} is not divisible by group_size={group}")
    return group


def _check_init_scale(scheme: QuantScheme, init_scale: torch.Tensor | None) -> None:
    """A searched scheme needs its scale, and only it takes one (reference 196-213)."""
    if scheme.scale_init is ScaleInit.SEARCHED and init_scale is None:
        raise ValueError("a SEARCHED scheme needs the searched scale: pass init_scale from "
                         "scale_search.search_scales")
    if scheme.scale_init is not ScaleInit.SEARCHED and init_scale is not None:
        raise ValueError("init_scale was given but the scheme's scale_init is not SEARCHED")


def _scheme_kw(scheme: QuantScheme, init_scale: torch.Tensor | None, rows: int, ng: int) -> dict:
    _check_init_scale(scheme, init_scale)
    init = None
    if init_scale is not None:
        init = init_scale.to(torch.float32).reshape(rows, ng).contiguous()
    return {"symmetric": scheme.symmetry is Symmetry.SYMMETRIC, "init_scale": init}


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
                  eps: float = DEFAULT_EPS_FP32,
                  init_scale: torch.Tensor | None = None) -> torch.Tensor:
    """Quantize-dequantize ``weight`` (bf16, (out, in)); returns float32 (out, in)."""
    rows, cols = weight.shape
    group = require_device_scheme(scheme, cols)
    kw = _scheme_kw(scheme, init_scale, rows, cols // group)
    params = params if params is not None else _unit_params(weight, group)
    v, a, b = _flat(params, rows, cols, group)
    out = torch.empty((rows, cols), dtype=torch.float32, device=weight.device)
    kernels.fq_forward(weight.to(torch.bfloat16).contiguous(), v, a, b, bits=scheme.bits,
                       group=group, eps=eps, wq_f32=out, **kw)
    return out


def quantize_codes(weight: torch.Tensor, params: Params | None, scheme: QuantScheme, *,
                   eps: float = DEFAULT_EPS_FP32, init_scale: torch.Tensor | None = None):
    """``(codes, scale, zero_point)`` grouped as the reference returns them.

    ``codes`` are (rows, n_groups, group) one byte each -- already the narrowed
    form of ``narrow_codes``: uint8, or int8 under a symmetric scheme --
    ``scale`` float32 (rows, n_groups, 1) and ``zero_point`` the same shape, or
    None under a symmetric scheme (the fixed ``2**(bits-1)`` applies).
    """
    rows, cols = weight.shape
    group = require_device_scheme(scheme, cols)
    ng = cols // group
    kw = _scheme_kw(scheme, init_scale, rows, ng)
    params = params if params is not None else _unit_params(weight, group)
    v, a, b = _flat(params, rows, cols, group)
    w = weight.to(torch.bfloat16).contiguous()
    scale = torch.empty((rows, ng), dtype=torch.float32, device=weight.device)
    zp = torch.empty_like(scale)
    kernels.fq_forward(w, v, a, b, bits=scheme.bits, group=group, eps=eps, scale=scale, zp=zp, **kw)
    bits = scheme.bits
    packable = (cols % (32 // bits) == 0) if 32 % bits == 0 else (cols % 32 == 0)
    if not packable:
        raise SchemeError(f"in_features={cols} does not tile {bits}-bit words")
    _, _, _, codes = kernels.pack_mlx(w, v, a, b, bits=bits, group=group, eps=eps, want_codes=True,
                                      **kw)
    zero_point = None if kw["symmetric"] else zp.view(rows, ng, 1)
    return codes.view(rows, ng, group), scale.view(rows, ng, 1), zero_point


def dequantize(codes: torch.Tensor, scale: torch.Tensor, zero_point: torch.Tensor | None,
               shape: tuple[int, int], scheme: QuantScheme) -> torch.Tensor:
    """``scale * codes`` (symmetric) or ``scale * (codes - zero_point)``, float32, ungrouped."""
    if zero_point is None:
        out = scale.float() * codes.float()
    else:
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
