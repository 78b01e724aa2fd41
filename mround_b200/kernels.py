"""Torch-tensor front end of the native kernels (the ``mround/kernels`` slot).

Each function validates the tensors it is handed (device, dtype, contiguity,
shape), passes raw pointers and the current CUDA stream to one C entry point
of ``libmround_b200.so``, and returns without synchronizing.  Every function
runs only on the GPU: a CPU tensor is refused with ``PlatformError``.
"""

from __future__ import annotations

import torch

from mround_b200._native import check, lib
from mround_b200.exceptions import PlatformError, SchemeError

__all__ = [
    "LossWorkspace",
    "colsumsq_split",
    "deltaloss",
    "fq_forward",
    "gemm",
    "gemm_batched",
    "gemm_tf32",
    "loss_apply",
    "loss_hist_pass",
    "loss_outlier",
    "loss_select_digit",
    "pack_mlx",
    "round_tf32",
    "scale_search",
    "split_bf16",
    "ste_signsgd",
]

DEVICE_GROUPS = (8, 16, 32, 64, 128, 256)

# Kernel launches issued through this module (bench.py reports them), and an
# optional timing hook for GEMM launches: when ``GEMM_EVENTS`` is a list, each
# K3 launch appends ``(start_event, end_event, algorithmic_flops, cost)``, cost
# being the launch's tensor work in bf16 products per algorithmic product
# (1-3 for the bf16 splits, TF32_PRODUCT_COST for one tf32 product).
LAUNCHES = [0]
GEMM_EVENTS: list | None = None


def _count(n: int = 1) -> None:
    LAUNCHES[0] += n


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None, dtype: torch.dtype, name: str, numel: int | None = None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise PlatformError(f"{name} must be a CUDA tensor (the tuning path has no CPU fallback)")
    if t.dtype != dtype:
        raise SchemeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise SchemeError(f"{name} must be contiguous")
    if numel is not None and t.numel() != numel:
        raise SchemeError(f"{name} has {t.numel()} elements, expected {numel}")
    return t.data_ptr()


def _weight_args(w, v, alpha, beta, group):
    if w.dim() != 2:
        raise SchemeError(f"expected a 2-D weight, got shape {tuple(w.shape)}")
    rows, cols = w.shape
    if group not in DEVICE_GROUPS or cols % group:
        raise SchemeError(f"group {group} is not supported on the device for {cols} columns")
    ng = rows * (cols // group)
    return (
        rows,
        cols,
        _ptr(w, torch.bfloat16, "w", rows * cols),
        _ptr(v, torch.float32, "v", rows * cols),
        _ptr(alpha, torch.float32, "alpha", ng),
        _ptr(beta, torch.float32, "beta", ng),
    )


def _scheme_args(symmetric: bool, init_scale, ng: int):
    if init_scale is not None and not symmetric:
        raise SchemeError("a searched scale belongs to a symmetric scheme")
    return int(bool(symmetric)), _ptr(init_scale, torch.float32, "init_scale", ng)


def fq_forward(w, v, alpha, beta, *, bits: int, group: int, eps: float, wq_hi=None, wq_lo=None,
               wq_f32=None, wq_t32=None, scale=None, zp=None, symmetric: bool = False,
               init_scale=None) -> None:
    """K1: write the fake-quantized weight (bf16 hi/lo split, float32 and/or
    its tf32 rounding -- the backward GEMMs' operand).

    ``symmetric`` selects the symmetric code range; ``init_scale`` (float32,
    one per group) the searched scale.
    """
    rows, cols, pw, pv, pa, pb = _weight_args(w, v, alpha, beta, group)
    n, ng = rows * cols, rows * (cols // group)
    sym, pinit = _scheme_args(symmetric, init_scale, ng)
    status = lib().mr_fq_forward(
        pw, pv, pa, pb, rows, cols, group, bits, sym, pinit, eps,
        _ptr(wq_hi, torch.bfloat16, "wq_hi", n), _ptr(wq_lo, torch.bfloat16, "wq_lo", n),
        _ptr(wq_f32, torch.float32, "wq_f32", n), _ptr(wq_t32, torch.float32, "wq_t32", n),
        _ptr(scale, torch.float32, "scale", ng),
        _ptr(zp, torch.float32, "zp", ng), _stream())
    check(status, "mr_fq_forward")
    _count()


def ste_signsgd(gq, w, v, alpha, beta, *, bits: int, group: int, eps: float, lr: float,
                lo: float, hi: float, update: bool = True, gv=None, galpha=None, gbeta=None,
                wq_hi=None, wq_lo=None, wq_t32=None, symmetric: bool = False,
                init_scale=None) -> None:
    """K2: straight-through gradients, then (if ``update``) the signed step in
    place and the next step's operands (bf16 hi/lo, tf32)."""
    rows, cols, pw, pv, pa, pb = _weight_args(w, v, alpha, beta, group)
    n, ng = rows * cols, rows * (cols // group)
    sym, pinit = _scheme_args(symmetric, init_scale, ng)
    status = lib().mr_ste_signsgd(
        _ptr(gq, torch.float32, "gq", n), pw, pv, pa, pb, rows, cols, group, bits, sym, pinit,
        eps, lr, lo,
        hi, int(bool(update)), _ptr(gv, torch.float32, "gv", n),
        _ptr(galpha, torch.float32, "galpha", ng), _ptr(gbeta, torch.float32, "gbeta", ng),
        _ptr(wq_hi, torch.bfloat16, "wq_hi", n), _ptr(wq_lo, torch.bfloat16, "wq_lo", n),
        _ptr(wq_t32, torch.float32, "wq_t32", n), _stream())
    check(status, "mr_ste_signsgd")
    _count()


def ste_signsgd_codes(gq, w, v, alpha, beta, *, bits: int, group: int, eps: float, lr: float,
                      lo: float, hi: float, codes, qscale, qzp=None, symmetric: bool = False,
                      init_scale=None) -> None:
    """K2's signed step, writing the next step's codes (uint8, one per weight)
    and per-group scale / zero point instead of the operands."""
    rows, cols, pw, pv, pa, pb = _weight_args(w, v, alpha, beta, group)
    n, ng = rows * cols, rows * (cols // group)
    sym, pinit = _scheme_args(symmetric, init_scale, ng)
    status = lib().mr_ste_signsgd_codes(
        _ptr(gq, torch.float32, "gq", n), pw, pv, pa, pb, rows, cols, group, bits, sym, pinit,
        eps, lr, lo, hi, _ptr(codes, torch.uint8, "codes", n),
        _ptr(qscale, torch.float32, "qscale", ng), _ptr(qzp, torch.float32, "qzp", ng), _stream())
    check(status, "mr_ste_signsgd_codes")
    _count()


MAX_K2_SEGMENTS = 8


def ste_signsgd_segments(segments: list[dict], *, group: int, eps: float,
                         symmetric: bool = False) -> None:
    """K2's signed step over up to ``MAX_K2_SEGMENTS`` matrices in one launch.

    Each segment is a dict with ``gq, w, v, alpha, beta`` (tensors), ``bits``,
    ``lr``, ``lo``, ``hi`` and optional ``init_scale``, and either the next
    operands (``wq_hi``, ``wq_lo``, ``wq_t32``) or the next codes (``codes``,
    ``qscale``, ``qzp``).  Bit for bit one ``ste_signsgd(update=True)`` /
    ``ste_signsgd_codes`` per segment."""
    from mround_b200._native import K2Segment

    if not 1 <= len(segments) <= MAX_K2_SEGMENTS:
        raise SchemeError(f"1 to {MAX_K2_SEGMENTS} segments per launch, got {len(segments)}")
    table = (K2Segment * len(segments))()
    for i, sg in enumerate(segments):
        rows, cols, pw, pv, pa, pb = _weight_args(sg["w"], sg["v"], sg["alpha"], sg["beta"], group)
        n, ng = rows * cols, rows * (cols // group)
        init = sg.get("init_scale")
        _, pinit = _scheme_args(symmetric, init, ng)
        table[i] = K2Segment(
            _ptr(sg["gq"], torch.float32, "gq", n), pw, pv, pa, pb, pinit, rows, cols, sg["bits"],
            sg["lr"], sg["lo"], sg["hi"],
            _ptr(sg.get("wq_hi"), torch.bfloat16, "wq_hi", n),
            _ptr(sg.get("wq_lo"), torch.bfloat16, "wq_lo", n),
            _ptr(sg.get("wq_t32"), torch.float32, "wq_t32", n),
            _ptr(sg.get("codes"), torch.uint8, "codes", n),
            _ptr(sg.get("qscale"), torch.float32, "qscale", ng),
            _ptr(sg.get("qzp"), torch.float32, "qzp", ng))
    status = lib().mr_ste_signsgd_segments(table, len(segments), group, int(bool(symmetric)), eps,
                                           _stream())
    check(status, "mr_ste_signsgd_segments")
    _count()


def dequant_split(codes, qscale, qzp, *, group: int, symmetric: bool, wq_hi=None, wq_lo=None,
                  wq_t32=None) -> None:
    """Operands (bf16 hi/lo, tf32) from codes and per-group scale / zero point."""
    rows, cols = codes.shape
    n, ng = rows * cols, rows * (cols // group)
    status = lib().mr_dequant_split(
        _ptr(codes, torch.uint8, "codes", n), _ptr(qscale, torch.float32, "qscale", ng),
        _ptr(qzp, torch.float32, "qzp", ng), rows, cols, group, int(bool(symmetric)),
        _ptr(wq_hi, torch.bfloat16, "wq_hi", n), _ptr(wq_lo, torch.bfloat16, "wq_lo", n),
        _ptr(wq_t32, torch.float32, "wq_t32", n), _stream())
    check(status, "mr_dequant_split")
    _count()


def pack_mlx(w, v, alpha, beta, *, bits: int, group: int, eps: float, want_codes: bool = False,
             symmetric: bool = False, init_scale=None):
    """K5: ``(packed uint32 as int32, scales bf16, biases bf16, codes or None)``.

    Codes are uint8, or int8 under a symmetric scheme.
    """
    rows, cols, pw, pv, pa, pb = _weight_args(w, v, alpha, beta, group)
    sym, pinit = _scheme_args(symmetric, init_scale, rows * (cols // group))
    if 32 % bits == 0:
        if cols % (32 // bits):
            raise SchemeError(f"cols={cols} does not tile {bits}-bit words")
        words = cols // (32 // bits)
    else:
        if cols % 32:
            raise SchemeError(f"cols={cols} is not a multiple of 32 at {bits} bits")
        words = cols // 32 * bits
    dev = w.device
    packed = torch.empty((rows, words), dtype=torch.int32, device=dev)
    scales = torch.empty((rows, cols // group), dtype=torch.bfloat16, device=dev)
    biases = torch.empty_like(scales)
    code_dtype = torch.int8 if sym else torch.uint8
    codes = torch.empty((rows, cols), dtype=code_dtype, device=dev) if want_codes else None
    status = lib().mr_pack_mlx(
        pw, pv, pa, pb, rows, cols, group, bits, sym, pinit, eps, packed.data_ptr(), scales.data_ptr(),
        biases.data_ptr(), None if codes is None else codes.data_ptr(), _stream())
    check(status, "mr_pack_mlx")
    _count()
    return packed, scales, biases, codes


class LossWorkspace:
    """Device scratch of the loss kernels (selection state, histogram, partial sums)."""

    def __init__(self, device: torch.device | str = "cuda") -> None:
        nbytes = int(lib().mr_loss_workspace_bytes())
        self.buffer = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        self.loss = torch.zeros((), dtype=torch.float64, device=device)
        self.thr = torch.zeros((), dtype=torch.float32, device=device)
        self.hist = torch.zeros(2048, dtype=torch.int32, device=device)

    @property
    def ptr(self) -> int:
        return self.buffer.data_ptr()


def loss_outlier(pred, target, ws: LossWorkspace, *, suppress: bool, denom: float, k: int,
                 grad=None, threshold: float | None = None) -> None:
    """K4 single-device: loss into ``ws.loss``, threshold into ``ws.thr``, grad optional."""
    n = pred.numel()
    pp = _ptr(pred, torch.float32, "pred")
    pt = _ptr(target, torch.float32, "target", n)
    status = lib().mr_loss_outlier(
        pp, pt, n, int(k), int(bool(suppress)), float(denom),
        -1.0 if threshold is None else float(threshold), _ptr(grad, torch.float32, "grad", n),
        ws.loss.data_ptr(), ws.thr.data_ptr(), ws.ptr, _stream())
    check(status, "mr_loss_outlier")
    _count(8 if (suppress and threshold is None) else 2)


def loss_hist_pass(pred, target, ws: LossWorkspace, pass_index: int) -> torch.Tensor:
    """One radix pass of the threshold selection; returns this rank's histogram."""
    n = pred.numel()
    status = lib().mr_loss_hist_pass(
        _ptr(pred, torch.float32, "pred"), _ptr(target, torch.float32, "target", n), n,
        int(pass_index), ws.ptr, ws.hist.data_ptr(), _stream())
    check(status, "mr_loss_hist_pass")
    _count()
    return ws.hist


def loss_select_digit(ws: LossWorkspace, k: int, pass_index: int) -> None:
    """Narrow the selection with the (possibly all-reduced) histogram in ``ws.hist``."""
    status = lib().mr_loss_select_digit(ws.hist.data_ptr(), int(k), int(pass_index), ws.ptr,
                                        ws.thr.data_ptr(), _stream())
    check(status, "mr_loss_select_digit")
    _count()


def loss_apply(pred, target, ws: LossWorkspace, *, suppress: bool, denom: float, grad=None) -> None:
    """Loss and gradient with the threshold already in ``ws.thr``."""
    n = pred.numel()
    status = lib().mr_loss_apply(
        _ptr(pred, torch.float32, "pred"), _ptr(target, torch.float32, "target", n), n,
        float(denom), ws.thr.data_ptr(), int(bool(suppress)), _ptr(grad, torch.float32, "grad", n),
        ws.loss.data_ptr(), ws.ptr, _stream())
    check(status, "mr_loss_apply")
    _count(2)


def deltaloss(g, w, *, bits: list[int] | tuple[int, ...], group: int, eps: float, out,
              symmetric: bool = False, grids=None) -> None:
    """K6: ``out[j] += sum |g * (RTN_bits[j](w) - w)|`` (``out`` float64, on device).

    ``grids``: one searched scale tensor per width (float32, one per group) for
    a searched scheme, else None.
    """
    import ctypes

    if w.dim() != 2:
        raise SchemeError("expected a 2-D weight")
    rows, cols = w.shape
    if grids is not None and not symmetric:
        raise SchemeError("searched grids belong to a symmetric scheme")
    widths = (ctypes.c_int * len(bits))(*[int(b) for b in bits])
    grid_arr = None
    if grids is not None:
        if len(grids) != len(bits):
            raise SchemeError("one searched grid per width")
        ptrs = [_ptr(gr, torch.float32, "grid", rows * (cols // group)) for gr in grids]
        grid_arr = ctypes.cast((ctypes.c_void_p * len(ptrs))(*ptrs), ctypes.c_void_p)
    status = lib().mr_deltaloss(
        _ptr(g, torch.float32, "g", rows * cols), _ptr(w, torch.bfloat16, "w", rows * cols),
        rows, cols, group, ctypes.cast(widths, ctypes.c_void_p), len(bits), int(bool(symmetric)),
        grid_arr, eps, _ptr(out, torch.float64, "out", len(bits)), _stream())
    check(status, "mr_deltaloss")
    _count()


def scale_search(w, *, bits: int, group: int, candidates, importance=None, out=None):
    """K8: the searched scale of every group of ``w`` (bf16 (rows, cols)).

    ``candidates``: effective ranges in evaluation order (anchor first), any
    sequence of floats, converted to float32.  ``importance``: float32 (cols,)
    or None.  Returns float32 (rows, cols // group).
    """
    import ctypes

    if w.dim() != 2:
        raise SchemeError("expected a 2-D weight")
    rows, cols = w.shape
    if group not in DEVICE_GROUPS or cols % group:
        raise SchemeError(f"group {group} is not supported on the device for {cols} columns")
    cands = [float(c) for c in candidates]
    if not 1 <= len(cands) <= 256:
        raise SchemeError("1 to 256 candidates")
    arr = (ctypes.c_float * len(cands))(*cands)
    if out is None:
        out = torch.empty((rows, cols // group), dtype=torch.float32, device=w.device)
    status = lib().mr_scale_search(
        _ptr(w, torch.bfloat16, "w", rows * cols), rows, cols, group, bits,
        ctypes.cast(arr, ctypes.c_void_p), len(cands),
        _ptr(importance, torch.float32, "importance", cols),
        _ptr(out, torch.float32, "out", rows * (cols // group)), _stream())
    check(status, "mr_scale_search")
    _count()
    return out


def colsumsq_split(hi, lo, out) -> None:
    """``out[c] += sum_r (hi + lo)[r, c]^2`` for a float32 activation in bf16 parts."""
    if hi.dim() != 2:
        raise SchemeError("expected a 2-D activation")
    rows, cols = hi.shape
    status = lib().mr_colsumsq_split(
        _ptr(hi, torch.bfloat16, "hi", rows * cols),
        _ptr(lo, torch.bfloat16, "lo", rows * cols) if lo is not None else None, rows, cols,
        _ptr(out, torch.float32, "out", cols), _stream())
    check(status, "mr_colsumsq_split")
    _count()


def split_bf16(x, hi=None, lo=None, *, want_lo: bool = True):
    """float32 -> (bf16 hi, bf16 lo); ``hi + lo`` carries 16 significant bits."""
    n = x.numel()
    if hi is None:
        hi = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    if lo is None and want_lo:
        lo = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    status = lib().mr_split_bf16(_ptr(x, torch.float32, "x"), n, _ptr(hi, torch.bfloat16, "hi", n),
                                 _ptr(lo, torch.bfloat16, "lo", n) if lo is not None else None,
                                 _stream())
    check(status, "mr_split_bf16")
    _count()
    return hi, lo


def gemm(a_hi, a_lo, b_hi, b_lo, c, *, m: int, n: int, k: int, a_kmajor: bool, b_kmajor: bool,
         lda: int, ldb: int, ldc: int, precision: int, bias=None, accumulate: bool = False) -> None:
    """K3: ``C[m, n] (+)= sum_k A[m, k] B[n, k]`` on the tcgen05 tensor cores."""
    timing = GEMM_EVENTS is not None
    if timing:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
    status = lib().mr_gemm(
        _ptr(a_hi, torch.bfloat16, "a_hi"), _ptr(a_lo, torch.bfloat16, "a_lo"), lda, int(a_kmajor),
        _ptr(b_hi, torch.bfloat16, "b_hi"), _ptr(b_lo, torch.bfloat16, "b_lo"), ldb, int(b_kmajor),
        _ptr(c, torch.float32, "c"), ldc, _ptr(bias, torch.float32, "bias"), int(bool(accumulate)),
        m, n, k, precision, _stream())
    check(status, "mr_gemm")
    _count()
    if timing:
        end.record()
        GEMM_EVENTS.append((start, end, 2.0 * m * n * k, precision))


def gemm_rs(a_hi, a_lo, b_hi, b_lo, *, m: int, n: int, k: int, a_kmajor: bool, b_kmajor: bool,
            lda: int, ldb: int, precision: int, dst_ptrs, ldd: int, rows_per_rank: int,
            flag_ptrs, done, epoch: int) -> None:
    """K3 whose rows go to their owner ranks over NVLink (fused reduce-scatter).

    ``dst_ptrs[o]`` / ``flag_ptrs[o]``: device addresses (ints) of rank o's
    slot and flag for this source rank; ``done``: this rank's zeroed int32
    counter; ``epoch``: the exchange's step number (> 0, increasing).
    """
    import ctypes

    world = len(dst_ptrs)
    if len(flag_ptrs) != world:
        raise SchemeError("one flag per destination rank")
    timing = GEMM_EVENTS is not None
    if timing:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
    dsts = (ctypes.c_void_p * world)(*dst_ptrs)
    flags = (ctypes.c_void_p * world)(*flag_ptrs)
    status = lib().mr_gemm_rs(
        _ptr(a_hi, torch.bfloat16, "a_hi"), _ptr(a_lo, torch.bfloat16, "a_lo"), lda, int(a_kmajor),
        _ptr(b_hi, torch.bfloat16, "b_hi"), _ptr(b_lo, torch.bfloat16, "b_lo"), ldb, int(b_kmajor),
        m, n, k, precision, ctypes.cast(dsts, ctypes.c_void_p), ldd, rows_per_rank,
        ctypes.cast(flags, ctypes.c_void_p), world, _ptr(done, torch.int32, "done", 1), int(epoch),
        _stream())
    check(status, "mr_gemm_rs")
    _count()
    if timing:
        end.record()
        GEMM_EVENTS.append((start, end, 2.0 * m * n * k, precision))


# tensor time of one tf32 product, in bf16 products (tf32 runs at half the rate)
TF32_PRODUCT_COST = 2


def gemm_tile(*, m: int, n: int, k: int, precision: int, a_kmajor: bool, b_kmajor: bool,
              batch: int = 1, causal: int = 0) -> tuple[int, int]:
    """The output tile (rows, columns) K3 uses for this shape."""
    args = (m, n, k, batch, precision, int(a_kmajor), int(b_kmajor), causal)
    rows, width = int(lib().mr_gemm_tile_m(*args)), int(lib().mr_gemm_tile_n(*args))
    check(min(rows, width, 0), "mr_gemm_tile")
    return rows, width


def gemm_tile_n(*, m: int, n: int, k: int, precision: int, a_kmajor: bool, b_kmajor: bool,
                batch: int = 1, causal: int = 0) -> int:
    """The output tile width (128, 224 or 256) K3 uses for this shape."""
    return gemm_tile(m=m, n=n, k=k, precision=precision, a_kmajor=a_kmajor, b_kmajor=b_kmajor,
                     batch=batch, causal=causal)[1]


def gemm_tf32(a, b, c, *, m: int, n: int, k: int, a_kmajor: bool, b_kmajor: bool, lda: int,
              ldb: int, ldc: int, bias=None, accumulate: bool = False) -> None:
    """K3, one tf32 product: ``C[m, n] (+)= sum_k A[m, k] B[n, k]`` with float32
    operands already rounded to tf32 (``round_tf32`` or a kernel's t32 output)."""
    timing = GEMM_EVENTS is not None
    if timing:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
    status = lib().mr_gemm_tf32(
        _ptr(a, torch.float32, "a"), lda, int(a_kmajor), _ptr(b, torch.float32, "b"), ldb,
        int(b_kmajor), _ptr(c, torch.float32, "c"), ldc, _ptr(bias, torch.float32, "bias"),
        int(bool(accumulate)), m, n, k, _stream())
    check(status, "mr_gemm_tf32")
    _count()
    if timing:
        end.record()
        GEMM_EVENTS.append((start, end, 2.0 * m * n * k, TF32_PRODUCT_COST))


def gemm_rs_tf32(a, b, *, m: int, n: int, k: int, a_kmajor: bool, b_kmajor: bool, lda: int,
                 ldb: int, dst_ptrs, ldd: int, rows_per_rank: int, flag_ptrs, done,
                 epoch: int) -> None:
    """``gemm_rs`` with one tf32 product of float32 operands."""
    import ctypes

    world = len(dst_ptrs)
    if len(flag_ptrs) != world:
        raise SchemeError("one flag per destination rank")
    timing = GEMM_EVENTS is not None
    if timing:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
    dsts = (ctypes.c_void_p * world)(*dst_ptrs)
    flags = (ctypes.c_void_p * world)(*flag_ptrs)
    status = lib().mr_gemm_rs_tf32(
        _ptr(a, torch.float32, "a"), lda, int(a_kmajor), _ptr(b, torch.float32, "b"), ldb,
        int(b_kmajor), m, n, k, ctypes.cast(dsts, ctypes.c_void_p), ldd, rows_per_rank,
        ctypes.cast(flags, ctypes.c_void_p), world, _ptr(done, torch.int32, "done", 1), int(epoch),
        _stream())
    check(status, "mr_gemm_rs_tf32")
    _count()
    if timing:
        end.record()
        GEMM_EVENTS.append((start, end, 2.0 * m * n * k, TF32_PRODUCT_COST))


def reduce_slots(slots, flags, epoch: int, out) -> None:
    """Wait for every source's flag to reach ``epoch``, then out = sum of the
    ``slots`` (world, ...) in rank order."""
    world = slots.shape[0]
    n = out.numel()
    status = lib().mr_reduce_slots(
        _ptr(slots, torch.float32, "slots"), slots[0].numel(), n, world,
        _ptr(flags, torch.int64, "flags", world), int(epoch), _ptr(out, torch.float32, "out", n),
        _stream())
    check(status, "mr_reduce_slots")
    _count()


def peer_send(dst_ptr: int, src, flag_ptr: int, epoch: int) -> None:
    """Copy ``src`` (contiguous float32 rows) to ``dst_ptr`` with the copy
    engine, then release ``epoch`` into the flag at ``flag_ptr`` -- both on the
    current stream."""
    if not src.is_contiguous():
        raise SchemeError("peer_send needs contiguous rows")
    status = lib().mr_peer_send(dst_ptr, _ptr(src, torch.float32, "src"), src.numel() * 4,
                                flag_ptr, int(epoch), _stream())
    check(status, "mr_peer_send")
    _count()


def causal_fraction(causal: int, m: int, n: int, k: int, seq: int, bk: int = 64) -> float:
    """Share of the dense tile work a causal mode of K3 actually computes
    (mirrors the kernel's tile and K-tile predicates; BM = 128, K slices of
    ``bk``: 64 when both operands are MN-major, else 32)."""
    if not causal:
        return 1.0
    bm = 128
    bn = 128 if n <= 128 else 256
    m_tiles = -(-m // bm)
    k_tiles = -(-k // bk)
    n_tiles = -(-n // bn)
    done = 0
    for tm in range(m_tiles):
        m0 = tm * bm
        if causal == 1:
            done += min(n_tiles, (m0 % seq + bm - 1) // bn + 1) * k_tiles
        elif causal == 2:
            done += min(k_tiles, (m0 % seq + bm + bk - 1) // bk) * n_tiles
        else:
            done += sum(1 for kt in range(k_tiles) if (kt * bk) % seq + bk - 1 >= m0) * n_tiles
    return done / (m_tiles * n_tiles * k_tiles)


def gemm_batched(a_hi, a_lo, b_hi, b_lo, c, *, m: int, n: int, k: int, batch: int, a_kmajor: bool,
                 b_kmajor: bool, lda: int, ldb: int, ldc: int, stride_a: int, stride_b: int,
                 stride_c: int, precision: int, accumulate: bool = False, causal: int = 0,
                 seq: int = 0) -> None:
    """K3 over ``batch`` equally shaped problems in one launch (``causal``: see the header)."""
    timing = GEMM_EVENTS is not None
    if timing:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
    status = lib().mr_gemm_batched(
        _ptr(a_hi, torch.bfloat16, "a_hi"), _ptr(a_lo, torch.bfloat16, "a_lo"), lda, stride_a,
        int(a_kmajor), _ptr(b_hi, torch.bfloat16, "b_hi"), _ptr(b_lo, torch.bfloat16, "b_lo"), ldb,
        stride_b, int(b_kmajor), _ptr(c, torch.float32, "c"), ldc, stride_c, None,
        int(bool(accumulate)), m, n, k, batch, precision, int(causal), int(seq), _stream())
    check(status, "mr_gemm_batched")
    _count()
    if timing:
        end.record()
        frac = causal_fraction(causal, m, n, k, seq, 64 if not (a_kmajor or b_kmajor) else 32)
        GEMM_EVENTS.append((start, end, 2.0 * m * n * k * batch * frac, precision))


# ---------------------------------------------------------------- block ops
def _pair(shape, device):
    return (torch.empty(shape, dtype=torch.bfloat16, device=device),
            torch.empty(shape, dtype=torch.bfloat16, device=device))


def _t32(shape, device, want: bool):
    return torch.empty(shape, dtype=torch.float32, device=device) if want else None


def rmsnorm_split(x, w, eps: float, *, t32: bool = False):
    """x (T, h) float32, w (h,) bf16 -> (hi, lo, rstd, tf32 copy or None)."""
    t, h = x.shape
    hi, lo = _pair((t, h), x.device)
    tt = _t32((t, h), x.device, t32)
    rstd = torch.empty(t, dtype=torch.float32, device=x.device)
    st = lib().mr_rmsnorm_split(_ptr(x, torch.float32, "x"), _ptr(w, torch.bfloat16, "w", h), t, h,
                                eps, hi.data_ptr(), lo.data_ptr(),
                                _ptr(tt, torch.float32, "t32", t * h), rstd.data_ptr(), _stream())
    check(st, "mr_rmsnorm_split")
    _count()
    return hi, lo, rstd, tt


def rmsnorm_bwd_split(dy, x, w, rstd, resid, *, split: bool = True, t32: bool = False, out=None):
    """RMSNorm backward plus ``resid`` (or None): ``(hi, lo)`` when ``split``,
    the tf32-rounded copy when ``t32``, and the float32 gradient written to
    ``out`` when given.  Returns (hi, lo, t32) with None for what was not asked."""
    t, h = x.shape
    hi, lo = _pair((t, h), x.device) if split else (None, None)
    tt = _t32((t, h), x.device, t32)
    st = lib().mr_rmsnorm_bwd_split(
        _ptr(dy, torch.float32, "dy", t * h), _ptr(x, torch.float32, "x"),
        _ptr(w, torch.bfloat16, "w", h), _ptr(rstd, torch.float32, "rstd", t),
        _ptr(resid, torch.float32, "resid", t * h), t, h, None if hi is None else hi.data_ptr(),
        None if lo is None else lo.data_ptr(), _ptr(tt, torch.float32, "t32", t * h),
        _ptr(out, torch.float32, "out", t * h), _stream())
    check(st, "mr_rmsnorm_bwd_split")
    _count()
    return hi, lo, tt


def rope_split(qkv, cos, sin, b: int, s: int, hq: int, hkv: int, d: int):
    dev = qkv.device
    q = _pair((b, hq, s, d), dev)
    k = _pair((b, hkv, s, d), dev)
    v = _pair((b, hkv, s, d), dev)
    st = lib().mr_rope_split(_ptr(qkv, torch.float32, "qkv", b * s * (hq + 2 * hkv) * d),
                             _ptr(cos, torch.float32, "cos", s * d // 2),
                             _ptr(sin, torch.float32, "sin", s * d // 2), b, s, hq, hkv, d,
                             q[0].data_ptr(), q[1].data_ptr(), k[0].data_ptr(), k[1].data_ptr(),
                             v[0].data_ptr(), v[1].data_ptr(), _stream())
    check(st, "mr_rope_split")
    _count()
    return q, k, v


def rope_bwd_split(dq, dk, dv, cos, sin, b: int, s: int, hq: int, hkv: int, d: int, *,
                   split: bool = True, t32: bool = False):
    """The qkv-row gradient as (hi, lo, tf32 copy), None for what was not asked."""
    shape = (b * s, (hq + 2 * hkv) * d)
    hi, lo = _pair(shape, dq.device) if split else (None, None)
    tt = _t32(shape, dq.device, t32)
    st = lib().mr_rope_bwd_split(_ptr(dq, torch.float32, "dq"), _ptr(dk, torch.float32, "dk"),
                                 _ptr(dv, torch.float32, "dv"), _ptr(cos, torch.float32, "cos"),
                                 _ptr(sin, torch.float32, "sin"), b, s, hq, hkv, d,
                                 None if hi is None else hi.data_ptr(),
                                 None if lo is None else lo.data_ptr(),
                                 _ptr(tt, torch.float32, "t32", shape[0] * shape[1]), _stream())
    check(st, "mr_rope_bwd_split")
    _count()
    return hi, lo, tt


def heads_split(src, b: int, s: int, h: int, d: int, *, merge: bool, t32: bool = False):
    """Head layout change as (hi, lo, tf32 copy or None)."""
    shape = (b * s, h * d) if merge else (b, h, s, d)
    hi, lo = _pair(shape, src.device)
    tt = _t32(shape, src.device, t32)
    st = lib().mr_heads_split(_ptr(src, torch.float32, "src", b * s * h * d), b, s, h, d, int(merge),
                              hi.data_ptr(), lo.data_ptr(),
                              _ptr(tt, torch.float32, "t32", b * s * h * d), _stream())
    check(st, "mr_heads_split")
    _count()
    return hi, lo, tt


def swiglu_split(gu, t: int, i: int, *, t32: bool = False):
    """silu(g) * u as (hi, lo, tf32 copy or None)."""
    hi, lo = _pair((t, i), gu.device)
    tt = _t32((t, i), gu.device, t32)
    st = lib().mr_swiglu_split(_ptr(gu, torch.float32, "gu", t * 2 * i), t, i, hi.data_ptr(),
                               lo.data_ptr(), _ptr(tt, torch.float32, "t32", t * i), _stream())
    check(st, "mr_swiglu_split")
    _count()
    return hi, lo, tt


def swiglu_bwd_split(dact, gu, t: int, i: int, *, split: bool = True, t32: bool = False):
    """The gate|up gradient as (hi, lo, tf32 copy), None for what was not asked."""
    hi, lo = _pair((t, 2 * i), gu.device) if split else (None, None)
    tt = _t32((t, 2 * i), gu.device, t32)
    st = lib().mr_swiglu_bwd_split(_ptr(dact, torch.float32, "dact", t * i),
                                   _ptr(gu, torch.float32, "gu", t * 2 * i), t, i,
                                   None if hi is None else hi.data_ptr(),
                                   None if lo is None else lo.data_ptr(),
                                   _ptr(tt, torch.float32, "t32", t * 2 * i), _stream())
    check(st, "mr_swiglu_bwd_split")
    _count()
    return hi, lo, tt


def ce_grad_split(logits, labels, scale: float):
    """(softmax(logits) - onehot(labels)) * scale per row, as bf16 (hi, lo)."""
    rows, vocab = logits.shape
    hi, lo = _pair((rows, vocab), logits.device)
    if labels.dtype != torch.int64 or not labels.is_contiguous() or labels.numel() != rows:
        raise SchemeError("labels must be a contiguous int64 tensor of one label per row")
    st = lib().mr_ce_grad_split(_ptr(logits, torch.float32, "logits"), labels.data_ptr(), rows,
                                vocab, float(scale), hi.data_ptr(), lo.data_ptr(), _stream())
    check(st, "mr_ce_grad_split")
    _count()
    return hi, lo


def round_tf32(x, out=None):
    """float32 -> its tf32 rounding (round to nearest, ties away), float32."""
    n = x.numel()
    if out is None:
        out = torch.empty_like(x)
    st = lib().mr_round_tf32(_ptr(x, torch.float32, "x"), n, _ptr(out, torch.float32, "out", n),
                             _stream())
    check(st, "mr_round_tf32")
    _count()
    return out


def softmax_causal_split(scores, rows: int, s: int, scale: float, band: bool = False):
    """Causal softmax (row r at position r % s) as bf16 hi/lo parts; ``scores``
    is left unchanged."""
    hi, lo = _pair(scores.shape, scores.device)
    st = lib().mr_softmax_causal_split(_ptr(scores, torch.float32, "scores", rows * s), rows, s,
                                       float(scale), int(band), hi.data_ptr(), lo.data_ptr(),
                                       _stream())
    check(st, "mr_softmax_causal_split")
    _count()
    return hi, lo


def softmax_bwd_split(dp, p, rows: int, s: int, scale: float, band: bool = False):
    """Softmax backward from dP (float32) and P as its (hi, lo) parts."""
    hi, lo = _pair(dp.shape, dp.device)
    st = lib().mr_softmax_bwd_split(_ptr(dp, torch.float32, "dp", rows * s),
                                    _ptr(p[0], torch.bfloat16, "p_hi", rows * s),
                                    _ptr(p[1], torch.bfloat16, "p_lo", rows * s), rows, s,
                                    float(scale), int(band), hi.data_ptr(), lo.data_ptr(),
                                    _stream())
    check(st, "mr_softmax_bwd_split")
    _count()
    return hi, lo
