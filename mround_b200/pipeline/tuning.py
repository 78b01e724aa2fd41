"""The per-block tuning step on one GPU (or one data-parallel rank).

One step of ``QuantizationRunner._tune`` (reference
mround/pipeline/runner.py:914-937) is, here:

1. forward of the block on the fake-quantized operands (K3 GEMMs for the
   linears and the attention products, K7 for norms, RoPE, softmax, SwiGLU);
2. K4: residual, exact outlier threshold (radix select; the histograms are
   all-reduced across data-parallel ranks), loss and dL/dout;
3. backward: K3 GEMMs for dX and dW; across data-parallel ranks each fused
   weight's dW is exchanged as soon as it is produced -- by default its rows
   go straight from the GEMM epilogue to their owner ranks over NVLink
   (``mr_gemm_rs``), or through the copy engines or an NCCL reduce-scatter;
4. K2 per tunable linear (on this rank's rows when the update is row-sharded):
   straight-through gradient, signed step, projection and -- fused into the
   same pass -- the next step's fake-quantized operand, all-gathered across
   ranks before the next forward reads it.

No host synchronisation happens inside a step: per-step losses stay on the
device and are read once per block.
"""

from __future__ import annotations

import dataclasses
import time

import torch

from mround_b200 import kernels
from mround_b200.core.quantizer import require_device_scheme
from mround_b200.core.scale_search import search_scales
from mround_b200.pipeline.block import TF32, DeviceBlock, FusedLinear, Precision
from mround_b200.pipeline.dist import DistContext
from mround_b200.schemes import QuantScheme, ScaleInit, Symmetry

__all__ = ["BlockTuner", "Member", "QuantizedLayer", "TunableLayer", "auto_exchange", "piece_bounds"]

OUTLIER_FRACTION = 0.001


def piece_bounds(size: int, pieces: int) -> list[tuple[int, int]]:
    """Contiguous, near-even runs (reference mround/pipeline/blocks.py:609-624)."""
    count = max(1, min(pieces, size))
    base, extra = divmod(size, count)
    bounds, start = [], 0
    for piece in range(count):
        stop = start + base + (1 if piece < extra else 0)
        bounds.append((start, stop))
        start = stop
    return bounds


@dataclasses.dataclass
class QuantizedLayer:
    """One committed layer, already in MLX's stored form.

    ``packed`` uint32 words (held as int32) (out, in*bits/32), ``scales`` and
    ``biases`` bf16 (out, n_groups), ``codes`` (out, in) when kept: uint8, or
    int8 under a symmetric scheme.
    """

    packed: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor
    scheme: QuantScheme
    shape: tuple[int, int]
    codes: torch.Tensor | None = None


@dataclasses.dataclass
class Member:
    path: str
    rows: tuple[int, int]
    scheme: QuantScheme
    group: int
    lr0: float


class TunableLayer:
    """V / alpha / beta of one fused weight and the operands derived from them.

    Members of one fused weight share the run's symmetry and scale
    initialisation; their widths may differ.  Under a searched scheme
    ``init_scale`` holds each group's searched scale (set by
    ``BlockTuner.search``) and the operand is formed only once it is set.
    """

    def __init__(self, layer: FusedLinear, members: list[Member], eps: float, *,
                 tf32: bool = False) -> None:
        """``tf32``: also keep the operand as tf32 values (``layer.wq_t32``),
        the B operand of a tf32 input-gradient GEMM."""
        self.layer = layer
        self.members = members
        self.eps = eps
        out, inn = layer.w.shape
        groups = {m.group for m in members}
        if len(groups) != 1:
            raise ValueError("members of one fused weight must share a group size")
        self.group = groups.pop()
        kinds = {(m.scheme.symmetry, m.scheme.scale_init) for m in members}
        if len(kinds) != 1:
            raise ValueError("members of one fused weight must share symmetry and scale_init")
        symmetry, scale_init = kinds.pop()
        self.symmetric = symmetry is Symmetry.SYMMETRIC
        self.searched = scale_init is ScaleInit.SEARCHED
        dev = layer.w.device
        self.v = torch.zeros((out, inn), dtype=torch.float32, device=dev)
        self.alpha = torch.ones((out, inn // self.group), dtype=torch.float32, device=dev)
        self.beta = torch.ones_like(self.alpha)
        self.init_scale = torch.zeros_like(self.alpha) if self.searched else None
        tuned_rows = sum(m.rows[1] - m.rows[0] for m in members)
        self.whole = tuned_rows == out  # every row is fake-quantized
        if self.whole:
            layer.wq_hi = torch.empty_like(layer.w)
            layer.wq_lo = torch.empty_like(layer.w)
        else:  # rows of untuned members stay exact
            layer.wq_hi = layer.w.clone()
            layer.wq_lo = torch.zeros_like(layer.w)
        # bf16 weights are exact in tf32: untuned rows keep the weight itself
        layer.wq_t32 = layer.w.float() if tf32 else None
        layer.grad = torch.empty((out, inn), dtype=torch.float32, device=dev)
        if not self.searched:
            self.requantize()

    def _slices(self, m: Member):
        r0, r1 = m.rows
        return (self.layer.w[r0:r1], self.v[r0:r1], self.alpha[r0:r1], self.beta[r0:r1])

    def _scheme_kw(self, m: Member) -> dict:
        r0, r1 = m.rows
        return {"symmetric": self.symmetric,
                "init_scale": None if self.init_scale is None else self.init_scale[r0:r1]}

    def requantize(self) -> None:
        """K1 on every member: refresh the operand from the current parameters."""
        self.layer.ready()
        for m in self.members:
            w, v, a, b = self._slices(m)
            r0, r1 = m.rows
            kernels.fq_forward(w, v, a, b, bits=m.scheme.bits, group=m.group, eps=self.eps,
                               wq_hi=self.layer.wq_hi[r0:r1], wq_lo=self.layer.wq_lo[r0:r1],
                               wq_t32=self._t32_rows(r0, r1), **self._scheme_kw(m))

    def _t32_rows(self, r0: int, r1: int):
        t32 = self.layer.wq_t32
        return None if t32 is None else t32[r0:r1]

    def _rate(self, m: Member, step: int, iters: int) -> float:
        return m.lr0 * (1.0 - step / iters) if step < iters else 0.0

    def _segment(self, m: Member, step: int, iters: int, r0: int, r1: int, grad: torch.Tensor,
                 out: dict) -> dict:
        """One K2 segment: rows [r0, r1) of member ``m``, their summed gradient
        ``grad`` and where the next operands or codes go (``out``)."""
        lo_b, hi_b = m.scheme.coefficient_bounds
        seg = {"gq": grad, "w": self.layer.w[r0:r1], "v": self.v[r0:r1],
               "alpha": self.alpha[r0:r1], "beta": self.beta[r0:r1], "bits": m.scheme.bits,
               "lr": self._rate(m, step, iters), "lo": lo_b, "hi": hi_b,
               "init_scale": None if self.init_scale is None else self.init_scale[r0:r1]}
        seg.update(out)
        return seg

    def segments(self, step: int, iters: int) -> list[dict]:
        """K2 segments of every member (all rows) writing the layer's operands."""
        out = []
        for m in self.members:
            r0, r1 = m.rows
            out.append(self._segment(m, step, iters, r0, r1, self.layer.grad[r0:r1], {
                "wq_hi": self.layer.wq_hi[r0:r1], "wq_lo": self.layer.wq_lo[r0:r1],
                "wq_t32": self._t32_rows(r0, r1)}))
        return out

    @property
    def launch_key(self) -> tuple:
        """Tunables with equal keys can share one K2 launch."""
        return (self.group, self.symmetric, self.init_scale is not None)

    def run_segments(self, segments: list[dict]) -> None:
        """K2 over ``segments`` (of tunables sharing this one's ``launch_key``),
        ``kernels.MAX_K2_SEGMENTS`` to a launch."""
        for i in range(0, len(segments), kernels.MAX_K2_SEGMENTS):
            kernels.ste_signsgd_segments(segments[i:i + kernels.MAX_K2_SEGMENTS], group=self.group,
                                         eps=self.eps, symmetric=self.symmetric)

    def update_rows(self, step: int, iters: int, s0: int, s1: int, grad: torch.Tensor,
                    hi: torch.Tensor, lo: torch.Tensor, t32: torch.Tensor | None = None) -> None:
        """K2 on rows [s0, s1) only: ``grad`` holds the summed gradient of those
        rows, and the next step's operand rows go to ``hi``/``lo`` (and ``t32``)
        -- this rank's part of the all-gather.  V/alpha/beta of other rows are
        left as they are."""
        segs = []
        for m in self.members:
            r0, r1 = max(m.rows[0], s0), min(m.rows[1], s1)
            if r0 >= r1:
                continue
            a, b = r0 - s0, r1 - s0
            segs.append(self._segment(m, step, iters, r0, r1, grad[a:b], {
                "wq_hi": hi[a:b], "wq_lo": lo[a:b], "wq_t32": None if t32 is None else t32[a:b]}))
        if segs:
            self.run_segments(segs)

    def update_rows_codes(self, step: int, iters: int, s0: int, s1: int, grad: torch.Tensor,
                          codes: torch.Tensor, qscale: torch.Tensor,
                          qzp: torch.Tensor | None) -> None:
        """``update_rows`` writing the next step's codes and per-group scale /
        zero point of rows [s0, s1) instead of their operands (every row of
        the weight is tuned; ``dequant`` rebuilds the operands)."""
        gpr = self.layer.in_features // self.group
        segs = []
        for m in self.members:
            r0, r1 = max(m.rows[0], s0), min(m.rows[1], s1)
            if r0 >= r1:
                continue
            a, b = r0 - s0, r1 - s0
            segs.append(self._segment(m, step, iters, r0, r1, grad[a:b], {
                "codes": codes[a:b],
                "qscale": qscale.view(-1)[a * gpr:b * gpr].view(b - a, gpr),
                "qzp": None if qzp is None else qzp.view(-1)[a * gpr:b * gpr].view(b - a, gpr)}))
        if segs:
            self.run_segments(segs)

    def dequant(self, codes: torch.Tensor, qscale: torch.Tensor,
                qzp: torch.Tensor | None) -> None:
        """The whole weight's operands (bf16 hi/lo and the tf32 copy) from the
        gathered codes and per-group scale / zero point."""
        kernels.dequant_split(codes, qscale, qzp, group=self.group, symmetric=self.symmetric,
                              wq_hi=self.layer.wq_hi, wq_lo=self.layer.wq_lo,
                              wq_t32=self.layer.wq_t32)

    def gradients(self) -> dict[str, tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
        """K2 without the update: (gV, galpha, gbeta) per member, from ``layer.grad``."""
        out = {}
        for m in self.members:
            w, v, a, b = self._slices(m)
            r0, r1 = m.rows
            gv, ga, gb = torch.empty_like(v), torch.empty_like(a), torch.empty_like(b)
            kernels.ste_signsgd(self.layer.grad[r0:r1], w, v, a, b, bits=m.scheme.bits,
                                group=m.group, eps=self.eps, lr=0.0, lo=0.0, hi=1.0, update=False,
                                gv=gv, galpha=ga, gbeta=gb, **self._scheme_kw(m))
            out[m.path] = (gv, ga, gb)
        return out

    def load(self, path: str, v: torch.Tensor, alpha: torch.Tensor, beta: torch.Tensor,
             init_scale: torch.Tensor | None = None) -> None:
        """Set one member's parameters (used by the parity tests)."""
        for m in self.members:
            if m.path == path:
                r0, r1 = m.rows
                self.v[r0:r1].copy_(v)
                self.alpha[r0:r1].copy_(alpha)
                self.beta[r0:r1].copy_(beta)
                if init_scale is not None:
                    if self.init_scale is None:
                        raise ValueError(f"{path} does not use a searched scale")
                    self.init_scale[r0:r1].copy_(init_scale)
        self.requantize()

    def reset(self) -> None:
        self.layer.ready()
        self.v.zero_()
        self.alpha.fill_(1.0)
        self.beta.fill_(1.0)
        self.requantize()

    def commit(self, keep_codes: bool = False) -> dict[str, QuantizedLayer]:
        """K5 per member, then make the layer's weight bf16(reconstruction)
        (reference mround/pipeline/runner.py:775-787)."""
        out: dict[str, QuantizedLayer] = {}
        self.layer.ready()
        committed = self.layer.w.clone()
        for m in self.members:
            w, v, a, b = self._slices(m)
            r0, r1 = m.rows
            kw = self._scheme_kw(m)
            packed, scales, biases, codes = kernels.pack_mlx(
                w, v, a, b, bits=m.scheme.bits, group=m.group, eps=self.eps, want_codes=keep_codes,
                **kw)
            kernels.fq_forward(w, v, a, b, bits=m.scheme.bits, group=m.group, eps=self.eps,
                               wq_hi=committed[r0:r1], **kw)
            out[m.path] = QuantizedLayer(packed.cpu(), scales.cpu(), biases.cpu(), m.scheme,
                                         (r1 - r0, w.shape[1]),
                                         None if codes is None else codes.cpu())
        self.layer.wq_hi, self.layer.wq_lo, self.layer.grad = committed, None, None
        self.layer.wq_t32 = None
        return out


def auto_exchange(world: int) -> str:
    """The weight-gradient exchange measured fastest inside the 7B tuning step
    on one 8-GPU B200 box (tf32 backward): the fused GEMM -> NVLink peer-store
    form up to four ranks (2 ranks: 6.25 ms of exchange against 7.38 with
    NCCL for the block's four weight gradients; 4 ranks: 16.72 / 16.61 ms
    steps), the NCCL reduce-scatter at eight (10.30 ms steps against 11.10:
    the epilogue's stores to seven peers hold the dW GEMMs back while NCCL's
    transfer overlaps the rest of the backward)."""
    return "p2p" if world <= 4 else "nccl"


@dataclasses.dataclass
class _Shard:
    """This rank's rows [s0, s1) of a fused weight under the row-sharded update:
    the summed gradient and the next operands (the all-gather's send buffers)."""

    s0: int
    s1: int
    grad: torch.Tensor
    hi: torch.Tensor | None
    lo: torch.Tensor | None
    t32: torch.Tensor | None
    codes: _Codes | None = None  # the gather of codes instead of operands


@dataclasses.dataclass
class _Codes:
    """The codes gather of one fused weight: this rank's rows (send buffers)
    and every rank's (receive buffers), one byte per weight plus a float32
    scale (and zero point) per group, against eight bytes per weight for the
    operands (bf16 hi + lo, tf32)."""

    codes: torch.Tensor
    qscale: torch.Tensor
    qzp: torch.Tensor | None
    all_codes: torch.Tensor
    all_qscale: torch.Tensor
    all_qzp: torch.Tensor | None


class _Dequant:
    """A pending entry of a fused weight (``FusedLinear.pending``): waits for
    the codes gather, then rebuilds the operands on the waiting stream."""

    def __init__(self, tunable: TunableLayer, codes: _Codes, works: list) -> None:
        self.tunable, self.codes, self.works = tunable, codes, works

    def wait(self) -> None:
        for w in self.works:
            if w is not None:
                w.wait()
        c = self.codes
        self.tunable.dequant(c.all_codes, c.all_qscale, c.all_qzp)


class BlockTuner:
    """Runs the tuning of one block over this rank's shard of the batches."""

    def __init__(self, block: DeviceBlock, schemes: dict[str, QuantScheme], lrs: dict[str, float],
                 *, suppress: bool, eps: float, precision: Precision, dist: DistContext,
                 pieces: int = 1, exchange: str = "auto", gather: str = "codes") -> None:
        """``exchange``: how the row-sharded update gathers each rank's rows of
        the gradient -- "p2p" (the weight-gradient GEMM stores them into their
        owners' slots over NVLink), "copy" (the GEMM writes locally and the
        copy engines move the rows into the same slots), "nccl" (a
        reduce-scatter after the GEMM) or "auto" (``auto_exchange``).
        ``gather``: what the ranks all-gather after their rows' signed step --
        "codes" (codes and per-group scale / zero point, rebuilt into operands
        on every rank; used for fused weights whose every row is tuned and
        whose width is a multiple of 8) or "operands" (bf16 hi/lo and tf32)."""
        if gather not in ("codes", "operands"):
            raise ValueError(f"gather must be 'codes' or 'operands', got {gather!r}")
        if exchange == "auto":
            exchange = auto_exchange(dist.world)
        if exchange not in ("p2p", "copy", "nccl"):
            raise ValueError(f"exchange must be 'p2p', 'copy', 'nccl' or 'auto', got {exchange!r}")
        self.exchange = exchange
        self.block = block
        self.suppress = suppress
        self.precision = precision
        self.dist = dist
        self.pieces = pieces
        self.tunables: list[TunableLayer] = []
        self.skipped: list[tuple[str, str]] = []
        for layer in block.layers.values():
            members = []
            for path, r0, r1 in layer.members:
                if path not in schemes:
                    continue
                scheme = schemes[path]
                try:
                    group = require_device_scheme(scheme, layer.in_features)
                except Exception as exc:  # noqa: BLE001 - reported like the reference's skip
                    self.skipped.append((path, str(exc)))
                    continue
                members.append(Member(path, (r0, r1), scheme, group, lrs[path]))
            if members:
                self.tunables.append(TunableLayer(layer, members, eps,
                                                  tf32=precision.grad_input == TF32))
                if dist.world > 1:
                    layer.grad_ready.append(self._reduce_hook)
        self.ws = kernels.LossWorkspace(block.device)
        self.importance: dict[str, torch.Tensor] = {}  # per fused layer, after search()
        self._pending: dict[int, object] = {}
        self._last_piece = True
        # Row-sharded update: every fused weight's rows divide by the rank count,
        # so rank r reduce-scatters the gradient, steps rows [r*R/N, (r+1)*R/N)
        # and all-gathers the operands; otherwise all-reduce and step everywhere.
        self.sharded = dist.world > 1 and all(t.layer.out_features % dist.world == 0
                                              for t in self.tunables)
        self._sharded_step = False
        self._dirty = False  # V/alpha/beta rows of other ranks are stale
        self._shards: dict[int, _Shard] = {}
        if self.sharded:
            for t in self.tunables:
                out, inn = t.layer.w.shape
                per = out // dist.world
                s0, s1 = dist.rank * per, (dist.rank + 1) * per
                grad = torch.empty((per, inn), dtype=torch.float32, device=block.device)
                if gather == "codes" and t.whole and inn % 8 == 0:
                    self._shards[id(t.layer)] = _Shard(s0, s1, grad, None, None, None,
                                                       self._codes_buffers(t, per))
                    continue
                # untuned rows of a partly tuned fused weight keep their exact operand
                t32 = t.layer.wq_t32
                self._shards[id(t.layer)] = _Shard(
                    s0, s1, grad, t.layer.wq_hi[s0:s1].clone(), t.layer.wq_lo[s0:s1].clone(),
                    None if t32 is None else t32[s0:s1].clone())
        # Fused GEMM -> reduce-scatter over NVLink peer memory (one piece per
        # step; at most 8 ranks; every rank agrees before it is used).
        self.peer = None
        self._epoch = 0
        if (self.sharded and exchange in ("p2p", "copy") and pieces == 1 and dist.world <= 8
                and all(t.layer.in_features % 4 == 0 for t in self.tunables)):
            from mround_b200.pipeline.peer import PeerExchange

            self.peer = PeerExchange(dist, [tuple(t.layer.w.shape) for t in self.tunables],
                                     block.device, copy_engine=exchange == "copy")
            for t, ex in zip(self.tunables, self.peer.layers):
                t.layer.exchange = ex

    def _codes_buffers(self, t: TunableLayer, per: int) -> _Codes:
        out, inn = t.layer.w.shape
        dev = self.block.device
        gpr = inn // t.group
        asym = not t.symmetric

        def f32(rows):
            return torch.empty((rows, gpr), dtype=torch.float32, device=dev)

        return _Codes(torch.empty((per, inn), dtype=torch.uint8, device=dev), f32(per),
                      f32(per) if asym else None,
                      torch.empty((out, inn), dtype=torch.uint8, device=dev), f32(out),
                      f32(out) if asym else None)

    # ------------------------------------------------------------ search
    def search(self, inputs: list[torch.Tensor]) -> float:
        """The v2 scale search for every searched member (reference
        ``QuantizationRunner._search_scales``, mround/pipeline/runner.py:712-760).

        One forward per calibration batch through the ORIGINAL weights collects
        each fused weight's importance (summed squared input per channel,
        runner.py:346-363, summed over all ranks' shards), then K8 searches every
        searched member at its own width.  Returns the seconds spent (0.0 when
        nothing searches).
        """
        searching = [t for t in self.tunables if t.searched]
        if not searching:
            return 0.0
        torch.cuda.synchronize(self.block.device)
        started = time.perf_counter()
        stash = {}
        collect = {}
        for t in self.tunables:
            layer = t.layer
            stash[layer.name] = (layer.wq_hi, layer.wq_lo, layer.wq_t32)
            layer.use_dense()
        for t in searching:
            collect[t.layer.name] = torch.zeros(t.layer.in_features, dtype=torch.float32,
                                                device=self.block.device)
        try:
            with torch.no_grad():
                for x in inputs:
                    self.block.forward_fused(x, self.precision, False, collect)
        finally:
            for t in self.tunables:
                t.layer.wq_hi, t.layer.wq_lo, t.layer.wq_t32 = stash[t.layer.name]
        for name in sorted(collect):
            self.dist.all_reduce_(collect[name])
        self.importance = collect
        for t in searching:
            for m in t.members:
                r0, r1 = m.rows
                search_scales(t.layer.w[r0:r1], m.scheme, importance=collect[t.layer.name],
                              out=t.init_scale[r0:r1])
            t.requantize()
        torch.cuda.synchronize(self.block.device)
        return time.perf_counter() - started

    # ------------------------------------------------------------ pieces
    def _reduce_hook(self, layer: FusedLinear) -> None:
        if not self._last_piece:
            return
        if layer.exchange is not None and layer.exchange.active:
            return  # the GEMM has already stored the rows with their owners
        if self._sharded_step:
            grad = self._shards[id(layer)].grad
            self._pending[id(layer)] = self.dist.reduce_scatter_async(grad, layer.grad)
        else:
            self._pending[id(layer)] = self.dist.all_reduce_async(layer.grad)

    def _update(self, step: int, iters: int) -> None:
        """The signed step of every tunable after the backward."""
        if not self._sharded_step:
            # every fused weight's gradient is whole; tunables of one scheme and
            # group share a launch
            launches: dict[tuple, list[TunableLayer]] = {}
            for t in self.tunables:
                self._wait(t.layer)
                launches.setdefault(t.launch_key, []).append(t)
            for alike in launches.values():
                alike[0].run_segments([sg for t in alike for sg in t.segments(step, iters)])
            return
        # Copy-engine exchange: every copy and flag release of this rank ends
        # before the first owner-side sum spins on this GPU, so no flag kernel
        # of this rank ever waits for an SM behind a spinning sum.
        for t in self.tunables:
            ex = t.layer.exchange
            if ex is not None and ex.active and ex.copy_engine:
                ex.wait_copies()
        # rows of this rank, then the operands' all-gather; qkv first, so the
        # next forward's first GEMM waits on the smallest gather only
        for t in self.tunables:
            sh = self._shards[id(t.layer)]
            ex = t.layer.exchange
            if ex is not None and ex.active:
                # every source's rows are in this rank's slots once its flag
                # carries this step's epoch; sum them in rank order
                kernels.reduce_slots(ex.slots, ex.flags, ex.epoch, sh.grad)
                ex.active = False
            else:
                self._wait(t.layer)
            if sh.codes is not None:
                c = sh.codes
                t.update_rows_codes(step, iters, sh.s0, sh.s1, sh.grad, c.codes, c.qscale, c.qzp)
                works = [self.dist.all_gather_async(c.all_codes, c.codes),
                         self.dist.all_gather_async(c.all_qscale, c.qscale)]
                if c.qzp is not None:
                    works.append(self.dist.all_gather_async(c.all_qzp, c.qzp))
                t.layer.pending.append(_Dequant(t, c, works))
                continue
            t.update_rows(step, iters, sh.s0, sh.s1, sh.grad, sh.hi, sh.lo, sh.t32)
            t.layer.pending.append(self.dist.all_gather_async(t.layer.wq_hi, sh.hi))
            t.layer.pending.append(self.dist.all_gather_async(t.layer.wq_lo, sh.lo))
            if sh.t32 is not None:
                t.layer.pending.append(self.dist.all_gather_async(t.layer.wq_t32, sh.t32))
        self._dirty = True

    def sync_params(self) -> None:
        """Make V/alpha/beta whole on every rank after row-sharded steps."""
        if not self._dirty:
            return
        for t in self.tunables:
            t.layer.ready()
            s0, s1 = self._shards[id(t.layer)].s0, self._shards[id(t.layer)].s1
            works = [self.dist.all_gather_async(buf, buf[s0:s1].clone())
                     for buf in (t.v, t.alpha, t.beta)]
            for w in works:
                if w is not None:
                    w.wait()
        self._dirty = False

    def _wait(self, layer: FusedLinear) -> None:
        work = self._pending.pop(id(layer), None)
        if work is not None:
            work.wait()

    # ------------------------------------------------------------ loss
    def _threshold(self, pred: torch.Tensor, target: torch.Tensor, k: int) -> None:
        """Exact global k-th largest |r| into ``ws.thr`` (three radix passes)."""
        for p in range(3):
            kernels.loss_hist_pass(pred, target, self.ws, p)
            self.dist.all_reduce_(self.ws.hist)
            kernels.loss_select_digit(self.ws, k, p)

    def loss(self, pred: torch.Tensor, target: torch.Tensor, *, grad: torch.Tensor | None,
             threshold_ready: bool = False) -> torch.Tensor:
        """This rank's share of the batch loss (device float64 scalar)."""
        n_global = pred.numel() * self.dist.world if not threshold_ready else self._n_global
        k = max(1, int(n_global * OUTLIER_FRACTION))
        if self.dist.world == 1 and not threshold_ready:
            kernels.loss_outlier(pred, target, self.ws, suppress=self.suppress, denom=float(n_global),
                                 k=k, grad=grad)
        else:
            if self.suppress and not threshold_ready:
                self._threshold(pred, target, k)
            kernels.loss_apply(pred, target, self.ws, suppress=self.suppress,
                               denom=float(n_global), grad=grad)
        return self.ws.loss.clone()

    # ------------------------------------------------------------ passes
    def output(self, x: torch.Tensor) -> torch.Tensor:
        with torch.no_grad():
            if self.pieces == 1:
                return self.block.forward_fused(x, self.precision, False)[0]
            parts = [self.block.forward_fused(x[lo:hi], self.precision, False)[0]
                     for lo, hi in piece_bounds(x.shape[0], self.pieces)]
            return torch.cat(parts, 0)

    def batch_loss(self, x: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        return self.loss(self.output(x), target, grad=None)

    def mean_loss(self, inputs: list[torch.Tensor], targets: list[torch.Tensor],
                  batches: list[int]) -> float:
        """Mean over batches of the global batch loss; one host read."""
        vals = torch.stack([self.batch_loss(inputs[i], targets[i]) for i in batches])
        self.dist.all_reduce_(vals)
        return float(vals.mean().item())

    def step(self, x: torch.Tensor, target: torch.Tensor, step: int, iters: int) -> torch.Tensor:
        """One signed-gradient step on one batch; returns this rank's loss share."""
        self._sharded_step = self.sharded
        if self.peer is not None:
            self._epoch += 1
            for t in self.tunables:
                t.layer.exchange.epoch = self._epoch
                t.layer.exchange.active = True
        bounds = piece_bounds(x.shape[0], self.pieces)
        if len(bounds) == 1:
            self._last_piece = True
            for t in self.tunables:
                t.layer.accumulate_grad = False
            out, saved = self.block.forward_fused(x, self.precision, True)
            grad = torch.empty_like(out)
            loss = self.loss(out, target, grad=grad)
            del out
            self.block.backward_fused(saved, grad, self.precision)
            del saved
        else:
            # whole-batch threshold first, then each piece against it
            self._n_global = x.numel() * self.dist.world
            if self.suppress:
                k = max(1, int(self._n_global * OUTLIER_FRACTION))
                self._threshold(self.output(x), target, k)
            loss = torch.zeros((), dtype=torch.float64, device=x.device)
            for i, (lo, hi) in enumerate(bounds):
                self._last_piece = i == len(bounds) - 1
                for t in self.tunables:
                    t.layer.accumulate_grad = i > 0
                out, saved = self.block.forward_fused(x[lo:hi], self.precision, True)
                grad = torch.empty_like(out)
                loss += self.loss(out, target[lo:hi], grad=grad, threshold_ready=True)
                del out
                self.block.backward_fused(saved, grad, self.precision)
                del saved
        self._update(step, iters)
        self._sharded_step = False
        return loss

    def gradient_only(self, x: torch.Tensor, target: torch.Tensor):
        """Forward, loss and backward without a step; returns (loss, grads by path)."""
        self.sync_params()
        self._last_piece = True
        for t in self.tunables:
            t.layer.accumulate_grad = False
        out, saved = self.block.forward_fused(x, self.precision, True)
        grad = torch.empty_like(out)
        loss = self.loss(out, target, grad=grad)
        self.block.backward_fused(saved, grad, self.precision)
        grads = {}
        for t in self.tunables:
            self._wait(t.layer)
            grads.update(t.gradients())
        return loss, grads

    def reset(self) -> None:
        for t in self.tunables:
            t.reset()
        self._dirty = False

    def close(self) -> None:
        """Release the peer mappings of the fused exchange and report a bounded
        wait that gave up (``DeviceError``)."""
        if self.peer is None:
            return
        from mround_b200._native import lib
        from mround_b200.exceptions import DeviceError

        status = int(lib().mr_peer_status(1))
        for t in self.tunables:
            t.layer.exchange = None
        self.peer.close()
        self.peer = None
        if status:
            raise DeviceError(f"the peer gradient exchange gave up waiting (status {status})")

    def snapshot(self) -> list[tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
        self.sync_params()
        return [(t.v.clone(), t.alpha.clone(), t.beta.clone()) for t in self.tunables]

    def commit(self, keep_codes: bool = False) -> dict[str, QuantizedLayer]:
        self.sync_params()
        out: dict[str, QuantizedLayer] = {}
        for t in self.tunables:
            out.update(t.commit(keep_codes))
        return out
