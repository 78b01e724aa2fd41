"""DeltaLoss sensitivity scoring of every block layer at every candidate width.

Restates ``score_widths`` (reference mround/pipeline/scoring.py:425-583) on the
device: a whole-model causal-LM backward (mean shifted cross-entropy,
``_causal_loss`` 183-192) through block linears whose weights are replaced by
their round-to-nearest quantize-dequantize (``_anchor`` 224-235), then for every
layer and width ``sum |g * (Q_b(W) - W)|`` accumulated over batches
(``_accumulate`` 238-266, the term of line 262).  The term is K6
(``mr_deltaloss``): it runs the moment a layer's weight-gradient GEMM finishes,
reading the gradient once for all widths it scores, so no gradient or
perturbation is ever held beyond its layer.

The backward is the blocks' explicit fused forward/backward (the same K3 GEMMs
and K7 element-wise kernels as the tuning step, plus the block-input gradient)
and the LM head on K3; the cross-entropy gradient is formed in place on the
logits.

``own_width`` takes one backward per width at that width's anchors (the
reference's procedure); ``widest`` one backward at the widest width, scoring
every width's perturbation against it.  Sequences are padded to a multiple of
8 tokens at the end; causal attention keeps real positions unaffected and the
loss averages the real positions only.
"""

from __future__ import annotations

import dataclasses
import time
from collections.abc import Callable, Sequence

import numpy as np
import torch

from mround_b200 import kernels
from mround_b200.exceptions import SchemeError
from mround_b200.pipeline.block import DeviceBlock, FusedLinear, Precision
from mround_b200.pipeline.dist import DistContext
from mround_b200.pipeline.model import SyntheticModel
from mround_b200.core.scale_search import search_scales
from mround_b200.schemes import DEFAULT_EPS_FP32, QuantScheme, ScaleInit, Symmetry

__all__ = ["SensitivityScores", "score_widths"]


@dataclasses.dataclass(frozen=True)
class SensitivityScores:
    scores: dict[str, dict[int, float]]
    shapes: dict[str, tuple[int, int]]
    skipped: tuple[tuple[str, str], ...]
    seconds: float


def score_widths(model: SyntheticModel, batches: Sequence[np.ndarray], widths: Sequence[int],
                 base_scheme: QuantScheme, *, expected_blocks: int | None = None,
                 eps: float = DEFAULT_EPS_FP32, gradient_source: str = "own_width",
                 progress: Callable[[str], None] | None = None,
                 device: torch.device | str = "cuda",
                 dist: DistContext | None = None) -> SensitivityScores:
    """Score every block linear at every width (float64 sums on the device).

    Under data parallelism (``dist`` with several ranks) rank r takes batches
    r, r + N, ...; the per-layer float64 sums are all-reduced, so every rank
    ends with the scores of all batches and plans identically.
    """
    if not widths:
        raise ValueError("no candidate widths to score")
    if gradient_source not in ("own_width", "widest"):
        raise ValueError(f"gradient_source must be 'own_width' or 'widest', got {gradient_source!r}")
    started = time.perf_counter()
    dev = torch.device(device)
    arch = model.arch
    if expected_blocks is not None and expected_blocks != arch.layers:
        from mround_b200.exceptions import ArchitectureError

        raise ArchitectureError(f"found {arch.layers} blocks but the configuration says {expected_blocks}")
    group = base_scheme.group_size
    widths = sorted(int(w) for w in widths)
    prec = Precision()
    blocks = [DeviceBlock(arch, model.block(i), dev) for i in range(arch.layers)]
    shapes, skipped, paths_by_layer = {}, [], {}
    for blk in blocks:
        name = model.block_name(blk.index)
        for layer in blk.layers.values():
            members = []
            for path, r0, r1 in layer.members:
                full = f"{name}.{path}"
                if layer.in_features % group:
                    skipped.append((full, f"last dimension {layer.in_features} is not a multiple of {group}"))
                    continue
                if group not in kernels.DEVICE_GROUPS:
                    raise SchemeError(f"group size {group} is not a device group size")
                shapes[full] = (r1 - r0, layer.in_features)
                members.append((full, r0, r1))
            paths_by_layer[id(layer)] = members
    if not shapes:
        raise ValueError("no layer in any block can be quantized at this group size")
    # one float32 gradient buffer per fused shape, shared by all blocks
    grad_pool: dict[tuple[int, int], torch.Tensor] = {}
    for blk in blocks:
        for layer in blk.layers.values():
            key = tuple(layer.w.shape)
            if key not in grad_pool:
                grad_pool[key] = torch.empty(key, dtype=torch.float32, device=dev)
            layer.grad = grad_pool[key]
    acc = {p: torch.zeros(len(widths), dtype=torch.float64, device=dev) for p in shapes}
    active: dict[str, list[int]] = {}
    symmetric = base_scheme.symmetry is Symmetry.SYMMETRIC
    searched = base_scheme.scale_init is ScaleInit.SEARCHED
    # searched schemes: each layer's unweighted searched scale at every width,
    # kept (a few numbers per group) to rebuild that width's quantize-dequantize
    # (reference _grids, mround/pipeline/scoring.py:195-210)
    grids: dict[tuple[int, int], torch.Tensor] = {}
    if searched:
        for blk in blocks:
            for layer in blk.layers.values():
                if layer.in_features % group:
                    continue
                for bits in widths:
                    scheme = dataclasses.replace(base_scheme, bits=bits)
                    out = torch.empty((layer.out_features, layer.in_features // group),
                                      dtype=torch.float32, device=dev)
                    search_scales(layer.w, scheme, out=out)
                    grids[(id(layer), bits)] = out

    def on_grad(layer: FusedLinear) -> None:
        for full, r0, r1 in paths_by_layer[id(layer)]:
            bits = active["bits"]
            out = torch.zeros(len(bits), dtype=torch.float64, device=dev)
            g = [grids[(id(layer), b)][r0:r1] for b in bits] if searched else None
            kernels.deltaloss(layer.grad[r0:r1], layer.w[r0:r1], bits=bits, group=group, eps=eps,
                              out=out, symmetric=symmetric, grids=g)
            idx = [widths.index(b) for b in bits]
            acc[full][idx] += out

    for blk in blocks:
        for layer in blk.layers.values():
            layer.grad_ready.append(on_grad)

    def set_anchors(bits: int) -> None:
        ones = {}
        for blk in blocks:
            for layer in blk.layers.values():
                o, i = layer.w.shape
                if layer.in_features % group:
                    layer.use_dense()
                    continue
                key = (o, i // group)
                if key not in ones:
                    ones[key] = torch.ones(key, dtype=torch.float32, device=dev)
                zeros = torch.zeros((o, i), dtype=torch.float32, device=dev)
                hi, lo = torch.empty_like(layer.w), torch.empty_like(layer.w)
                kernels.fq_forward(layer.w, zeros, ones[key], ones[key], bits=bits, group=group,
                                   eps=eps, wq_hi=hi, wq_lo=lo, symmetric=symmetric,
                                   init_scale=grids.get((id(layer), bits)))
                layer.wq_hi, layer.wq_lo = hi, lo

    embed = model.embed_tokens().to(dev)
    head = model.lm_head().to(dev).contiguous()
    final_norm = model.final_norm().to(dev)

    hidden = arch.hidden

    def backward_pass(batch: np.ndarray) -> None:
        """Mean shifted cross-entropy of one batch, backward through every block
        (explicit fused forward/backward; each block's weight-gradient GEMMs run
        the K6 hooks)."""
        tokens = torch.as_tensor(batch, dtype=torch.long, device=dev)
        inp, labels = tokens[:, :-1], tokens[:, 1:]
        b, s = inp.shape
        pad = (-s) % 8
        if pad:
            inp = torch.cat([inp, inp[:, -1:].expand(b, pad)], dim=1)
        sp = s + pad
        x = embed[inp].float().contiguous()
        saved_all = []
        for blk in blocks:
            x, saved = blk.forward_fused(x, prec, True)
            saved_all.append(saved)
        x2 = x.reshape(b * sp, hidden)
        n_hi, n_lo, rstd_f, _ = kernels.rmsnorm_split(x2, final_norm, arch.rms_eps)
        t = b * s
        real = n_hi.view(b, sp, hidden)[:, :s].reshape(t, hidden), \
            n_lo.view(b, sp, hidden)[:, :s].reshape(t, hidden)
        vocab = head.shape[0]
        logits = torch.empty((t, vocab), dtype=torch.float32, device=dev)
        kernels.gemm(real[0], real[1], head, None, logits, m=t, n=vocab, k=hidden, a_kmajor=True,
                     b_kmajor=True, lda=hidden, ldb=hidden, ldc=vocab, precision=2)
        # d(mean CE)/dlogits = (softmax - onehot) / t, one row-wise kernel
        g_hi, g_lo = kernels.ce_grad_split(logits, labels.reshape(-1).contiguous(), 1.0 / t)
        del logits
        dh = torch.empty((t, hidden), dtype=torch.float32, device=dev)
        kernels.gemm(g_hi, g_lo, head, None, dh, m=t, n=hidden, k=vocab, a_kmajor=True,
                     b_kmajor=False, lda=vocab, ldb=hidden, ldc=hidden, precision=2)
        del g_hi, g_lo
        dn = torch.zeros((b, sp, hidden), dtype=torch.float32, device=dev)
        dn[:, :s] = dh.view(b, s, hidden)
        del dh
        dx = torch.empty((b * sp, hidden), dtype=torch.float32, device=dev)
        kernels.rmsnorm_bwd_split(dn.view(b * sp, hidden), x2, final_norm, rstd_f, None,
                                  split=False, out=dx)
        del dn, x, x2
        dx = dx.view(b, sp, hidden)
        for i in range(len(blocks) - 1, -1, -1):
            dx = blocks[i].backward_fused(saved_all[i], dx, prec, want_dx=i > 0)
            saved_all[i] = None

    schedule = [(w, [w]) for w in widths] if gradient_source == "own_width" else [(widths[-1], widths)]
    done = 0
    dist = dist or DistContext()
    mine = list(batches)[dist.rank::dist.world]
    for anchor_bits, scored in schedule:
        set_anchors(anchor_bits)
        active["bits"] = scored
        for batch in mine:
            backward_pass(batch)
            done += 1
            if progress is not None:
                progress(f"  scoring: backward {done}/{len(mine) * len(schedule)} "
                         f"at {time.perf_counter() - started:.0f}s")
    if dist.world > 1:
        names = sorted(acc)
        stacked = torch.stack([acc[p] for p in names])
        dist.all_reduce_(stacked)
        acc = {p: stacked[i] for i, p in enumerate(names)}
    torch.cuda.synchronize(dev)
    for blk in blocks:
        for layer in blk.layers.values():
            layer.grad_ready.clear()
            layer.grad = None
    scores = {p: {w: float(acc[p][j].item()) for j, w in enumerate(widths)} for p in shapes}
    return SensitivityScores(scores, shapes, tuple(skipped), time.perf_counter() - started)
