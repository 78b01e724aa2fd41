"""One decoder block on the device: fused weights, forward, backward.

The block is the mlx-lm Llama/Qwen2 decoder layer the reference runs in
``block_output`` (mround/pipeline/blocks.py:578-606), in float32 semantics.
The tuning path (``forward_fused`` / ``backward_fused``) runs every op on this
library's kernels -- the linears and the attention products on the tcgen05
GEMM (K3), norms, RoPE, softmax and SwiGLU on K7 -- with an explicit
backward; ``DeviceBlock.forward`` is an autograd form (K3 linears, torch for
the rest) kept as a cross-check:

    h1  = rmsnorm(x) * w_in            q|k|v = h1 @ Wqkv^T (+ b)
    q,k = rope(q), rope(k)             a = causal_gqa_sdpa(q, k, v)
    h   = x + a @ Wo^T                 h2 = rmsnorm(h) * w_post
    g|u = h2 @ Wgu^T                   out = h + (silu(g) * u) @ Wdown^T

Linears that share an input are fused by concatenating their rows (q|k|v and
gate|up), which keeps every quantization group intact because groups run
along the input dimension.  The fused weight lives once in HBM as bf16, and
the tunable state beside it (V, alpha, beta as float32; the fake-quantized
operand as bf16 hi/lo; the weight gradient as float32).

Float32 activations enter the GEMM as two bf16 parts (hi = bf16(x),
lo = bf16(x - hi)).  ``Precision`` chooses how many products each GEMM role
issues; three products (hi*hi + hi*lo + lo*hi) reproduce a float32 GEMM to
about 2**-16 relative, which the block loss needs: it is a small difference
of two large outputs (the reference's own float32 requirement,
mround/pipeline/runner.py module docstring).
"""

from __future__ import annotations

import dataclasses
import math

import torch
import torch.nn.functional as F

from mround_b200 import kernels
from mround_b200.pipeline.arch import Arch
from mround_b200.pipeline.attention import attention
from mround_b200.pipeline.model import BlockParams

__all__ = ["FusedLinear", "DeviceBlock", "Precision", "FUSION", "TF32", "TUNING_PRECISION"]

# fused GEMM groups: name -> member linears (row order)
FUSION: dict[str, tuple[str, ...]] = {
    "qkv": ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"),
    "o": ("self_attn.o_proj",),
    "gate_up": ("mlp.gate_proj", "mlp.up_proj"),
    "down": ("mlp.down_proj",),
}


# Precision code of one tf32 product (float32 operands rounded to tf32).
TF32 = 4


@dataclasses.dataclass(frozen=True)
class Precision:
    """Tensor-core form per GEMM role: 1-3 bf16 products (3 = the
    float32-faithful hi/lo split, 1 = plain bf16), or ``TF32`` (one tf32
    product of tf32-rounded float32 operands, 11 significant bits each, at the
    tensor time of two bf16 products).  The forward stays at 3 in every
    configuration: the loss is a small difference of two large outputs."""

    forward: int = 3
    grad_input: int = 3
    grad_weight: int = 3

    def __post_init__(self) -> None:
        if self.forward not in (1, 2, 3):
            raise ValueError(f"forward precision must be 1, 2 or 3, got {self.forward}")
        for role in (self.grad_input, self.grad_weight):
            if role not in (1, 2, 3, TF32):
                raise ValueError(f"gradient precision must be 1, 2, 3 or TF32 ({TF32}), got {role}")


# The tuning step's default: the forward as the three-product split, both
# backward products as one tf32 product each.  Measured at the Qwen2.5-7B
# block shapes: weight gradients within 3.4e-4 (max-normalised) of float64,
# against 2.5e-5 with three bf16 products everywhere; the bar is 1e-3.
TUNING_PRECISION = Precision(3, TF32, TF32)


class FusedLinear:
    """A row-concatenation of block linears that share one input.

    Attributes:
        members: ``(path, row_start, row_stop)`` per linear.
        w: dense bf16 weight (out, in) -- the original, never modified.
        bias: float32 (out,) or None (Qwen2 q/k/v carry a bias).
        wq_hi / wq_lo: the operand the forward uses (bf16 hi/lo parts of the
            fake-quantized weight; ``wq_lo`` None means ``wq_hi`` is exact).
        wq_t32: the same weight rounded to tf32 (float32), the operand of a
            tf32 input-gradient GEMM, or None.
        grad: float32 (out, in) buffer the weight-gradient GEMM writes, or None.
    """

    def __init__(self, name: str, members: list[tuple[str, int, int]], w: torch.Tensor,
                 bias: torch.Tensor | None) -> None:
        self.name = name
        self.members = members
        self.w = w
        self.bias = bias
        self.wq_hi: torch.Tensor = w
        self.wq_lo: torch.Tensor | None = None
        self.wq_t32: torch.Tensor | None = None  # tf32 operand of the input-gradient GEMM
        self.grad: torch.Tensor | None = None
        self.accumulate_grad = False
        self.grad_ready: list = []  # callbacks run right after this layer's weight gradient
        self.pending: list = []  # collectives that must finish before wq_hi/wq_lo are read
        self.exchange = None  # peer slots of the fused GEMM -> reduce-scatter (LayerExchange)

    @property
    def out_features(self) -> int:
        return self.w.shape[0]

    @property
    def in_features(self) -> int:
        return self.w.shape[1]

    def use_dense(self) -> None:
        self.ready()
        self.wq_hi, self.wq_lo, self.wq_t32 = self.w, None, None

    def operand_t32(self) -> torch.Tensor:
        """The weight operand as tf32 values.  A bf16 weight (dense or
        committed) is exact in tf32 and is widened once; a tunable weight's
        copy is kept current by K1/K2."""
        if self.wq_t32 is None:
            if self.wq_lo is not None:
                raise RuntimeError(f"{self.name}: no tf32 operand of the fake-quantized weight")
            self.wq_t32 = self.wq_hi.float()
        return self.wq_t32

    def ready(self) -> None:
        """Order the current stream after the collectives still writing the operands."""
        for work in self.pending:
            work.wait()
        self.pending.clear()


def _split(x2: torch.Tensor, want_lo: bool):
    return kernels.split_bf16(x2, want_lo=want_lo)


class _LinearFn(torch.autograd.Function):
    """y = x @ W^T (+ b) on K3; backward writes dL/dW into ``layer.grad``."""

    @staticmethod
    def forward(ctx, x, anchor, layer: FusedLinear, prec: Precision):
        if TF32 in (prec.grad_input, prec.grad_weight):
            raise ValueError("the autograd form of the block runs bf16 products only")
        layer.ready()
        lead = x.shape[:-1]
        x2 = x.reshape(-1, layer.in_features)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        t = x2.shape[0]
        fwd = prec.forward if layer.wq_lo is not None else min(prec.forward, 2)
        need_lo = fwd >= 2 or (anchor.requires_grad and prec.grad_weight == 3)
        x_hi, x_lo = _split(x2, need_lo)
        y = torch.empty((t, layer.out_features), dtype=torch.float32, device=x.device)
        kernels.gemm(x_hi, x_lo, layer.wq_hi, layer.wq_lo, y, m=t, n=layer.out_features,
                     k=layer.in_features, a_kmajor=True, b_kmajor=True, lda=layer.in_features,
                     ldb=layer.in_features, ldc=layer.out_features, precision=fwd,
                     bias=layer.bias)
        ctx.layer = layer
        ctx.prec = prec
        ctx.lead = lead
        ctx.save_for_backward(x_hi, x_lo if x_lo is not None else x_hi)
        ctx.has_lo = x_lo is not None
        return y.view(*lead, layer.out_features)

    @staticmethod
    def backward(ctx, dy):
        layer: FusedLinear = ctx.layer
        prec: Precision = ctx.prec
        x_hi, x_lo = ctx.saved_tensors
        if not ctx.has_lo:
            x_lo = None
        n_out, n_in = layer.out_features, layer.in_features
        dy2 = dy.reshape(-1, n_out)
        if not dy2.is_contiguous() or dy2.dtype != torch.float32:
            dy2 = dy2.float().contiguous()
        t = dy2.shape[0]
        need_dy_lo = max(prec.grad_input, prec.grad_weight) >= 2
        dy_hi, dy_lo = _split(dy2, need_dy_lo)
        if layer.grad is not None:
            p = prec.grad_weight if x_lo is not None else min(prec.grad_weight, 2)
            # dW[o, i] = sum_t dy[t, o] x[t, i]: both operands M/N-major
            kernels.gemm(dy_hi, dy_lo, x_hi, x_lo, layer.grad, m=n_out, n=n_in, k=t,
                         a_kmajor=False, b_kmajor=False, lda=n_out, ldb=n_in, ldc=n_in,
                         precision=p, accumulate=layer.accumulate_grad)
            for hook in layer.grad_ready:
                hook(layer)
        dx = None
        if ctx.needs_input_grad[0]:
            p = prec.grad_input if layer.wq_lo is not None else min(prec.grad_input, 2)
            dx2 = torch.empty((t, n_in), dtype=torch.float32, device=dy.device)
            # dx[t, i] = sum_o dy[t, o] W[o, i]: B is N-major
            kernels.gemm(dy_hi, dy_lo, layer.wq_hi, layer.wq_lo, dx2, m=t, n=n_in, k=n_out,
                         a_kmajor=True, b_kmajor=False, lda=n_out, ldb=n_in, ldc=n_in,
                         precision=p)
            dx = dx2.view(*ctx.lead, n_in)
        return dx, None, None, None


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def rope_tables(seq_len: int, head_dim: int, theta: float, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin (seq_len, head_dim/2) of the non-interleaved rotary embedding."""
    half = head_dim // 2
    inv = theta ** (-torch.arange(0, half, dtype=torch.float64, device=device) * 2.0 / head_dim)
    ang = torch.arange(seq_len, dtype=torch.float64, device=device)[:, None] * inv[None, :]
    return torch.cos(ang).float(), torch.sin(ang).float()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x (B, H, S, D): rotate the two halves of each head vector."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat((x1 * cos - x2 * sin, x1 * sin + x2 * cos), dim=-1)


class DeviceBlock:
    """A decoder block resident on one GPU, ready to run forward and backward."""

    def __init__(self, arch: Arch, params: BlockParams, device: torch.device | str = "cuda") -> None:
        self.arch = arch
        self.index = params.index
        self.device = torch.device(device)
        self.input_norm = params.input_norm.to(self.device)
        self.post_norm = params.post_norm.to(self.device)
        self.layers: dict[str, FusedLinear] = {}
        for name, paths in FUSION.items():
            ws, bs, members, row = [], [], [], 0
            for path in paths:
                w = params.linears[path]
                members.append((path, row, row + w.shape[0]))
                row += w.shape[0]
                ws.append(w)
                if path in params.biases:
                    bs.append(params.biases[path].float())
            w = torch.cat(ws, 0).to(self.device).contiguous()
            bias = torch.cat(bs, 0).to(self.device).contiguous() if bs else None
            self.layers[name] = FusedLinear(name, members, w, bias)
        self._rope: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        self.anchor = torch.zeros((), device=self.device, requires_grad=True)

    def member_paths(self) -> list[str]:
        return [p for layer in self.layers.values() for p, _, _ in layer.members]

    def _tables(self, seq_len: int):
        if seq_len not in self._rope:
            self._rope[seq_len] = rope_tables(seq_len, self.arch.head_dim, self.arch.rope_theta,
                                              self.device)
        return self._rope[seq_len]

    def forward(self, x: torch.Tensor, prec: Precision, *, train: bool = False) -> torch.Tensor:
        """x (B, S, hidden) float32 -> block output, float32."""
        a = self.arch
        anchor = self.anchor if train else self.anchor.detach()
        lin = lambda name, inp: _LinearFn.apply(inp, anchor, self.layers[name], prec)  # noqa: E731
        b, s, _ = x.shape
        h1 = rms_norm(x, self.input_norm, a.rms_eps)
        qkv = lin("qkv", h1)
        q, k, v = qkv.split([a.q_dim, a.kv_dim, a.kv_dim], dim=-1)
        q = q.view(b, s, a.heads, a.head_dim).transpose(1, 2)
        k = k.view(b, s, a.kv_heads, a.head_dim).transpose(1, 2)
        v = v.view(b, s, a.kv_heads, a.head_dim).transpose(1, 2)
        cos, sin = self._tables(s)
        q = apply_rope(q, cos, sin)
        k = apply_rope(k, cos, sin)
        att = attention(q, k, v, 1.0 / math.sqrt(a.head_dim))
        att = att.transpose(1, 2).reshape(b, s, a.q_dim)
        h = x + lin("o", att)
        h2 = rms_norm(h, self.post_norm, a.rms_eps)
        gu = lin("gate_up", h2)
        g, u = gu.split([a.intermediate, a.intermediate], dim=-1)
        return h + lin("down", F.silu(g) * u)


# ---------------------------------------------------------------------------
# Explicit fused path: the same block, forward and backward written out.
#
# Every element-wise step is one kernel that writes the next GEMM operand as
# bf16 hi/lo (csrc/blockops.cu); the residual additions are folded into the
# GEMMs (C is preloaded with the residual and accumulated into); the backward
# never forms the block-input gradient, which the tuning step does not need.
# Saved for the backward: the operand splits, P (float32 and hi/lo), h, gu,
# and the second norm's rstd.

def _mm(a, b, c, *, m, n, k, a_kmajor, b_kmajor, lda, ldb, prec, bias=None, accumulate=False):
    kernels.gemm(a[0], a[1] if prec >= 2 else None, b[0], b[1] if prec == 3 else None, c, m=m, n=n,
                 k=k, a_kmajor=a_kmajor, b_kmajor=b_kmajor, lda=lda, ldb=ldb, ldc=n,
                 precision=prec, bias=bias, accumulate=accumulate)


def _bmm(a, b, c, *, m, n, k, batch, a_kmajor, b_kmajor, lda, ldb, sa, sb, sc, causal=0, seq=0):
    kernels.gemm_batched(a[0], a[1], b[0], b[1], c, m=m, n=n, k=k, batch=batch, a_kmajor=a_kmajor,
                         b_kmajor=b_kmajor, lda=lda, ldb=ldb, ldc=n, stride_a=sa, stride_b=sb,
                         stride_c=sc, precision=3, causal=causal, seq=seq)


def _wprec(layer: FusedLinear, want: int) -> int:
    if want == TF32:
        return TF32
    return want if layer.wq_lo is not None else min(want, 2)


def _fused_forward(self: DeviceBlock, x: torch.Tensor, prec: Precision, save: bool,
                   collect: dict[str, torch.Tensor] | None = None):
    """Block forward.  ``collect`` maps fused-layer names to float32 (in_features,)
    accumulators: each receives the summed squared input its GEMM sees (the
    importance statistics of the searched scale).  With ``save`` and a tf32
    weight-gradient precision, the linears' inputs are also kept as tf32
    copies (the weight-gradient GEMMs' B operands), written by the same
    element-wise kernels."""
    a = self.arch

    def stats(name, op):
        if collect is not None and name in collect:
            kernels.colsumsq_split(op[0], op[1], collect[name])

    b, s, h = x.shape
    t = b * s
    hq, hkv, d, inter = a.heads, a.kv_heads, a.head_dim, a.intermediate
    rep, nb = hq // hkv, b * hkv
    scale = 1.0 / math.sqrt(d)
    t32 = save and prec.grad_weight == TF32
    x2 = x.reshape(t, h)
    L = self.layers
    h1_hi, h1_lo, rstd1, h1_t = kernels.rmsnorm_split(x2, self.input_norm, a.rms_eps, t32=t32)
    h1 = (h1_hi, h1_lo, h1_t)
    qkv_l = L["qkv"]
    stats("qkv", h1)
    L["qkv"].ready()
    qkv = torch.empty((t, qkv_l.out_features), dtype=torch.float32, device=x.device)
    p = _wprec(qkv_l, prec.forward)
    _mm(h1, (qkv_l.wq_hi, qkv_l.wq_lo), qkv, m=t, n=qkv_l.out_features, k=h, a_kmajor=True,
        b_kmajor=True, lda=h, ldb=h, prec=p, bias=qkv_l.bias)
    cos, sin = self._tables(s)
    q, k, v = kernels.rope_split(qkv, cos, sin, b, s, hq, hkv, d)
    del qkv
    band = s % 128 == 0  # causal tile skipping needs 128-aligned heads
    c1, c2 = (1, 2) if band else (0, 0)
    scores = torch.empty((nb, rep * s, s), dtype=torch.float32, device=x.device)
    _bmm(q, k, scores, m=rep * s, n=s, k=d, batch=nb, a_kmajor=True, b_kmajor=True, lda=d, ldb=d,
         sa=rep * s * d, sb=s * d, sc=rep * s * s, causal=c1, seq=s)
    probs = kernels.softmax_causal_split(scores, nb * rep * s, s, scale, band)  # P as hi/lo
    del scores
    o = torch.empty((b, hq, s, d), dtype=torch.float32, device=x.device)
    _bmm(probs, v, o, m=rep * s, n=d, k=s, batch=nb, a_kmajor=True, b_kmajor=False, lda=s, ldb=d,
         sa=rep * s * s, sb=s * d, sc=rep * s * d, causal=c2, seq=s)
    att = kernels.heads_split(o, b, s, hq, d, merge=True, t32=t32)
    del o
    o_l = L["o"]
    stats("o", att)
    o_l.ready()
    hres = x2.clone()
    _mm(att, (o_l.wq_hi, o_l.wq_lo), hres, m=t, n=h, k=hq * d, a_kmajor=True, b_kmajor=True,
        lda=hq * d, ldb=hq * d, prec=_wprec(o_l, prec.forward), accumulate=True)
    h2_hi, h2_lo, rstd2, h2_t = kernels.rmsnorm_split(hres, self.post_norm, a.rms_eps, t32=t32)
    gu_l = L["gate_up"]
    stats("gate_up", (h2_hi, h2_lo))
    gu_l.ready()
    gu = torch.empty((t, 2 * inter), dtype=torch.float32, device=x.device)
    _mm((h2_hi, h2_lo), (gu_l.wq_hi, gu_l.wq_lo), gu, m=t, n=2 * inter, k=h, a_kmajor=True,
        b_kmajor=True, lda=h, ldb=h, prec=_wprec(gu_l, prec.forward))
    act = kernels.swiglu_split(gu, t, inter, t32=t32)
    dn_l = L["down"]
    stats("down", act)
    dn_l.ready()
    out = hres.clone()
    _mm(act, (dn_l.wq_hi, dn_l.wq_lo), out, m=t, n=h, k=inter, a_kmajor=True, b_kmajor=True,
        lda=inter, ldb=inter, prec=_wprec(dn_l, prec.forward), accumulate=True)
    saved = None
    if save:
        saved = dict(shape=(b, s, h), h1=h1, q=q, k=k, v=v, probs=probs, att=att, hres=hres,
                     rstd2=rstd2, h2=(h2_hi, h2_lo, h2_t), gu=gu, act=act, x=x2, rstd1=rstd1)
    return out.view(b, s, h), saved


def _fused_backward(self: DeviceBlock, saved: dict, dout: torch.Tensor, prec: Precision,
                    want_dx: bool = False) -> torch.Tensor | None:
    """Weight gradients of every fused linear that has a ``grad`` buffer, and,
    with ``want_dx``, the gradient of the block input (float32, the shape of
    ``dout``) -- the whole-model backward of the DeltaLoss scoring needs it;
    the tuning step does not.

    Every gradient operand of a linear's GEMMs is produced as an operand
    triple (hi, lo, t32): the bf16 split when a bf16 product reads it, the
    tf32-rounded copy when a tf32 product does."""
    a = self.arch
    b, s, h = saved["shape"]
    t = b * s
    hq, hkv, d, inter = a.heads, a.kv_heads, a.head_dim, a.intermediate
    rep, nb = hq // hkv, b * hkv
    scale = 1.0 / math.sqrt(d)
    L = self.layers
    tf_w, tf_x = prec.grad_weight == TF32, prec.grad_input == TF32
    need_t32 = tf_w or tf_x
    need_split = not (tf_w and tf_x)
    dout2 = dout.reshape(t, h)
    g_out = (*(kernels.split_bf16(dout2) if need_split else (None, None)),
             kernels.round_tf32(dout2) if need_t32 else None)

    def weight_grad(layer, dy, x_in, n_out, n_in):
        if layer.grad is None:
            return
        ex = layer.exchange
        # dW[o, i] = sum_t dy[t, o] x[t, i]: both operands M/N-major
        kw = dict(m=n_out, n=n_in, k=t, a_kmajor=False, b_kmajor=False, lda=n_out, ldb=n_in)
        if ex is not None and ex.active and not layer.accumulate_grad and ex.copy_engine:
            # the whole gradient locally, then the copy engines move each
            # owner's rows over NVLink while the backward goes on
            if tf_w:
                kernels.gemm_tf32(dy[2], x_in[2], layer.grad, ldc=n_in, **kw)
            else:
                kernels.gemm(dy[0], dy[1], x_in[0], x_in[1], layer.grad, ldc=n_in,
                             precision=prec.grad_weight, **kw)
            ex.send(layer.grad)
        elif ex is not None and ex.active and not layer.accumulate_grad:
            # rows go straight to their owner ranks over NVLink
            rs = dict(dst_ptrs=ex.dst_ptrs, ldd=n_in, rows_per_rank=ex.rows_per_rank,
                      flag_ptrs=ex.flag_ptrs, done=ex.done, epoch=ex.epoch)
            if tf_w:
                kernels.gemm_rs_tf32(dy[2], x_in[2], **kw, **rs)
            else:
                kernels.gemm_rs(dy[0], dy[1], x_in[0], x_in[1], precision=prec.grad_weight,
                                **kw, **rs)
        elif tf_w:
            kernels.gemm_tf32(dy[2], x_in[2], layer.grad, ldc=n_in,
                              accumulate=layer.accumulate_grad, **kw)
        else:
            kernels.gemm(dy[0], dy[1], x_in[0], x_in[1], layer.grad, ldc=n_in,
                         precision=prec.grad_weight, accumulate=layer.accumulate_grad, **kw)
        for hook in layer.grad_ready:
            hook(layer)

    def input_grad(layer, dy, n_out, n_in):
        # dx[t, i] = sum_o dy[t, o] W[o, i]: B is N-major
        out = torch.empty((t, n_in), dtype=torch.float32, device=dout.device)
        if tf_x:
            kernels.gemm_tf32(dy[2], layer.operand_t32(), out, m=t, n=n_in, k=n_out, a_kmajor=True,
                              b_kmajor=False, lda=n_out, ldb=n_in, ldc=n_in)
        else:
            _mm(dy, (layer.wq_hi, layer.wq_lo), out, m=t, n=n_in, k=n_out, a_kmajor=True,
                b_kmajor=False, lda=n_out, ldb=n_in, prec=_wprec(layer, prec.grad_input))
        return out

    dn_l, gu_l, o_l, qkv_l = L["down"], L["gate_up"], L["o"], L["qkv"]
    weight_grad(dn_l, g_out, saved["act"], h, inter)
    dact = input_grad(dn_l, g_out, h, inter)
    del g_out
    g_gu = kernels.swiglu_bwd_split(dact, saved["gu"], t, inter, split=need_split, t32=need_t32)
    del dact
    weight_grad(gu_l, g_gu, saved["h2"], 2 * inter, h)
    dh2 = input_grad(gu_l, g_gu, 2 * inter, h)
    del g_gu
    g_h_f32 = torch.empty_like(dout2) if want_dx else None
    g_h = kernels.rmsnorm_bwd_split(dh2, saved["hres"], self.post_norm, saved["rstd2"], dout2,
                                    split=need_split, t32=need_t32, out=g_h_f32)
    del dh2
    weight_grad(o_l, g_h, saved["att"], h, hq * d)
    datt = input_grad(o_l, g_h, h, hq * d)
    g_o = kernels.heads_split(datt, b, s, hq, d, merge=False)
    del datt
    q, k, v, probs = saved["q"], saved["k"], saved["v"], saved["probs"]
    band = s % 128 == 0
    c1, c2, c3 = (1, 2, 3) if band else (0, 0, 0)
    dp = torch.empty((nb, rep * s, s), dtype=torch.float32, device=dout.device)
    _bmm(g_o, v, dp, m=rep * s, n=s, k=d, batch=nb, a_kmajor=True, b_kmajor=True, lda=d, ldb=d,
         sa=rep * s * d, sb=s * d, sc=rep * s * s, causal=c1, seq=s)
    g_s = kernels.softmax_bwd_split(dp, probs, nb * rep * s, s, scale, band)
    del dp
    dq = torch.empty((b, hq, s, d), dtype=torch.float32, device=dout.device)
    _bmm(g_s, k, dq, m=rep * s, n=d, k=s, batch=nb, a_kmajor=True, b_kmajor=False, lda=s, ldb=d,
         sa=rep * s * s, sb=s * d, sc=rep * s * d, causal=c2, seq=s)
    dk = torch.empty((b, hkv, s, d), dtype=torch.float32, device=dout.device)
    _bmm(g_s, q, dk, m=s, n=d, k=rep * s, batch=nb, a_kmajor=False, b_kmajor=False, lda=s, ldb=d,
         sa=rep * s * s, sb=rep * s * d, sc=s * d, causal=c3, seq=s)
    dv = torch.empty((b, hkv, s, d), dtype=torch.float32, device=dout.device)
    _bmm(probs, g_o, dv, m=s, n=d, k=rep * s, batch=nb, a_kmajor=False, b_kmajor=False, lda=s,
         ldb=d, sa=rep * s * s, sb=rep * s * d, sc=s * d, causal=c3, seq=s)
    del g_s
    cos, sin = self._tables(s)
    g_qkv = kernels.rope_bwd_split(dq, dk, dv, cos, sin, b, s, hq, hkv, d, split=need_split,
                                   t32=need_t32)
    del dq, dk, dv
    weight_grad(qkv_l, g_qkv, saved["h1"], qkv_l.out_features, h)
    if not want_dx:
        return None
    dh1 = input_grad(qkv_l, g_qkv, qkv_l.out_features, h)
    del g_qkv
    dx = torch.empty_like(dout2)
    # h = x + attention: the input gradient is the first norm's backward plus dL/dh
    kernels.rmsnorm_bwd_split(dh1, saved["x"], self.input_norm, saved["rstd1"], g_h_f32,
                              split=False, out=dx)
    return dx.view(b, s, h)


DeviceBlock.forward_fused = _fused_forward
DeviceBlock.backward_fused = _fused_backward
