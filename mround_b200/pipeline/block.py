"""One decoder block on the device: fused weights, forward, backward.

The block is the mlx-lm Llama/Qwen2 decoder layer the reference runs in
``block_output`` (mround/pipeline/blocks.py:578-606), restated in torch
float32 with its linears on the tcgen05 GEMM (K3):

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

__all__ = ["FusedLinear", "DeviceBlock", "Precision", "FUSION"]

# fused GEMM groups: name -> member linears (row order)
FUSION: dict[str, tuple[str, ...]] = {
    "qkv": ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"),
    "o": ("self_attn.o_proj",),
    "gate_up": ("mlp.gate_proj", "mlp.up_proj"),
    "down": ("mlp.down_proj",),
}


@dataclasses.dataclass(frozen=True)
class Precision:
    """Products per GEMM role: 3 = float32-faithful split, 1 = plain bf16."""

    forward: int = 3
    grad_input: int = 3
    grad_weight: int = 3


class FusedLinear:
    """A row-concatenation of block linears that share one input.

    Attributes:
        members: ``(path, row_start, row_stop)`` per linear.
        w: dense bf16 weight (out, in) -- the original, never modified.
        bias: float32 (out,) or None (Qwen2 q/k/v carry a bias).
        wq_hi / wq_lo: the operand the forward uses (bf16 hi/lo parts of the
            fake-quantized weight; ``wq_lo`` None means ``wq_hi`` is exact).
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
        self.grad: torch.Tensor | None = None
        self.accumulate_grad = False
        self.grad_ready: list = []  # callbacks run right after this layer's weight gradient

    @property
    def out_features(self) -> int:
        return self.w.shape[0]

    @property
    def in_features(self) -> int:
        return self.w.shape[1]

    def use_dense(self) -> None:
        self.wq_hi, self.wq_lo = self.w, None


def _split(x2: torch.Tensor, want_lo: bool):
    return kernels.split_bf16(x2, want_lo=want_lo)


class _LinearFn(torch.autograd.Function):
    """y = x @ W^T (+ b) on K3; backward writes dL/dW into ``layer.grad``."""

    @staticmethod
    def forward(ctx, x, anchor, layer: FusedLinear, prec: Precision):
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
