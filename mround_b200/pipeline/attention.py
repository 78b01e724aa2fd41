"""Causal grouped-query attention with its products on the tcgen05 GEMM (K3).

The decoder layer's attention (mlx-lm's ``scaled_dot_product_attention`` with
the "causal" mask, inside the reference's ``block_output``,
mround/pipeline/blocks.py:578-606) in float32 semantics: every product runs
as a batched three-product bf16 split GEMM, one launch per product over all
(batch, kv-head) pairs; the softmax and its backward run in float32.

Layout: q is (B, Hq, S, D) contiguous, so the ``rep = Hq / Hkv`` query heads
that share kv-head g are ``rep * S`` consecutive rows -- one GEMM problem per
(b, g) with M = rep*S.  k, v are (B, Hkv, S, D).

    scores = q k^T        A = q (K-major, k = D), B = k (K-major)
    o      = p v          A = p (K-major, k = S), B = v (N-major: n = D)
    dp     = do v^T       A = do (K-major), B = v (K-major)
    dq     = ds k         A = ds (K-major), B = k (N-major)
    dk     = ds^T q       A = ds (M-major, m = S, k = rep*S), B = q (N-major)
    dv     = p^T do       A = p (M-major), B = do (N-major)
"""

from __future__ import annotations

import torch

from mround_b200 import kernels

__all__ = ["attention"]

_MASKS: dict[tuple[int, str], torch.Tensor] = {}


def _mask(s: int, device) -> torch.Tensor:
    key = (s, str(device))
    if key not in _MASKS:
        _MASKS[key] = torch.ones(s, s, dtype=torch.bool, device=device).triu(1)
    return _MASKS[key]


def _split(x):
    return kernels.split_bf16(x)


def _bmm(a, b, c, *, m, n, k, batch, a_kmajor, b_kmajor, lda, ldb, ldc, sa, sb, sc):
    kernels.gemm_batched(a[0], a[1], b[0], b[1], c, m=m, n=n, k=k, batch=batch,
                         a_kmajor=a_kmajor, b_kmajor=b_kmajor, lda=lda, ldb=ldb, ldc=ldc,
                         stride_a=sa, stride_b=sb, stride_c=sc, precision=3)


class _Attention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, scale: float):
        bsz, hq, s, d = q.shape
        hkv = k.shape[1]
        rep = hq // hkv
        nb = bsz * hkv
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        qs, ks, vs = _split(q), _split(k), _split(v)
        scores = torch.empty((nb, rep * s, s), dtype=torch.float32, device=q.device)
        _bmm(qs, ks, scores, m=rep * s, n=s, k=d, batch=nb, a_kmajor=True, b_kmajor=True,
             lda=d, ldb=d, ldc=s, sa=rep * s * d, sb=s * d, sc=rep * s * s)
        view = scores.view(nb * rep, s, s)
        view.mul_(scale).masked_fill_(_mask(s, q.device), float("-inf"))
        p = torch.softmax(view, dim=-1)
        del scores, view
        ps = _split(p)
        out = torch.empty((bsz, hq, s, d), dtype=torch.float32, device=q.device)
        _bmm(ps, vs, out, m=rep * s, n=d, k=s, batch=nb, a_kmajor=True, b_kmajor=False,
             lda=s, ldb=d, ldc=d, sa=rep * s * s, sb=s * d, sc=rep * s * d)
        ctx.save_for_backward(qs[0], qs[1], ks[0], ks[1], vs[0], vs[1], p, ps[0], ps[1])
        ctx.dims = (bsz, hq, hkv, s, d, scale)
        return out

    @staticmethod
    def backward(ctx, dout):
        q_hi, q_lo, k_hi, k_lo, v_hi, v_lo, p, p_hi, p_lo = ctx.saved_tensors
        bsz, hq, hkv, s, d, scale = ctx.dims
        rep, nb = hq // hkv, bsz * hkv
        dos = _split(dout.contiguous().float())
        dp = torch.empty((nb * rep, s, s), dtype=torch.float32, device=dout.device)
        _bmm(dos, (v_hi, v_lo), dp, m=rep * s, n=s, k=d, batch=nb, a_kmajor=True, b_kmajor=True,
             lda=d, ldb=d, ldc=s, sa=rep * s * d, sb=s * d, sc=rep * s * s)
        # softmax backward, scaled: ds = scale * p * (dp - sum(dp * p))
        row = (dp * p).sum(-1, keepdim=True)
        dp.sub_(row).mul_(p).mul_(scale)
        dss = _split(dp)
        del dp, row
        dq = torch.empty((bsz, hq, s, d), dtype=torch.float32, device=dout.device)
        _bmm(dss, (k_hi, k_lo), dq, m=rep * s, n=d, k=s, batch=nb, a_kmajor=True, b_kmajor=False,
             lda=s, ldb=d, ldc=d, sa=rep * s * s, sb=s * d, sc=rep * s * d)
        dk = torch.empty((bsz, hkv, s, d), dtype=torch.float32, device=dout.device)
        _bmm(dss, (q_hi, q_lo), dk, m=s, n=d, k=rep * s, batch=nb, a_kmajor=False, b_kmajor=False,
             lda=s, ldb=d, ldc=d, sa=rep * s * s, sb=rep * s * d, sc=s * d)
        dv = torch.empty((bsz, hkv, s, d), dtype=torch.float32, device=dout.device)
        _bmm((p_hi, p_lo), dos, dv, m=s, n=d, k=rep * s, batch=nb, a_kmajor=False, b_kmajor=False,
             lda=s, ldb=d, ldc=d, sa=rep * s * s, sb=rep * s * d, sc=s * d)
        return dq, dk, dv, None


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """q (B, Hq, S, D), k/v (B, Hkv, S, D) float32 -> (B, Hq, S, D) float32."""
    return _Attention.apply(q, k, v, scale)
