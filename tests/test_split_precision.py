"""Why every weight GEMM of the tuning step uses the three-product bf16 split.

CPU emulation of K3's product sets (3: hi*hi + hi*lo + lo*hi, 2: the second
operand's lo part dropped, 1: hi*hi; float32 accumulation) on a scaled-down
Qwen2 block under 2-bit fake quantization, against a float64 reference of the
same block.  The bar is the one the GPU parity tests apply: loss within 1e-3
relative and every weight gradient within 1e-3 of the reference after
normalising by its largest magnitude.

The three-product split passes with a wide margin.  Dropping the weight's lo
part in the forward fails by an order of magnitude: the loss gradient is the
output residual of the quantized block, which is small next to the output, so
a 2^-9 relative perturbation of the forward moves it by ~1 %.
"""

from __future__ import annotations

import math

import pytest
import torch

H, NH, KV, D, INTER, T, GROUP, BITS = 512, 8, 2, 64, 1536, 128, 64, 2


def _split(a):
    hi = a.to(torch.bfloat16).float()
    return hi, (a - hi).to(torch.bfloat16).float()


def _mm(a, b, products):
    ah, al = _split(a)
    bh, bl = _split(b)
    out = ah @ bh
    if products == 3:
        out = out + ah @ bl
    if products >= 2:
        out = out + al @ bh
    return out


class _Linear(torch.autograd.Function):
    """y = x W^T with K3's operand roles: forward A = x, B = W; input gradient
    A = dY, B = W; weight gradient A = dY^T, B = X."""

    @staticmethod
    def forward(ctx, x, w, fwd, grad_in, grad_w):
        ctx.save_for_backward(x, w)
        ctx.roles = (grad_in, grad_w)
        return _mm(x, w.t(), fwd)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        grad_in, grad_w = ctx.roles
        return _mm(dy, w, grad_in), _mm(dy.t(), x, grad_w), None, None, None


def _fake_quant(w, gen):
    rows, cols = w.shape
    g = w.reshape(rows, cols // GROUP, GROUP)
    v = (torch.rand(g.shape, generator=gen, dtype=torch.float64) - 0.5) * 0.6
    lo_c = 0.7 + 0.3 * torch.rand(rows, cols // GROUP, 1, generator=gen, dtype=torch.float64)
    hi_c = 0.7 + 0.3 * torch.rand(rows, cols // GROUP, 1, generator=gen, dtype=torch.float64)
    top = g.amax(-1, keepdim=True).clamp(min=0) * hi_c
    bot = g.amin(-1, keepdim=True).clamp(max=0) * lo_c
    maxq = 2 ** BITS - 1
    s = ((top - bot) / maxq).clamp(min=1e-8)
    zp = torch.round(-bot / s)
    q = torch.clamp(torch.round(g / s + v) + zp, 0, maxq)
    return (s * (q - zp)).reshape(rows, cols).float().double()


def _rope(x):
    t, d = x.shape[1], x.shape[-1]
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    ang = torch.arange(t, dtype=torch.float64)[:, None] * inv[None]
    cos = torch.cat([ang.cos(), ang.cos()], -1).to(x.dtype)
    sin = torch.cat([ang.sin(), ang.sin()], -1).to(x.dtype)
    return x * cos + torch.cat([-x[..., d // 2:], x[..., : d // 2]], -1) * sin


def _block(x, w, bias, lin):
    t = x.shape[0]

    def rms(z):
        return z * torch.rsqrt(z.pow(2).mean(-1, keepdim=True) + 1e-6)

    h = rms(x)
    q = _rope((lin(h, w["q"]) + bias["q"]).view(t, NH, D).transpose(0, 1))
    k = _rope((lin(h, w["k"]) + bias["k"]).view(t, KV, D).transpose(0, 1))
    v = (lin(h, w["v"]) + bias["v"]).view(t, KV, D).transpose(0, 1)
    k, v = k.repeat_interleave(NH // KV, 0), v.repeat_interleave(NH // KV, 0)
    s = (q @ k.transpose(1, 2) / math.sqrt(D)).masked_fill(
        torch.ones(t, t, dtype=torch.bool).triu(1), float("-inf"))
    o = (torch.softmax(s, -1) @ v).transpose(0, 1).reshape(t, NH * D)
    h1 = x + lin(o, w["o"])
    h2 = rms(h1)
    return h1 + lin(torch.nn.functional.silu(lin(h2, w["gate"])) * lin(h2, w["up"]), w["down"])


@pytest.fixture(scope="module")
def problem():
    gen = torch.Generator().manual_seed(0)
    shapes = {"q": (NH * D, H), "k": (KV * D, H), "v": (KV * D, H), "o": (H, NH * D),
              "gate": (INTER, H), "up": (INTER, H), "down": (H, INTER)}
    w0 = {n: (torch.randn(*s, generator=gen) * 0.02).to(torch.bfloat16).double()
          for n, s in shapes.items()}
    bias = {n: (torch.randn(shapes[n][0], generator=gen) * 0.02).to(torch.bfloat16).double()
            for n in ("q", "k", "v")}
    wq = {n: _fake_quant(w, gen) for n, w in w0.items()}
    x = torch.randn(T, H, generator=gen, dtype=torch.float64)
    x[:, :8] *= 20.0  # outlier channels
    x = x.float().double()
    with torch.no_grad():
        target = _block(x, w0, bias, lambda a, b: a @ b.t())
    leaves = {n: t.clone().requires_grad_(True) for n, t in wq.items()}
    loss = (_block(x, leaves, bias, lambda a, b: a @ b.t()) - target).pow(2).mean()
    loss.backward()
    return x, target, bias, wq, loss.item(), {n: t.grad for n, t in leaves.items()}


def _errors(problem, roles):
    x, target, bias, wq, loss_ref, grad_ref = problem
    leaves = {n: t.float().clone().requires_grad_(True) for n, t in wq.items()}
    b32 = {n: b.float() for n, b in bias.items()}
    pred = _block(x.float(), leaves, b32, lambda a, b: _Linear.apply(a, b, *roles))
    loss = (pred - target.float()).pow(2).mean()
    loss.backward()
    worst = max(((leaves[n].grad.double() - g).abs().max() / g.abs().max()).item()
                for n, g in grad_ref.items())
    return abs(loss.item() - loss_ref) / loss_ref, worst


def test_three_product_split_meets_the_bar(problem):
    loss_err, grad_err = _errors(problem, (3, 3, 3))
    assert loss_err < 1e-5
    assert grad_err < 1e-4


def test_two_product_forward_misses_the_bar(problem):
    _, grad_err = _errors(problem, (2, 3, 3))
    assert grad_err > 2e-3
