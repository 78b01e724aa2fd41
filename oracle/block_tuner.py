"""Torch-CPU float32 restatement of the per-block tuning loop. TEST ORACLE ONLY.

Also the timed CPU baseline of ``bench.py --impl reference`` (the reference's
own MLX loop cannot run without MLX; this is labelled a restatement).

Follows, in torch float32 on the CPU:

- the fake-quantized linear of ``_TunableLinear.__call__``
  (mround/pipeline/runner.py:346-368) with the STE ops of
  mround/core/quantizer.py: ``round_ste`` (110-116), ``clip_ste`` with an
  inclusive boundary (119-149), the asymmetric scale and zero point
  (254-266) and ``fake_quantize`` (341-347).  Gradients come from torch
  autograd through these ops, as MLX's come from ``mx.value_and_grad`` --
  an independent route from the hand-derived backward of the CUDA kernel;
- the mlx-lm decoder layer (RMSNorm, q/k/v with Qwen2 bias, non-interleaved
  RoPE, causal GQA attention, SwiGLU), as ``block_output`` runs it
  (mround/pipeline/blocks.py:578-606);
- the losses of mround/core/losses.py:42-107;
- ``QuantizationRunner._tune`` (mround/pipeline/runner.py:790-953): mean loss
  over the batches, ``iters`` steps cycling ``step % n_batches``, signSGD with
  linear decay and projection, mean loss again, revert if not improved; and
  ``_commit`` (761-788): the committed weight is bf16(reconstruction).
"""

from __future__ import annotations

import math
import time

import torch
import torch.nn.functional as F

__all__ = ["OracleBlock", "fake_quant_ste", "loss_fn", "tune_block"]

V_BOUND = 0.5


def _round_ste(x):
    return x + (torch.round(x) - x).detach()  # torch.round is ties-to-even


def _clip_ste(x, lo, hi):
    inside = ((x >= lo) & (x <= hi)).to(x.dtype).detach()
    through = x * inside
    return through + (torch.clamp(x, lo, hi) - through).detach()


def _clamp_magnitude(s, eps):
    """sign(s) * max(|s|, eps), sign(0) = +1 (mround/core/quantizer.py:216-225)."""
    sign = torch.sign(s).detach()
    sign = torch.where(sign == 0, torch.ones_like(sign), sign)
    return sign * torch.clamp(s.abs(), min=eps)


def fake_quant_ste(w, v, alpha, beta, bits, group, eps=1e-8, *, symmetric=False, init_scale=None):
    """Differentiable fake quantization of w (out, in) float32.

    Asymmetric (default), symmetric observed range (``symmetric``) or
    searched (``init_scale``, (out, in/group)): mround/core/quantizer.py:
    228-266, 319-347.
    """
    rows, cols = w.shape
    g = w.view(rows, cols // group, group)
    a = alpha.view(rows, cols // group, 1)
    b = beta.view(rows, cols // group, 1)
    if symmetric or init_scale is not None:
        maxq = float(2 ** (bits - 1))
        if init_scale is not None:
            s = init_scale.view(rows, cols // group, 1) * b
        else:
            gmax = g.amax(-1, keepdim=True)
            gmin = g.amin(-1, keepdim=True)
            pos_mag = torch.where(gmax > 0, gmax, torch.zeros_like(gmax)) * a
            neg_mag = -(torch.where(gmin < 0, gmin, torch.zeros_like(gmin)) * b)
            pos = (pos_mag >= neg_mag).detach()
            dominant = torch.where(pos, pos_mag, neg_mag)
            s = torch.where(pos, -dominant, dominant) / maxq
        scale = _clamp_magnitude(s, eps)
        raw = g / scale + v.view(g.shape)
        codes = _clip_ste(_round_ste(raw), -maxq, maxq - 1.0)
        return (scale * codes).view(rows, cols)
    maxq = float(2**bits - 1)
    gmax = g.amax(-1, keepdim=True)
    gmin = g.amin(-1, keepdim=True)
    w_max = torch.where(gmax > 0, gmax, torch.zeros_like(gmax)) * a
    w_min = torch.where(gmin < 0, gmin, torch.zeros_like(gmin)) * b
    scale = torch.clamp((w_max - w_min) / maxq, min=eps)
    zp = _round_ste(-w_min / scale)
    raw = g / scale + v.view(g.shape)
    codes = _clip_ste(_round_ste(raw) + zp, 0.0, maxq)
    return (scale * (codes - zp)).view(rows, cols)


def rms_norm(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def rope(x, theta):
    s, d = x.shape[-2], x.shape[-1]
    half = d // 2
    inv = theta ** (-torch.arange(0, half, dtype=torch.float64) * 2.0 / d)
    ang = torch.arange(s, dtype=torch.float64)[:, None] * inv[None, :]
    cos, sin = torch.cos(ang).float(), torch.sin(ang).float()
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat((x1 * cos - x2 * sin, x1 * sin + x2 * cos), dim=-1)


def attention(q, k, v, scale):
    """Causal grouped-query attention, explicit float32 math."""
    rep = q.shape[1] // k.shape[1]
    k = k.repeat_interleave(rep, dim=1)
    v = v.repeat_interleave(rep, dim=1)
    s = q.shape[-2]
    scores = (q @ k.transpose(-1, -2)) * scale
    mask = torch.ones(s, s, dtype=torch.bool).triu(1)
    scores = scores.masked_fill(mask, float("-inf"))
    return torch.softmax(scores, dim=-1) @ v


LINEARS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
           "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


class OracleBlock:
    """A decoder block on the CPU in float32.

    ``weights[path]`` are float32 exact widenings of the bf16 weights.
    ``params[path] = (v, alpha, beta)`` float32 leaves; ``None`` runs dense.
    ``committed[path]`` (if set) replaces the weight by a given tensor.
    """

    def __init__(self, arch, block_params, bits: dict[str, int], group: int, *,
                 symmetric: bool = False, init_scales: dict[str, torch.Tensor] | None = None):
        self.arch = arch
        self.symmetric = symmetric
        self.init_scales = init_scales
        self.w = {p: t.float() for p, t in block_params.linears.items()}
        self.b = {p: t.float() for p, t in block_params.biases.items()}
        self.n_in = block_params.input_norm.float()
        self.n_post = block_params.post_norm.float()
        self.bits = bits
        self.group = group
        self.committed: dict[str, torch.Tensor] = {}

    def init_params(self):
        out = {}
        for p in LINEARS:
            rows, cols = self.w[p].shape
            ng = cols // self.group
            out[p] = (torch.zeros(rows, cols), torch.ones(rows, ng), torch.ones(rows, ng))
        return out

    def weight(self, p, params):
        if p in self.committed:
            return self.committed[p]
        if params is None:
            return self.w[p]
        v, a, b = params[p]
        init = None if self.init_scales is None else self.init_scales[p]
        return fake_quant_ste(self.w[p], v, a, b, self.bits[p], self.group,
                              symmetric=self.symmetric, init_scale=init)

    def forward(self, x, params=None):
        ar = self.arch
        bsz, s, _ = x.shape

        def lin(p, inp):
            y = inp @ self.weight(p, params).t()
            return y + self.b[p] if p in self.b else y

        h1 = rms_norm(x, self.n_in, ar.rms_eps)
        q = lin("self_attn.q_proj", h1).view(bsz, s, ar.heads, ar.head_dim).transpose(1, 2)
        k = lin("self_attn.k_proj", h1).view(bsz, s, ar.kv_heads, ar.head_dim).transpose(1, 2)
        v = lin("self_attn.v_proj", h1).view(bsz, s, ar.kv_heads, ar.head_dim).transpose(1, 2)
        q, k = rope(q, ar.rope_theta), rope(k, ar.rope_theta)
        att = attention(q, k, v, 1.0 / math.sqrt(ar.head_dim)).transpose(1, 2).reshape(bsz, s, -1)
        h = x + lin("self_attn.o_proj", att)
        h2 = rms_norm(h, self.n_post, ar.rms_eps)
        return h + lin("mlp.down_proj", F.silu(lin("mlp.gate_proj", h2)) * lin("mlp.up_proj", h2))


def loss_fn(pred, target, suppress: bool, fraction: float = 0.001):
    r = pred - target
    n = r.numel()
    if not suppress:
        return (r * r).mean(), None
    k = max(1, int(n * fraction))
    thr = torch.sort(r.detach().abs().reshape(-1)).values[n - k]
    kept = r * (r.abs() < thr).float()
    return (kept * kept).sum() / n, thr


def tune_block(block: OracleBlock, inputs, targets, *, iters: int, lr0: float, suppress: bool,
               lo: float = 0.1, hi: float = 1.0, record_grads_at: int | None = None,
               step_budget_s: float | None = None, max_steps: int | None = None,
               warmup_steps: int = 0):
    """Restated ``_tune``; returns a dict with losses, params and timing.

    ``record_grads_at`` stores the loss and parameter gradients of that step
    (for parity tests).  ``step_budget_s`` stops early after that many seconds
    of timed steps, ``max_steps`` after that many timed steps (a bounded
    timing sample); the first ``warmup_steps`` steps run untimed.  The result
    says how many steps were timed (``steps_run``) and their seconds;
    ``score_seconds`` is the time of the first scoring pass (one forward and
    loss per batch).
    """
    params = block.init_params()
    nb = len(inputs)

    def mean_loss(pr):
        with torch.no_grad():
            vals = [float(loss_fn(block.forward(inputs[i], pr), targets[i], suppress)[0])
                    for i in range(nb)]
        return sum(vals) / nb, vals

    t_score = time.perf_counter()
    initial, _ = mean_loss(params)
    score_seconds = time.perf_counter() - t_score
    step_losses, recorded = [], None
    t0 = time.perf_counter()
    ran = 0

    def grad_of(t):
        # a parameter that does not reach the loss (alpha under a searched
        # scale) has no gradient: sign(0) = 0 leaves it in place
        return t.grad if t.grad is not None else torch.zeros_like(t)

    for step in range(iters):
        leaves = {p: tuple(t.clone().requires_grad_(True) for t in params[p]) for p in params}
        loss, _ = loss_fn(block.forward(inputs[step % nb], leaves), targets[step % nb], suppress)
        loss.backward()
        step_losses.append(float(loss.detach()))
        if record_grads_at == step:
            recorded = {p: tuple(grad_of(t).clone() for t in leaves[p]) for p in leaves}
            recorded["__loss__"] = float(loss)
        lr = lr0 * (1.0 - step / iters)
        lr32 = torch.tensor(lr, dtype=torch.float32)
        new = {}
        for p, (v, a, b) in leaves.items():
            nv = torch.clamp(v.detach() - lr32 * torch.sign(grad_of(v)), -V_BOUND, V_BOUND)
            na = torch.clamp(a.detach() - lr32 * torch.sign(grad_of(a)), lo, hi)
            nb_ = torch.clamp(b.detach() - lr32 * torch.sign(grad_of(b)), lo, hi)
            new[p] = (nv, na, nb_)
        params = new
        if step < warmup_steps:
            t0 = time.perf_counter()
            continue
        ran += 1
        if step_budget_s is not None and time.perf_counter() - t0 > step_budget_s:
            break
        if max_steps is not None and ran >= max_steps:
            break
    step_seconds = time.perf_counter() - t0
    finished = ran + min(warmup_steps, iters) == iters
    final, _ = mean_loss(params) if finished else (float("nan"), None)
    reverted = finished and final >= initial
    return {
        "initial_loss": initial,
        "final_loss": initial if reverted else final,
        "reverted": reverted,
        "params": block.init_params() if reverted else params,
        "step_losses": step_losses,
        "recorded": recorded,
        "steps_run": ran,
        "step_seconds": step_seconds,
        "score_seconds": score_seconds,
    }
