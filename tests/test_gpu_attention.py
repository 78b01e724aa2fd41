"""Attention on K3 against a float64 reference of the same math (causal GQA)."""

from __future__ import annotations

import math

import pytest
import torch

from tests.conftest import relative_error

pytestmark = pytest.mark.gpu


def reference(q, k, v, scale):
    rep = q.shape[1] // k.shape[1]
    k = k.repeat_interleave(rep, 1)
    v = v.repeat_interleave(rep, 1)
    s = q.shape[2]
    sc = (q @ k.transpose(-1, -2)) * scale
    sc = sc.masked_fill(torch.ones(s, s, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
    return torch.softmax(sc, -1) @ v


@pytest.mark.parametrize("b,hq,hkv,s,d", [(2, 4, 2, 128, 32), (1, 7, 1, 256, 128), (2, 14, 2, 64, 64)])
def test_attention_forward_backward(b, hq, hkv, s, d):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mround_b200.pipeline.attention import attention

    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(b, hq, s, d, device="cuda", generator=g).requires_grad_(True)
    k = torch.randn(b, hkv, s, d, device="cuda", generator=g).requires_grad_(True)
    v = torch.randn(b, hkv, s, d, device="cuda", generator=g).requires_grad_(True)
    do = torch.randn(b, hq, s, d, device="cuda", generator=g)
    scale = 1.0 / math.sqrt(d)
    out = attention(q, k, v, scale)
    out.backward(do)
    q64, k64, v64 = (t.detach().double().requires_grad_(True) for t in (q, k, v))
    ref = reference(q64, k64, v64, scale)
    ref.backward(do.double())
    assert relative_error(out.detach().cpu().numpy(), ref.detach().cpu().numpy()) < 5e-5
    for got, want in ((q.grad, q64.grad), (k.grad, k64.grad), (v.grad, v64.grad)):
        assert relative_error(got.cpu().numpy(), want.cpu().numpy()) < 5e-5


@pytest.mark.parametrize("s,band", [(64, False), (256, True), (2048, True), (1000, False)])
def test_softmax_kernels_match_float64(s, band):
    """K7 causal softmax and its backward against float64: P = hi + lo to 2^-15
    of the row's maximum; zeros above the diagonal up to the band limit."""
    from mround_b200 import kernels

    g = torch.Generator(device="cuda").manual_seed(s)
    rows = 3 * s
    scores = torch.randn(rows, s, device="cuda", generator=g) * 3.0
    dp = torch.randn(rows, s, device="cuda", generator=g)
    scale = 0.088
    keep = scores.clone()
    p = kernels.softmax_causal_split(scores, rows, s, scale, band)
    ds = kernels.softmax_bwd_split(dp, p, rows, s, scale, band)
    torch.cuda.synchronize()
    assert torch.equal(scores, keep), "scores are read-only"
    pos = torch.arange(rows, device="cuda") % s
    col = torch.arange(s, device="cuda")
    mask = col[None, :] <= pos[:, None]
    ref = torch.softmax((scores.double() * scale).masked_fill(~mask, float("-inf")), -1)
    got = p[0].double() + p[1].double()
    dref = scale * ref * (dp.double() - (dp.double() * ref).sum(-1, keepdim=True))
    dgot = ds[0].double() + ds[1].double()
    lim = torch.minimum(((pos // 128) + 2) * 128, torch.tensor(s, device="cuda")) if band \
        else torch.full_like(pos, s)
    written = col[None, :] < lim[:, None]
    assert ((got - ref).abs() * written).max() <= 2.0 ** -15
    assert (got[written & ~mask] == 0).all()
    tol = 2.0 ** -14 * dref.abs().max()
    assert ((dgot - dref).abs() * written).max() <= tol


def _rot(x1, x2, c, sn):
    return x1 * c - x2 * sn, x1 * sn + x2 * c


@pytest.mark.parametrize("b,s,hq,hkv,d", [(2, 64, 4, 2, 64), (1, 48, 3, 1, 128), (2, 16, 2, 1, 12)])
def test_rope_and_head_layout_kernels_match_float64(b, s, hq, hkv, d):
    """K7 RoPE (+bwd) and the head merge/split against float64 (head dims
    divisible by 8 take the token-row kernels; d = 12 the element-wise ones).
    hi + lo carries 16 significant bits, so values agree to 2^-15 of the largest."""
    from mround_b200 import kernels

    g = torch.Generator(device="cuda").manual_seed(d)
    h = hq + 2 * hkv
    half = d // 2
    qkv = torch.randn(b * s, h * d, device="cuda", generator=g)
    ang = torch.rand(s, half, device="cuda", generator=g) * 6.0
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    q, k, v = kernels.rope_split(qkv, cos, sin, b, s, hq, hkv, d)
    x = qkv.double().view(b, s, h, d).permute(0, 2, 1, 3)  # (b, h, s, d)
    c, sn = cos.double()[None, None], sin.double()[None, None]
    o1, o2 = _rot(x[..., :half], x[..., half:], c, sn)
    rot = torch.cat([o1, o2], -1)
    want = {"q": rot[:, :hq], "k": rot[:, hq:hq + hkv], "v": x[:, hq + hkv:]}
    for name, got in (("q", q), ("k", k), ("v", v)):
        val = got[0].double() + got[1].double()
        ref = want[name]
        assert (val - ref).abs().max().item() <= 2.0 ** -15 * ref.abs().max().item(), name

    dq = torch.randn(b, hq, s, d, device="cuda", generator=g)
    dk = torch.randn(b, hkv, s, d, device="cuda", generator=g)
    dv = torch.randn(b, hkv, s, d, device="cuda", generator=g)
    hi, lo, _ = kernels.rope_bwd_split(dq, dk, dv, cos, sin, b, s, hq, hkv, d)
    dd = torch.cat([dq, dk, dv], 1).double()  # (b, h, s, d)
    g1 = dd[..., :half] * c + dd[..., half:] * sn
    g2 = dd[..., half:] * c - dd[..., :half] * sn
    back = torch.cat([g1, g2], -1)
    back[:, hq + hkv:] = dd[:, hq + hkv:]
    ref = back.permute(0, 2, 1, 3).reshape(b * s, h * d)
    val = hi.double() + lo.double()
    assert (val - ref).abs().max().item() <= 2.0 ** -15 * ref.abs().max().item()

    if d % 4 == 0:
        heads = torch.randn(b, h, s, d, device="cuda", generator=g)
        mh, ml, _ = kernels.heads_split(heads, b, s, h, d, merge=True)
        ref = heads.permute(0, 2, 1, 3).reshape(b * s, h * d)
        assert torch.equal(mh.float() + ml.float(), (ref.to(torch.bfloat16).float()
                                                      + (ref - ref.to(torch.bfloat16).float())
                                                      .to(torch.bfloat16).float()))
        rows = torch.randn(b * s, h * d, device="cuda", generator=g)
        sh, sl, _ = kernels.heads_split(rows, b, s, h, d, merge=False)
        ref = rows.view(b, s, h, d).permute(0, 2, 1, 3)
        assert torch.equal(sh.float() + sl.float(), (ref.to(torch.bfloat16).float()
                                                      + (ref - ref.to(torch.bfloat16).float())
                                                      .to(torch.bfloat16).float()))


@pytest.mark.parametrize("rows,vocab", [(7, 512), (64, 151936), (3, 49152)])
def test_ce_grad_split_matches_float64(rows, vocab):
    """The scoring backward's cross-entropy gradient kernel against a float64
    softmax minus the one-hot labels, scaled by 1/rows (hi + lo to 2^-15)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mround_b200 import kernels

    g = torch.Generator(device="cuda").manual_seed(rows)
    logits = torch.randn(rows, vocab, device="cuda", generator=g) * 4.0
    labels = torch.randint(0, vocab, (rows,), device="cuda", generator=g)
    hi, lo = kernels.ce_grad_split(logits, labels, 1.0 / rows)
    ref = torch.softmax(logits.double(), -1)
    ref[torch.arange(rows, device="cuda"), labels] -= 1.0
    ref /= rows
    got = hi.double() + lo.double()
    assert (got - ref).abs().max().item() <= 2.0 ** -15 * ref.abs().max().item()
