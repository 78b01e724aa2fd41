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
