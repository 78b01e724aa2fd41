"""CUDA kernels K1, K2, K4, K5, K6 against the float32 oracle, through the C ABI.

Bar: bit-exact for codes, reconstructions, packed words, scales/biases and
the parameter updates given the same gradient; gradients within 1e-3
max-normalised of the oracle (the reference's bar,
tests/unit/test_mlx_parity.py:264-311) -- in practice ~1e-6; the loss and its
threshold exact or to float64 summation order.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import deltaloss as o_dl
from oracle import losses_fp32 as o_loss
from oracle import packing as o_pack
from oracle import quant_fp32 as o_q
from tests.conftest import relative_error

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-3


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mround_b200 import kernels

    return kernels


def bf16_weight(rng, rows, cols, outliers=True):
    w = rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32)
    if outliers:
        hot = rng.random(size=(rows, cols)) < 0.001
        w[hot] *= 20.0
    return o_pack.bf16_to_f32(o_pack.bf16_bits(w))


def make_case(seed, rows, cols, group, v_range=0.5):
    rng = np.random.default_rng(seed)
    w = bf16_weight(rng, rows, cols)
    ng = cols // group
    v = rng.uniform(-v_range, v_range, size=(rows, cols)).astype(np.float32)
    a = rng.uniform(0.5, 1.0, size=(rows, ng)).astype(np.float32)
    b = rng.uniform(0.5, 1.0, size=(rows, ng)).astype(np.float32)
    gq = rng.normal(0.0, 1e-3, size=(rows, cols)).astype(np.float32)
    return w, v, a, b, gq


def to_dev(w, v, a, b):
    return (torch.from_numpy(w).to(torch.bfloat16).cuda(), torch.from_numpy(v).cuda(),
            torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda())


def bf16_np(t):
    return o_pack.bf16_to_f32(t.view(torch.int16).cpu().numpy().view(np.uint16))


SHAPES = [(24, 256), (96, 896), (40, 1536)]
CONFIGS = [(b, g) for b in (2, 3, 4, 8) for g in (32, 64, 128)]


@pytest.mark.parametrize("bits,group", CONFIGS)
@pytest.mark.parametrize("shape", SHAPES)
def test_fq_forward_bit_exact(K, bits, group, shape):
    rows, cols = shape
    if cols % group:
        pytest.skip("shape not groupable")
    w, v, a, b, _ = make_case(bits * 100 + group, rows, cols, group)
    qdq, codes, scale, zp = o_q.fake_quantize(w, v, a, b, bits, group)
    dw, dv, da, db = to_dev(w, v, a, b)
    hi = torch.empty_like(dw)
    lo = torch.empty_like(dw)
    f32 = torch.empty_like(dv)
    s = torch.empty_like(da)
    z = torch.empty_like(da)
    K.fq_forward(dw, dv, da, db, bits=bits, group=group, eps=1e-8, wq_hi=hi, wq_lo=lo,
                 wq_f32=f32, scale=s, zp=z)
    torch.cuda.synchronize()
    assert np.array_equal(f32.cpu().numpy().view(np.uint32), qdq.view(np.uint32))
    assert np.array_equal(s.cpu().numpy(), scale)
    assert np.array_equal(z.cpu().numpy(), zp)
    hi_np, lo_np = bf16_np(hi), bf16_np(lo)
    assert np.array_equal(hi_np, o_pack.bf16_to_f32(o_pack.bf16_bits(qdq)))
    # hi + lo carries the float32 reconstruction to 16 significant bits
    assert np.all(np.abs((hi_np.astype(np.float64) + lo_np) - qdq) <= np.abs(qdq) * 2.0**-16 + 1e-30)


def test_fq_forward_golden_cases(K, golden):
    for key in [f"q_b{b}_g{g}" for b in (2, 3, 4, 8) for g in (32, 64, 128)]:
        bits, group = int(key.split("_")[1][1:]), int(key.split("_")[2][1:])
        w, v, a, b = (golden[f"{key}_{n}"] for n in ("w", "v", "alpha", "beta"))
        dw, dv, da, db = to_dev(w, v, a, b)
        f32 = torch.empty_like(dv)
        z = torch.empty_like(da)
        K.fq_forward(dw, dv, da, db, bits=bits, group=group, eps=1e-8, wq_f32=f32, zp=z)
        torch.cuda.synchronize()
        assert np.array_equal(z.cpu().numpy(), golden[f"{key}_zp"])
        assert relative_error(f32.cpu().numpy(), golden[f"{key}_qdq"]) < 2e-5


def test_edge_groups_on_device(K):
    # single-sign, all-zero and boundary groups, widened to the device's group of 8
    rows = [[-2.0, -1.5, -1.0, -0.5], [1.0, 1.5, 2.0, 0.25], [-1.0, 0.0, 1.0, 0.5],
            [0.0, 0.0, 0.0, 0.0], [1.0, 0.9, 0.5, -0.3]]
    w = np.array([r * 4 for r in rows], np.float32) * 0.01  # 16 columns, groups of 8
    w = o_pack.bf16_to_f32(o_pack.bf16_bits(w))
    for bits in (2, 4, 8):
        ones = np.ones((w.shape[0], 2), np.float32)
        qdq, codes, scale, zp = o_q.fake_quantize(w, np.zeros_like(w), ones, ones, bits, 8)
        dw, dv, da, db = to_dev(w, np.zeros_like(w), ones, ones)
        f32, z = torch.empty_like(dv), torch.empty_like(da)
        K.fq_forward(dw, dv, da, db, bits=bits, group=8, eps=1e-8, wq_f32=f32, zp=z)
        packed, sc, bi, cd = K.pack_mlx(dw, dv, da, db, bits=bits, group=8, eps=1e-8, want_codes=True)
        torch.cuda.synchronize()
        assert np.array_equal(f32.cpu().numpy().view(np.uint32), qdq.view(np.uint32))
        assert np.array_equal(z.cpu().numpy().view(np.uint32), zp.view(np.uint32))
        assert np.array_equal(cd.cpu().numpy(), codes.astype(np.uint8))
        s_bits, b_bits = o_pack.to_affine(scale, zp)
        assert np.array_equal(bi.view(torch.int16).cpu().numpy().view(np.uint16), b_bits)


@pytest.mark.parametrize("bits,group", CONFIGS)
def test_ste_gradients_match_oracle(K, bits, group):
    rows, cols = 48, 512
    w, v, a, b, gq = make_case(7 + bits + group, rows, cols, group)
    gv_o, ga_o, gb_o = o_q.ste_grads(w, v, a, b, gq, bits, group)
    dw, dv, da, db = to_dev(w, v, a, b)
    g = torch.from_numpy(gq).cuda()
    gv, ga, gb = torch.empty_like(dv), torch.empty_like(da), torch.empty_like(da)
    K.ste_signsgd(g, dw, dv, da, db, bits=bits, group=group, eps=1e-8, lr=0.0, lo=0.1, hi=1.0,
                  update=False, gv=gv, galpha=ga, gbeta=gb)
    torch.cuda.synchronize()
    assert np.array_equal(gv.cpu().numpy(), gv_o), "gV = g*scale*inside is exact"
    assert relative_error(ga.cpu().numpy(), ga_o) < GRAD_TOL
    assert relative_error(gb.cpu().numpy(), gb_o) < GRAD_TOL
    # much tighter in practice: the group sums differ only in order
    assert relative_error(ga.cpu().numpy(), ga_o) < 1e-5
    assert relative_error(gb.cpu().numpy(), gb_o) < 1e-5


@pytest.mark.parametrize("bits,group", [(2, 64), (3, 32), (4, 128), (8, 64)])
def test_signsgd_update_and_fused_requant_bit_exact(K, bits, group):
    rows, cols = 64, 1024
    w, v, a, b, gq = make_case(3 + bits, rows, cols, group)
    lr = o_q.lr_at(0.005, 200, 17)
    dw, dv, da, db = to_dev(w, v, a, b)
    g = torch.from_numpy(gq).cuda()
    gv, ga, gb = torch.empty_like(dv), torch.empty_like(da), torch.empty_like(da)
    hi, lo = torch.empty_like(dw), torch.empty_like(dw)
    K.ste_signsgd(g, dw, dv, da, db, bits=bits, group=group, eps=1e-8, lr=lr, lo=0.1, hi=1.0,
                  update=True, gv=gv, galpha=ga, gbeta=gb, wq_hi=hi, wq_lo=lo)
    torch.cuda.synchronize()
    # the update, given the device's own gradients, is the oracle's step exactly
    v_o, a_o, b_o = o_q.signsgd_step(v, a, b, gv.cpu().numpy(), ga.cpu().numpy(),
                                     gb.cpu().numpy(), lr, 0.1, 1.0)
    assert np.array_equal(dv.cpu().numpy(), v_o)
    assert np.array_equal(da.cpu().numpy(), a_o)
    assert np.array_equal(db.cpu().numpy(), b_o)
    # and the signs it used agree with the oracle's gradients
    _, ga_o, gb_o = o_q.ste_grads(w, v, a, b, gq, bits, group)
    big = np.abs(ga_o) > 1e-6 * np.abs(ga_o).max()
    assert np.array_equal(np.sign(ga.cpu().numpy())[big], np.sign(ga_o)[big])
    # fused re-quantization == K1 on the updated parameters
    qdq, _, _, _ = o_q.fake_quantize(w, v_o, a_o, b_o, bits, group)
    assert np.array_equal(bf16_np(hi), o_pack.bf16_to_f32(o_pack.bf16_bits(qdq)))


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_pack_mlx_bit_exact(K, bits, group):
    rows, cols = 40, 896 if group != 128 else 1024
    w, v, a, b, _ = make_case(bits * 31 + group, rows, cols, group)
    _, codes, scale, zp = o_q.fake_quantize(w, v, a, b, bits, group)
    words = o_pack.pack_codes(codes.astype(np.int64), bits)
    s_bits, b_bits = o_pack.to_affine(scale, zp)
    dw, dv, da, db = to_dev(w, v, a, b)
    packed, sc, bi, cd = K.pack_mlx(dw, dv, da, db, bits=bits, group=group, eps=1e-8, want_codes=True)
    torch.cuda.synchronize()
    assert np.array_equal(cd.cpu().numpy(), codes.astype(np.uint8))
    assert np.array_equal(packed.cpu().numpy().view(np.uint32), words)
    assert np.array_equal(sc.view(torch.int16).cpu().numpy().view(np.uint16), s_bits)
    assert np.array_equal(bi.view(torch.int16).cpu().numpy().view(np.uint16), b_bits)


def test_pack_golden_layout(K, golden):
    # the packed words of codes produced on the device follow the reference packer's layout
    for bits in (2, 3, 4, 5, 6, 7, 8):
        codes = golden[f"pack_b{bits}_codes"]
        assert np.array_equal(o_pack.pack_codes(codes, bits), golden[f"pack_b{bits}_words"])


@pytest.mark.parametrize("shape", [(2, 16, 64), (3, 129, 96), (8, 64, 576)])
@pytest.mark.parametrize("suppress", [True, False])
def test_loss_matches_oracle(K, shape, suppress):
    rng = np.random.default_rng(sum(shape))
    pred = rng.normal(0, 1, size=shape).astype(np.float32)
    tgt = (pred + rng.standard_t(3, size=shape) * 0.05).astype(np.float32)
    loss_o, grad_o, thr_o = o_loss.loss_and_grad(pred, tgt, suppress=suppress)
    ws = K.LossWorkspace()
    dp, dt = torch.from_numpy(pred).cuda(), torch.from_numpy(tgt).cuda()
    grad = torch.empty_like(dp)
    n = pred.size
    K.loss_outlier(dp, dt, ws, suppress=suppress, denom=float(n), k=o_loss.outlier_k(n), grad=grad)
    torch.cuda.synchronize()
    if suppress:
        assert ws.thr.item() == thr_o, "threshold is the exact order statistic"
    assert ws.loss.item() == pytest.approx(loss_o, rel=1e-12)
    assert np.array_equal(grad.cpu().numpy(), grad_o)


def test_loss_with_ties_excludes_all_ties(K):
    # several errors equal to the threshold are all excluded (strict <)
    r = np.zeros(5000, np.float32)
    r[:3] = 9.0
    r[3:8] = 4.0  # k = 5 -> threshold 4.0, and all five 4.0s are dropped
    r[8:] = np.linspace(0.0, 1.0, 4992, dtype=np.float32)
    loss_o, grad_o, thr_o = o_loss.loss_and_grad(r, np.zeros_like(r), suppress=True)
    ws = K.LossWorkspace()
    grad = torch.empty(5000, device="cuda")
    K.loss_outlier(torch.from_numpy(r).cuda(), torch.zeros(5000, device="cuda"), ws, suppress=True,
                   denom=5000.0, k=5, grad=grad)
    torch.cuda.synchronize()
    assert thr_o == 4.0 and ws.thr.item() == 4.0
    assert np.array_equal(grad.cpu().numpy(), grad_o)


def test_loss_piece_uses_given_threshold_and_denominator(K):
    rng = np.random.default_rng(4)
    pred = rng.normal(size=(4, 32, 64)).astype(np.float32)
    tgt = np.zeros_like(pred)
    _, _, thr = o_loss.loss_and_grad(pred, tgt, suppress=True)
    whole = pred.size
    ws = K.LossWorkspace()
    total = 0.0
    for lo, hi in ((0, 2), (2, 4)):
        loss_o, grad_o, _ = o_loss.loss_and_grad(pred[lo:hi], tgt[lo:hi], suppress=True,
                                                 elements=whole, threshold=thr)
        grad = torch.empty(pred[lo:hi].shape, device="cuda")
        K.loss_outlier(torch.from_numpy(np.ascontiguousarray(pred[lo:hi])).cuda(),
                       torch.from_numpy(np.ascontiguousarray(tgt[lo:hi])).cuda(), ws,
                       suppress=True, denom=float(whole), k=1, grad=grad, threshold=float(thr))
        torch.cuda.synchronize()
        assert ws.loss.item() == pytest.approx(loss_o, rel=1e-12)
        assert np.array_equal(grad.cpu().numpy(), grad_o)
        total += ws.loss.item()
    full, _, _ = o_loss.loss_and_grad(pred, tgt, suppress=True)
    assert total == pytest.approx(full, rel=1e-12)


@pytest.mark.parametrize("group", [32, 64, 128])
def test_deltaloss_matches_oracle(K, group):
    rng = np.random.default_rng(group)
    rows, cols = 64, 768
    w = bf16_weight(rng, rows, cols)
    g = rng.normal(0, 1e-2, size=(rows, cols)).astype(np.float32)
    out = torch.zeros(3, dtype=torch.float64, device="cuda")
    K.deltaloss(torch.from_numpy(g).cuda(), torch.from_numpy(w).to(torch.bfloat16).cuda(),
                bits=(2, 3, 4), group=group, eps=1e-8, out=out)
    torch.cuda.synchronize()
    for j, bits in enumerate((2, 3, 4)):
        assert out[j].item() == pytest.approx(o_dl.delta_loss(w, g, bits, group), rel=1e-6)


def test_deltaloss_golden(K, golden):
    w, g = golden["dl_w"], golden["dl_g"]
    for group in (32, 64):
        out = torch.zeros(3, dtype=torch.float64, device="cuda")
        K.deltaloss(torch.from_numpy(g).cuda(), torch.from_numpy(w).to(torch.bfloat16).cuda(),
                    bits=(2, 3, 4), group=group, eps=1e-8, out=out)
        torch.cuda.synchronize()
        for j, bits in enumerate((2, 3, 4)):
            assert out[j].item() == pytest.approx(float(golden[f"dl_b{bits}_g{group}"]), rel=1e-5)


def test_split_bf16(K):
    x = torch.randn(1000003, device="cuda")
    hi, lo = K.split_bf16(x)
    torch.cuda.synchronize()
    xs = x.cpu().numpy()
    h = bf16_np(hi)
    assert np.array_equal(h, o_pack.bf16_to_f32(o_pack.bf16_bits(xs)))
    rec = h.astype(np.float64) + bf16_np(lo)
    assert np.all(np.abs(rec - xs) <= np.abs(xs) * 2.0**-16)


def test_cpu_tensor_is_refused(K):
    from mround_b200.exceptions import PlatformError

    w = torch.zeros(8, 64, dtype=torch.bfloat16)
    with pytest.raises(PlatformError):
        K.fq_forward(w, torch.zeros(8, 64), torch.ones(8, 1), torch.ones(8, 1), bits=2, group=64,
                     eps=1e-8, wq_f32=torch.zeros(8, 64))


def test_division_matches_ieee_over_quantizer_range(K):
    """The quantizer's reciprocal-plus-correction division equals IEEE a / b bit for bit."""
    from mround_b200._native import lib

    g = torch.Generator(device="cuda").manual_seed(0)
    n = 1 << 24
    mant = 1.0 + torch.rand(n, device="cuda", generator=g)
    sign = torch.where(torch.rand(n, device="cuda", generator=g) < 0.5, -1.0, 1.0)
    a = sign * mant * torch.exp2(torch.randint(-40, 4, (n,), device="cuda", generator=g).float())
    b = (1.0 + torch.rand(n, device="cuda", generator=g)) * torch.exp2(
        torch.randint(-27, 2, (n,), device="cuda", generator=g).float())
    # bf16-valued weights against scales built like the quantizer's
    a[: n // 2] = a[: n // 2].to(torch.bfloat16).float()
    a[:1024] = 0.0
    a[1024:2048] = -0.0  # the zero point of a group without negative weights: rint(-0 / s)
    b[:2048] = 1e-8
    # signed (symmetric) scales, and the constant divisors 2^b - 1 and 2^(b-1)
    b[n // 4: n // 2] = -b[n // 4: n // 2]
    divisors = torch.tensor([3.0, 7.0, 15.0, 31.0, 63.0, 127.0, 255.0, 2.0, 4.0, 128.0],
                            device="cuda")
    b[n // 2: n // 2 + (1 << 20)] = divisors[torch.randint(0, 10, (1 << 20,), device="cuda",
                                                           generator=g)]
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib().mr_selftest_division(a.data_ptr(), b.data_ptr(), n, bad.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert bad.item() == 0
