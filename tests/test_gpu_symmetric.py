"""Symmetric and searched schemes on the device (K1, K2, K5, K6 modes), the
scale search (K8) and the importance statistics, through the C ABI.

Bar: codes, reconstructions, scales, packed words, scales/biases and
parameter updates bit-exact against the float32 oracle; gradients 1e-3
max-normalised (the reference's bar, tests/unit/test_mlx_parity.py:264-311),
in practice ~1e-6; the search bit-exact against the float32 oracle that sums
in the kernel's order, and against the reference's float64 search the same
choice in >= 98 % of groups (95 % weighted) with no worse reconstruction where
it differs (test_mlx_parity.py:615-670).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import deltaloss as o_dl
from oracle import packing as o_pack
from oracle import quant_fp32 as o_q
from oracle import scale_search as o_s
from tests.conftest import relative_error

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-3
CONFIGS = [(b, g) for b in (2, 3, 4, 8) for g in (32, 64, 128)]


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mround_b200 import kernels

    return kernels


def bf16_round(x):
    return o_pack.bf16_to_f32(o_pack.bf16_bits(np.asarray(x, np.float32)))


def make_case(seed, rows, cols, group, searched):
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32)
    hot = rng.random(size=(rows, cols)) < 0.001
    w[hot] *= 20.0
    w = bf16_round(w)
    ng = cols // group
    v = rng.uniform(-0.5, 0.5, size=(rows, cols)).astype(np.float32)
    lo, hi = (0.5, 1.5) if searched else (0.5, 1.0)
    a = rng.uniform(lo, hi, size=(rows, ng)).astype(np.float32)
    b = rng.uniform(lo, hi, size=(rows, ng)).astype(np.float32)
    gq = rng.normal(0.0, 1e-3, size=(rows, cols)).astype(np.float32)
    return w, v, a, b, gq


def dev(*arrays):
    out = []
    for i, x in enumerate(arrays):
        t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        out.append(t.to(torch.bfloat16) if i == 0 else t)
    return out


def bf16_np(t):
    return o_pack.bf16_to_f32(t.view(torch.int16).cpu().numpy().view(np.uint16))


def init_for(K, w, bits, group, searched):
    """The searched scale from the oracle (float32), or None."""
    if not searched:
        return None, None
    init = o_s.search_scales_f32(w, bits, group).reshape(w.shape[0], -1)
    return init, torch.from_numpy(init).cuda()


@pytest.mark.parametrize("searched", [False, True])
@pytest.mark.parametrize("bits,group", CONFIGS)
def test_fq_forward_sym_bit_exact(K, bits, group, searched):
    rows, cols = 48, 768 if group != 128 else 1024
    w, v, a, b, _ = make_case(bits * 10 + group + searched, rows, cols, group, searched)
    init, dinit = init_for(K, w, bits, group, searched)
    qdq, codes, scale, zp = o_q.fake_quantize(w, v, a, b, bits, group, symmetric=True,
                                              init_scale=init)
    dw, dv, da, db = dev(w, v, a, b)
    f32, hi, lo = torch.empty_like(dv), torch.empty_like(dw), torch.empty_like(dw)
    s = torch.empty_like(da)
    K.fq_forward(dw, dv, da, db, bits=bits, group=group, eps=1e-8, wq_hi=hi, wq_lo=lo, wq_f32=f32,
                 scale=s, symmetric=True, init_scale=dinit)
    torch.cuda.synchronize()
    assert np.array_equal(f32.cpu().numpy().view(np.uint32), qdq.view(np.uint32))
    assert np.array_equal(s.cpu().numpy().view(np.uint32), scale.view(np.uint32))
    assert np.array_equal(bf16_np(hi), bf16_round(qdq))
    if not searched:
        assert (s.cpu().numpy() < 0).any() and (s.cpu().numpy() > 0).any(), "signed scales"


def test_fq_forward_sym_golden(K, golden):
    for key in [f"s{i}_b{b}_g{g}" for i in ("o", "s") for b in (2, 3, 4, 8) for g in (32, 64, 128)]:
        bits, group = int(key.split("_")[1][1:]), int(key.split("_")[2][1:])
        w, v, a, b = (golden[f"{key}_{n}"] for n in ("w", "v", "alpha", "beta"))
        init = golden.get(f"{key}_init")
        dw, dv, da, db = dev(w, v, a, b)
        f32, s = torch.empty_like(dv), torch.empty_like(da)
        K.fq_forward(dw, dv, da, db, bits=bits, group=group, eps=1e-8, wq_f32=f32, scale=s,
                     symmetric=True,
                     init_scale=None if init is None else torch.from_numpy(init).cuda())
        torch.cuda.synchronize()
        assert relative_error(s.cpu().numpy(), golden[f"{key}_scale"]) < 2e-5, key
        assert relative_error(f32.cpu().numpy(), golden[f"{key}_qdq"]) < 2e-5, key


@pytest.mark.parametrize("searched", [False, True])
@pytest.mark.parametrize("bits,group", CONFIGS)
def test_ste_sym_gradients_match_oracle(K, bits, group, searched):
    rows, cols = 48, 512
    w, v, a, b, gq = make_case(31 + bits + group + searched, rows, cols, group, searched)
    init, dinit = init_for(K, w, bits, group, searched)
    gv_o, ga_o, gb_o = o_q.ste_grads(w, v, a, b, gq, bits, group, symmetric=True, init_scale=init)
    dw, dv, da, db = dev(w, v, a, b)
    g = torch.from_numpy(gq).cuda()
    gv, ga, gb = torch.empty_like(dv), torch.empty_like(da), torch.empty_like(da)
    K.ste_signsgd(g, dw, dv, da, db, bits=bits, group=group, eps=1e-8, lr=0.0, lo=0.1, hi=1.5,
                  update=False, gv=gv, galpha=ga, gbeta=gb, symmetric=True, init_scale=dinit)
    torch.cuda.synchronize()
    assert np.array_equal(gv.cpu().numpy(), gv_o), "gV = g*scale*inside is exact"
    assert relative_error(ga.cpu().numpy(), ga_o) < 1e-5
    assert relative_error(gb.cpu().numpy(), gb_o) < 1e-5
    if searched:
        assert not ga.cpu().numpy().any(), "alpha is inert under a searched scale"
    else:
        both = (ga.cpu().numpy() != 0) & (gb.cpu().numpy() != 0)
        assert not both.any(), "only the dominant side's coefficient receives gradient"


def test_ste_sym_golden(K, golden):
    for key in [f"s{i}_b{b}_g{g}" for i in ("o", "s") for b in (2, 3, 4, 8) for g in (32, 64, 128)]:
        bits, group = int(key.split("_")[1][1:]), int(key.split("_")[2][1:])
        w, v, a, b, gq = (golden[f"{key}_{n}"] for n in ("w", "v", "alpha", "beta", "gq"))
        init = golden.get(f"{key}_init")
        dw, dv, da, db = dev(w, v, a, b)
        gv, ga, gb = torch.empty_like(dv), torch.empty_like(da), torch.empty_like(da)
        K.ste_signsgd(torch.from_numpy(gq).cuda(), dw, dv, da, db, bits=bits, group=group,
                      eps=1e-8, lr=0.0, lo=0.1, hi=1.5, update=False, gv=gv, galpha=ga, gbeta=gb,
                      symmetric=True,
                      init_scale=None if init is None else torch.from_numpy(init).cuda())
        torch.cuda.synchronize()
        for name, got in (("gv", gv), ("galpha", ga), ("gbeta", gb)):
            err = relative_error(got.cpu().numpy(), golden[f"{key}_{name}"])
            assert err < GRAD_TOL, (key, name, err)


@pytest.mark.parametrize("searched", [False, True])
@pytest.mark.parametrize("bits,group", [(2, 64), (3, 32), (4, 128), (8, 64)])
def test_sym_update_and_fused_requant_bit_exact(K, bits, group, searched):
    rows, cols = 64, 1024
    w, v, a, b, gq = make_case(5 + bits + searched, rows, cols, group, searched)
    init, dinit = init_for(K, w, bits, group, searched)
    lo_b, hi_b = (0.5, 1.5) if searched else (0.1, 1.0)
    lr = o_q.lr_at(0.005, 200, 17)
    dw, dv, da, db = dev(w, v, a, b)
    g = torch.from_numpy(gq).cuda()
    gv, ga, gb = torch.empty_like(dv), torch.empty_like(da), torch.empty_like(da)
    hi, lo = torch.empty_like(dw), torch.empty_like(dw)
    K.ste_signsgd(g, dw, dv, da, db, bits=bits, group=group, eps=1e-8, lr=lr, lo=lo_b, hi=hi_b,
                  update=True, gv=gv, galpha=ga, gbeta=gb, wq_hi=hi, wq_lo=lo, symmetric=True,
                  init_scale=dinit)
    torch.cuda.synchronize()
    v_o, a_o, b_o = o_q.signsgd_step(v, a, b, gv.cpu().numpy(), ga.cpu().numpy(),
                                     gb.cpu().numpy(), lr, lo_b, hi_b)
    assert np.array_equal(dv.cpu().numpy(), v_o)
    assert np.array_equal(da.cpu().numpy(), a_o)
    assert np.array_equal(db.cpu().numpy(), b_o)
    qdq, _, _, _ = o_q.fake_quantize(w, v_o, a_o, b_o, bits, group, symmetric=True,
                                     init_scale=init)
    assert np.array_equal(bf16_np(hi), bf16_round(qdq))


@pytest.mark.parametrize("searched", [False, True])
@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("group", [32, 64])
def test_pack_mlx_sym_bit_exact(K, bits, group, searched):
    rows, cols = 40, 896
    w, v, a, b, _ = make_case(bits * 7 + group + searched, rows, cols, group, searched)
    init, dinit = init_for(K, w, bits, group, searched)
    _, codes, scale, _ = o_q.fake_quantize(w, v, a, b, bits, group, symmetric=True, init_scale=init)
    half = 1 << (bits - 1)
    words = o_pack.pack_codes((codes + half).astype(np.int64), bits)
    s_bits, b_bits = o_pack.to_affine(scale, None, bits)
    dw, dv, da, db = dev(w, v, a, b)
    packed, sc, bi, cd = K.pack_mlx(dw, dv, da, db, bits=bits, group=group, eps=1e-8,
                                    want_codes=True, symmetric=True, init_scale=dinit)
    torch.cuda.synchronize()
    assert cd.dtype == torch.int8
    assert np.array_equal(cd.cpu().numpy(), codes.astype(np.int8))
    assert np.array_equal(packed.cpu().numpy().view(np.uint32), words)
    assert np.array_equal(sc.view(torch.int16).cpu().numpy().view(np.uint16), s_bits)
    assert np.array_equal(bi.view(torch.int16).cpu().numpy().view(np.uint16), b_bits)
    # stored code 0 decodes to the bias: W = scales * q_u + biases
    s = bf16_np(sc).repeat(group, axis=1)
    bia = bf16_np(bi).repeat(group, axis=1)
    recon = s * (codes + half) + bia
    assert np.allclose(recon, (bf16_np(sc).repeat(group, axis=1) * codes), rtol=1e-6, atol=1e-9)


def test_sym_edge_groups(K):
    # single-sign, all-zero, a |max| tie and a group where the negative side dominates
    rows = [[-2.0, -1.5, -1.0, -0.5], [1.0, 1.5, 2.0, 0.25], [-1.0, 0.0, 1.0, 0.5],
            [0.0, 0.0, 0.0, 0.0], [1.0, 0.9, 0.5, -0.3]]
    w = bf16_round(np.array([r * 4 for r in rows], np.float32) * 0.01)
    for bits in (2, 4, 8):
        ones = np.ones((w.shape[0], 2), np.float32)
        zeros = np.zeros_like(w)
        qdq, codes, scale, _ = o_q.fake_quantize(w, zeros, ones, ones, bits, 8, symmetric=True)
        assert scale[3, 0] == np.float32(1e-8)
        dw, dv, da, db = dev(w, zeros, ones, ones)
        f32, s = torch.empty_like(dv), torch.empty_like(da)
        K.fq_forward(dw, dv, da, db, bits=bits, group=8, eps=1e-8, wq_f32=f32, scale=s,
                     symmetric=True)
        packed, sc, bi, cd = K.pack_mlx(dw, dv, da, db, bits=bits, group=8, eps=1e-8,
                                        want_codes=True, symmetric=True)
        torch.cuda.synchronize()
        assert np.array_equal(f32.cpu().numpy().view(np.uint32), qdq.view(np.uint32))
        assert np.array_equal(s.cpu().numpy().view(np.uint32), scale.view(np.uint32))
        assert np.array_equal(cd.cpu().numpy(), codes.astype(np.int8))


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
@pytest.mark.parametrize("group", [16, 32, 64, 128])
@pytest.mark.parametrize("weighted", [False, True])
def test_scale_search_bit_exact_vs_oracle(K, bits, group, weighted):
    rng = np.random.default_rng(bits * 1000 + group + weighted)
    rows, cols = 64, 512
    w = rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32)
    w[rng.random(size=w.shape) < 0.002] *= 20.0
    w = bf16_round(w)
    w[3, :group] = 0.0  # an all-zero group
    imp = rng.uniform(0.1, 10.0, size=cols).astype(np.float32) if weighted else None
    want = o_s.search_scales_f32(w, bits, group, imp).reshape(rows, -1)
    got = K.scale_search(torch.from_numpy(w).to(torch.bfloat16).cuda(), bits=bits, group=group,
                         candidates=o_s.candidates(bits).tolist(),
                         importance=None if imp is None else torch.from_numpy(imp).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert got[3, 0].item() == 0.0


def test_scale_search_golden(K, golden):
    from mround_b200.core.scale_search import search_scales
    from mround_b200.schemes import QuantScheme

    for key in [f"srch_b{b}_g{g}" for b in (2, 3, 4, 8) for g in (32, 64)]:
        bits, group = int(key.split("_")[1][1:]), int(key.split("_")[2][1:])
        w = golden[f"{key}_w"]
        got = search_scales(torch.from_numpy(w).to(torch.bfloat16).cuda(),
                            QuantScheme(bits=bits, group_size=group)).cpu().numpy()
        want = golden[f"{key}_scale"]
        same = np.isclose(got, want, rtol=1e-5, atol=1e-8)
        assert same.mean() >= 0.98, (key, same.mean())
        grouped = w.astype(np.float64).reshape(-1, group)
        nmax = float(2 ** (bits - 1))
        for row in np.flatnonzero(~same.ravel()):
            losses = []
            for s in (float(got.ravel()[row]), float(want.ravel()[row])):
                inv = 0.0 if s == 0 else 1.0 / s
                c = np.clip(np.rint(inv * grouped[row]), -nmax, nmax - 1)
                losses.append(float(np.sum((s * c - grouped[row]) ** 2)))
            assert losses[0] <= losses[1] * (1 + 1e-4), (key, row, losses)
    w, imp = golden["srch_imp_w"], golden["srch_imp_importance"]
    got = search_scales(torch.from_numpy(w).to(torch.bfloat16).cuda(),
                        QuantScheme(bits=3, group_size=16),
                        importance=torch.from_numpy(imp).cuda()).cpu().numpy()
    assert np.isclose(got, golden["srch_imp_scale"], rtol=1e-5, atol=1e-8).mean() >= 0.95
    for bits in (2, 4):
        got = search_scales(torch.from_numpy(golden["srch_edge_w"]).to(torch.bfloat16).cuda(),
                            QuantScheme(bits=bits, group_size=16)).cpu().numpy()
        assert np.allclose(got, golden[f"srch_edge_b{bits}_scale"], rtol=1e-5, atol=1e-8)


def test_scale_search_large_matrix_matches_reference_f64(K):
    # a full-width 7B down projection slice: the choice statistic over 100k+ groups
    rng = np.random.default_rng(77)
    rows, cols, group, bits = 448, 18944, 64, 2
    w = bf16_round(rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32))
    got = K.scale_search(torch.from_numpy(w).to(torch.bfloat16).cuda(), bits=bits, group=group,
                         candidates=o_s.candidates(bits).tolist()).cpu().numpy().reshape(-1, 1)
    # the float64 oracle on the first 64 rows (18944 groups)
    want = o_s.search_scales_f64(w[:64], bits, group)
    same = np.isclose(got[: want.shape[0]], want, rtol=1e-5, atol=1e-8)
    assert same.mean() >= 0.98
    # and the float32 oracle in the kernel's summation order, exactly
    want32 = o_s.search_scales_f32(w[:64], bits, group)
    assert np.array_equal(got[: want.shape[0]].view(np.uint32), want32.view(np.uint32))


def test_colsumsq_matches_float64(K):
    rng = np.random.default_rng(3)
    x = rng.normal(0.0, 1.0, size=(1000, 896)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    hi, lo = K.split_bf16(xd)
    out = torch.full((896,), 0.5, device="cuda")
    K.colsumsq_split(hi, lo, out)
    torch.cuda.synchronize()
    parts = bf16_np(hi).astype(np.float64) + bf16_np(lo)
    want = 0.5 + (parts ** 2).sum(axis=0)
    assert np.allclose(out.cpu().numpy(), want, rtol=1e-5)


@pytest.mark.parametrize("searched", [False, True])
@pytest.mark.parametrize("group", [32, 64])
def test_deltaloss_sym_matches_oracle(K, group, searched):
    rng = np.random.default_rng(group + 7 * searched)
    rows, cols = 64, 768
    w = bf16_round(rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32))
    g = rng.normal(0.0, 1e-2, size=(rows, cols)).astype(np.float32)
    widths = (2, 3, 4)
    grids = [o_s.search_scales_f32(w, b, group).reshape(rows, -1) for b in widths] if searched \
        else [None] * 3
    want = [o_dl.delta_loss(w, g, b, group, symmetric=True, init_scale=gr)
            for b, gr in zip(widths, grids)]
    out = torch.zeros(3, dtype=torch.float64, device="cuda")
    K.deltaloss(torch.from_numpy(g).cuda(), torch.from_numpy(w).to(torch.bfloat16).cuda(),
                bits=widths, group=group, eps=1e-8, out=out, symmetric=True,
                grids=[torch.from_numpy(x).cuda() for x in grids] if searched else None)
    torch.cuda.synchronize()
    assert np.allclose(out.cpu().numpy(), want, rtol=1e-6)
