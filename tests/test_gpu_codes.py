"""K2's codes output and the operand rebuild (mr_ste_signsgd_codes,
mr_dequant_split), through the C ABI.

The row-sharded update exchanges codes and per-group scale / zero point
instead of operands; every rank rebuilds the operands from them.  Bar: the
rebuilt bf16 hi/lo and tf32 operands, and the updated V/alpha/beta, bit for
bit those of mr_ste_signsgd with the operand outputs; the codes and scales
bit for bit the float32 oracle's (mround/core/quantizer.py:317-347 of the
reference) after the oracle's signed step.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import packing as o_pack
from oracle import quant_fp32 as o_q
from oracle import scale_search as o_s

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mround_b200 import kernels

    return kernels


def bf16_round(x):
    return o_pack.bf16_to_f32(o_pack.bf16_bits(np.asarray(x, np.float32)))


def make_case(seed, rows, cols, group, bounds):
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32)
    hot = rng.random(size=(rows, cols)) < 0.001
    w[hot] *= 20.0
    w = bf16_round(w)
    ng = cols // group
    v = rng.uniform(-0.5, 0.5, size=(rows, cols)).astype(np.float32)
    a = rng.uniform(*bounds, size=(rows, ng)).astype(np.float32)
    b = rng.uniform(*bounds, size=(rows, ng)).astype(np.float32)
    gq = rng.normal(0.0, 1e-3, size=(rows, cols)).astype(np.float32)
    return w, v, a, b, gq


def dev(w, *rest):
    return [torch.from_numpy(w).cuda().to(torch.bfloat16)] + [
        torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in rest]


MODES = ["asym", "sym", "searched"]


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("bits,group", [(2, 64), (3, 32), (4, 128), (8, 64), (4, 16)])
def test_codes_then_dequant_equals_operand_update(K, mode, bits, group):
    rows, cols = 48, 1024
    symmetric, searched = mode != "asym", mode == "searched"
    bounds = (0.5, 1.5) if searched else (0.5, 1.0)
    lo_b, hi_b = (0.5, 1.5) if searched else (0.1, 1.0)
    w, v, a, b, gq = make_case(bits * 31 + group + len(mode), rows, cols, group, bounds)
    init = o_s.search_scales_f32(w, bits, group).reshape(rows, -1) if searched else None
    dinit = None if init is None else torch.from_numpy(init).cuda()
    lr = o_q.lr_at(0.005, 200, 17)
    g = torch.from_numpy(gq).cuda()
    kw = dict(bits=bits, group=group, eps=1e-8, lr=lr, lo=lo_b, hi=hi_b, symmetric=symmetric,
              init_scale=dinit)

    # the operand form
    dw, dv, da, db = dev(w, v, a, b)
    hi, lo = torch.empty_like(dw), torch.empty_like(dw)
    t32 = torch.empty(rows, cols, dtype=torch.float32, device="cuda")
    K.ste_signsgd(g, dw, dv, da, db, update=True, wq_hi=hi, wq_lo=lo, wq_t32=t32, **kw)

    # the codes form, then the rebuild
    cw, cv, ca, cb = dev(w, v, a, b)
    codes = torch.empty(rows, cols, dtype=torch.uint8, device="cuda")
    qscale = torch.empty(rows, cols // group, dtype=torch.float32, device="cuda")
    qzp = None if symmetric else torch.empty_like(qscale)
    K.ste_signsgd_codes(g, cw, cv, ca, cb, codes=codes, qscale=qscale, qzp=qzp, **kw)
    hi2, lo2 = torch.empty_like(hi), torch.empty_like(lo)
    t32b = torch.empty_like(t32)
    K.dequant_split(codes, qscale, qzp, group=group, symmetric=symmetric, wq_hi=hi2, wq_lo=lo2,
                    wq_t32=t32b)
    torch.cuda.synchronize()

    for x, y in ((dv, cv), (da, ca), (db, cb)):
        assert torch.equal(x, y)
    assert torch.equal(hi.view(torch.int16), hi2.view(torch.int16))
    assert torch.equal(lo.view(torch.int16), lo2.view(torch.int16))
    assert torch.equal(t32.view(torch.int32), t32b.view(torch.int32))

    # codes and scales against the oracle after its own signed step
    gv, ga, gb = (torch.empty_like(dv), torch.empty_like(da), torch.empty_like(db))
    ow, ov, oa, ob = dev(w, v, a, b)
    K.ste_signsgd(g, ow, ov, oa, ob, update=False, gv=gv, galpha=ga, gbeta=gb, **kw)
    torch.cuda.synchronize()
    v_o, a_o, b_o = o_q.signsgd_step(v, a, b, gv.cpu().numpy(), ga.cpu().numpy(),
                                     gb.cpu().numpy(), lr, lo_b, hi_b)
    _, codes_o, scale_o, zp_o = o_q.fake_quantize(w, v_o, a_o, b_o, bits, group,
                                                  symmetric=symmetric, init_scale=init)
    got = codes.cpu().numpy()
    got = got.view(np.int8).astype(np.int64) if symmetric else got.astype(np.int64)
    assert np.array_equal(got, codes_o.astype(np.int64))
    assert np.array_equal(qscale.cpu().numpy().ravel(), np.asarray(scale_o, np.float32).ravel())
    if not symmetric:
        assert np.array_equal(qzp.cpu().numpy().ravel(), np.asarray(zp_o, np.float32).ravel())


def test_dequant_refuses_a_width_that_is_not_whole_groups(K):
    from mround_b200.exceptions import SchemeError

    codes = torch.zeros(4, 100, dtype=torch.uint8, device="cuda")
    qscale = torch.ones(4, 1, dtype=torch.float32, device="cuda")
    with pytest.raises(SchemeError):
        K.dequant_split(codes, qscale, None, group=64, symmetric=False,
                        wq_hi=torch.empty(4, 100, dtype=torch.bfloat16, device="cuda"))


@pytest.mark.parametrize("mode", MODES)
def test_segmented_launch_equals_one_launch_per_matrix(K, mode):
    """One mr_ste_signsgd_segments launch over a block's worth of matrices
    (different shapes, widths, rates; operand and codes outputs mixed) gives
    every output bit for bit as one call per matrix."""
    group = 64
    symmetric, searched = mode != "asym", mode == "searched"
    bounds = (0.5, 1.5) if searched else (0.5, 1.0)
    lo_b, hi_b = (0.5, 1.5) if searched else (0.1, 1.0)
    # (rows, cols, bits, lr, output): a 0.5B block's shapes, scaled down in rows
    specs = [(112, 896, 2, 0.004, "operands"), (16, 896, 3, 0.005, "codes"),
             (16, 896, 2, 0.006, "operands"), (112, 896, 4, 0.004, "codes"),
             (608, 896, 2, 0.003, "operands"), (608, 896, 8, 0.002, "operands"),
             (112, 4864, 2, 0.001, "codes")]
    single, grouped = [], []
    for i, (rows, cols, bits, lr, form) in enumerate(specs):
        w, v, a, b, gq = make_case(100 + i + len(mode), rows, cols, group, bounds)
        init = o_s.search_scales_f32(w, bits, group).reshape(rows, -1) if searched else None
        dinit = None if init is None else torch.from_numpy(init).cuda()
        g = torch.from_numpy(gq).cuda()
        for store in (single, grouped):
            dw, dv, da, db = dev(w, v, a, b)
            out = {}
            if form == "operands":
                out = {"wq_hi": torch.empty_like(dw), "wq_lo": torch.empty_like(dw),
                       "wq_t32": torch.empty(rows, cols, device="cuda")}
            else:
                ng = rows * cols // group
                out = {"codes": torch.empty(rows, cols, dtype=torch.uint8, device="cuda"),
                       "qscale": torch.empty(ng, device="cuda"),
                       "qzp": None if symmetric else torch.empty(ng, device="cuda")}
            store.append(dict(gq=g, w=dw, v=dv, alpha=da, beta=db, bits=bits, lr=lr, lo=lo_b,
                              hi=hi_b, init_scale=dinit, form=form, **out))
    for sg in single:
        kw = dict(bits=sg["bits"], group=group, eps=1e-8, lr=sg["lr"], lo=lo_b, hi=hi_b,
                  symmetric=symmetric, init_scale=sg["init_scale"])
        if sg["form"] == "operands":
            K.ste_signsgd(sg["gq"], sg["w"], sg["v"], sg["alpha"], sg["beta"], update=True,
                          wq_hi=sg["wq_hi"], wq_lo=sg["wq_lo"], wq_t32=sg["wq_t32"], **kw)
        else:
            K.ste_signsgd_codes(sg["gq"], sg["w"], sg["v"], sg["alpha"], sg["beta"],
                                codes=sg["codes"], qscale=sg["qscale"], qzp=sg["qzp"], **kw)
    K.ste_signsgd_segments(
        [{k: x for k, x in sg.items() if k != "form"} for sg in grouped], group=group, eps=1e-8,
        symmetric=symmetric)
    torch.cuda.synchronize()
    for a, b in zip(single, grouped):
        for key in ("v", "alpha", "beta", "wq_hi", "wq_lo", "wq_t32", "codes", "qscale", "qzp"):
            x, y = a.get(key), b.get(key)
            if x is None:
                assert y is None
                continue
            if x.dtype == torch.bfloat16:
                x, y = x.view(torch.int16), y.view(torch.int16)
            elif x.dtype == torch.float32:
                x, y = x.view(torch.int32), y.view(torch.int32)
            assert torch.equal(x, y), key
