"""K3's tf32 mode (mr_gemm_tf32) and the tf32 operand producers, on the device.

A tf32 product multiplies the upper 19 bits of each float32 operand exactly
and accumulates in float32; with operands already rounded to tf32 (which
every producer here does) the kernel must agree with a float64 product of
those same values to float32 accumulation error.  Tested: every operand
majorness (MN-major float32 tiles take the 32-byte-atom swizzle), ragged
m/n/k edges, bias and accumulation, long K, and the rounding itself
(mr_round_tf32, the element-wise kernels' t32 outputs, K1/K2's wq_t32)
against a bit-level restatement: round to nearest, ties away from zero.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mround_b200 import kernels

    return kernels


def tf32_ref(x: torch.Tensor) -> torch.Tensor:
    """float32 -> tf32 value: add half of the dropped 13-bit field to the
    magnitude bits and clear it (round to nearest, ties away from zero)."""
    i = x.float().contiguous().view(torch.int32)
    return ((i + 0x1000) & ~0x1FFF).view(torch.float32)


def run_case(K, m, n, k, a_kmajor, b_kmajor, bias=False, accumulate=False, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = tf32_ref(torch.randn(m, k, device="cuda", generator=g))
    b = tf32_ref(torch.randn(n, k, device="cuda", generator=g) * 0.02)
    A = a if a_kmajor else a.t().contiguous()
    B = b if b_kmajor else b.t().contiguous()
    lda = k if a_kmajor else m
    ldb = k if b_kmajor else n
    c = torch.randn(m, n, device="cuda", generator=g) if accumulate else torch.zeros(m, n, device="cuda")
    c0 = c.clone()
    bvec = torch.randn(n, device="cuda", generator=g) if bias else None
    K.gemm_tf32(A, B, c, m=m, n=n, k=k, a_kmajor=a_kmajor, b_kmajor=b_kmajor, lda=lda, ldb=ldb,
                ldc=n, bias=bvec, accumulate=accumulate)
    torch.cuda.synchronize()
    ref = a.double() @ b.double().t()
    if bias:
        ref = ref + bvec.double()
    if accumulate:
        ref = ref + c0.double()
    err = (c.double() - ref).abs().max().item()
    scale = ref.abs().max().item()
    bound = 2e-5 * scale + 1e-6 * (k ** 0.5)
    assert err <= bound, f"max err {err:.3e} > {bound:.3e} (scale {scale:.3e})"
    from mround_b200._native import lib

    assert lib().mr_gemm_status(1) == 0


@pytest.mark.parametrize("a_kmajor", [True, False])
@pytest.mark.parametrize("b_kmajor", [True, False])
@pytest.mark.parametrize("n", [512, 96])
def test_layouts(K, a_kmajor, b_kmajor, n):
    run_case(K, 256, n, 320, a_kmajor, b_kmajor)


@pytest.mark.parametrize("m,n,k", [(200, 300, 104), (128, 960, 576), (37, 8, 16), (384, 256, 1000)])
def test_ragged_edges(K, m, n, k):
    # float32 leading dimensions must be multiples of 4
    if k % 4 == 0:
        run_case(K, m, n, k, True, True)
    if m % 4 == 0 and n % 4 == 0:
        run_case(K, m, n, k, False, False)
    if k % 4 == 0 and n % 4 == 0:
        run_case(K, m, n, k, True, False)


@pytest.mark.parametrize("a_kmajor", [True, False])
@pytest.mark.parametrize("b_kmajor", [True, False])
@pytest.mark.parametrize("m,n", [(2048, 3584), (2000, 3488)])
def test_224_wide_tiles(K, a_kmajor, b_kmajor, m, n):
    """224-wide output tiles (seven 128-byte chunks of an MN-major tf32 B
    tile): the 8-rank share of the 7B batch against a 3584-wide output, and
    a ragged last tile."""
    assert K.gemm_tile_n(m=m, n=n, k=160, precision=4, a_kmajor=a_kmajor,
                         b_kmajor=b_kmajor) == 224
    run_case(K, m, n, 160, a_kmajor, b_kmajor, bias=True)
    run_case(K, m, n, 64, a_kmajor, b_kmajor, accumulate=True, seed=1)


@pytest.mark.parametrize("a_kmajor", [True, False])
@pytest.mark.parametrize("b_kmajor", [True, False])
@pytest.mark.parametrize("m,n", [(1900, 4096), (16384, 3584)])
def test_256_row_tiles(K, a_kmajor, b_kmajor, m, n):
    """256-row tiles (two 128-row MMAs per K step sharing the B tile; chosen
    for K long enough to cover their unoverlapped epilogue): a last tile
    whose second half lies wholly past m (1900 = 7 x 256 + 108), and the 7B
    step's 16384 x 3584 shape at 224 columns."""
    for k in (6144, 6400):
        assert K.gemm_tile(m=m, n=n, k=k, precision=4, a_kmajor=a_kmajor,
                           b_kmajor=b_kmajor)[0] == 256
    run_case(K, m, n, 6144, a_kmajor, b_kmajor, bias=True)
    run_case(K, m, n, 6400, a_kmajor, b_kmajor, accumulate=True, seed=2)


def test_bias_and_accumulate(K):
    run_case(K, 256, 384, 192, True, True, bias=True)
    run_case(K, 256, 384, 192, False, False, accumulate=True)
    run_case(K, 128, 256, 64, True, False, bias=True, accumulate=True)


def test_long_k(K):
    run_case(K, 256, 256, 8192, False, False)


def test_unrounded_operands_lose_only_the_dropped_bits(K):
    """The tensor core reads the upper 19 bits: an unrounded operand gives the
    product of its truncation, never anything worse than tf32 resolution."""
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(128, 256, device="cuda", generator=g)
    b = torch.randn(128, 256, device="cuda", generator=g)
    c = torch.zeros(128, 128, device="cuda")
    K.gemm_tf32(a, b, c, m=128, n=128, k=256, a_kmajor=True, b_kmajor=True, lda=256, ldb=256,
                ldc=128)
    ref = a.double() @ b.double().t()
    assert (c.double() - ref).abs().max().item() <= 2.0 ** -9 * (a.abs() @ b.abs().t()).max().item()


def test_round_tf32_is_round_to_nearest_ties_away(K):
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(1 << 16, device="cuda", generator=g) * 10.0
    # exact ties and their neighbours, both signs, zeros and a subnormal
    base = torch.tensor([1.0, -1.0, 3.0, 0.0, -0.0, 1e-40], device="cuda")
    ties = (base.view(torch.int32) | 0x1000).view(torch.float32)
    below = (base.view(torch.int32) | 0x0FFF).view(torch.float32)
    x = torch.cat([x, base, ties, below, x[:7]])  # a length that is not a multiple of 4
    got = K.round_tf32(x)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), tf32_ref(x).view(torch.int32))


def test_elementwise_t32_outputs_round_the_same_values(K):
    """Each kernel's t32 output is the tf32 rounding of the value its float32
    or hi/lo output carries."""
    g = torch.Generator(device="cuda").manual_seed(2)
    t, h, inter = 64, 256, 384
    x = torch.randn(t, h, device="cuda", generator=g)
    w = (1.0 + 0.1 * torch.randn(h, device="cuda", generator=g)).to(torch.bfloat16)
    _, _, rstd, t32 = K.rmsnorm_split(x, w, 1e-6, t32=True)
    want = x * rstd[:, None] * w.float()
    assert (t32 - want).abs().max().item() <= 2.0 ** -10 * want.abs().max().item()
    assert torch.equal(t32.view(torch.int32) & 0x1FFF, torch.zeros_like(t32.view(torch.int32)))
    dy = torch.randn(t, h, device="cuda", generator=g)
    out = torch.empty(t, h, device="cuda")
    hi, lo, t32 = K.rmsnorm_bwd_split(dy, x, w, rstd, None, split=False, t32=True, out=out)
    assert hi is None and lo is None
    assert torch.equal(t32.view(torch.int32), tf32_ref(out).view(torch.int32))
    gu = torch.randn(t, 2 * inter, device="cuda", generator=g)
    dact = torch.randn(t, inter, device="cuda", generator=g)
    hi, lo, t32 = K.swiglu_bwd_split(dact, gu, t, inter, split=True, t32=True)
    full = hi.float() + lo.float()
    assert (t32 - full).abs().max().item() <= 2.0 ** -10 * full.abs().max().item()
    assert torch.equal(t32.view(torch.int32) & 0x1FFF, torch.zeros_like(t32.view(torch.int32)))


def test_fake_quant_t32_is_the_rounded_weight(K):
    """K1's and K2's wq_t32 are the tf32 rounding of the float32 fake-quantized
    weight K1 writes as wq_f32."""
    g = torch.Generator(device="cuda").manual_seed(4)
    rows, cols, group = 64, 256, 64
    w = (torch.randn(rows, cols, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    v = (torch.rand(rows, cols, device="cuda", generator=g) - 0.5) * 0.6
    a = 0.7 + 0.3 * torch.rand(rows, cols // group, device="cuda", generator=g)
    b = 0.7 + 0.3 * torch.rand(rows, cols // group, device="cuda", generator=g)
    f32 = torch.empty(rows, cols, device="cuda")
    t32 = torch.empty(rows, cols, device="cuda")
    K.fq_forward(w, v, a, b, bits=2, group=group, eps=1e-8, wq_f32=f32, wq_t32=t32)
    assert torch.equal(t32.view(torch.int32), tf32_ref(f32).view(torch.int32))
    # K2 with update: the next operand equals K1 on the updated parameters
    gq = torch.randn(rows, cols, device="cuda", generator=g) * 1e-3
    hi = torch.empty(rows, cols, dtype=torch.bfloat16, device="cuda")
    lo = torch.empty_like(hi)
    t32b = torch.empty(rows, cols, device="cuda")
    K.ste_signsgd(gq, w, v, a, b, bits=2, group=group, eps=1e-8, lr=0.01, lo=0.1, hi=1.0,
                  update=True, wq_hi=hi, wq_lo=lo, wq_t32=t32b)
    K.fq_forward(w, v, a, b, bits=2, group=group, eps=1e-8, wq_f32=f32)
    torch.cuda.synchronize()
    assert torch.equal(t32b.view(torch.int32), tf32_ref(f32).view(torch.int32))
