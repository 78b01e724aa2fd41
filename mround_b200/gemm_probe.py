"""Run one GEMM shape of the 7B tuning step three times (the K3 ncu driver).

Usage: python -m mround_b200.gemm_probe <shape> <tokens>

``shape`` is one of the block's weight GEMMs at ``tokens`` rows of activation
(16384 = the 8 x 2048 batch on one GPU, 2048 = one sequence per GPU at eight):
gate_up (forward), dX_gu (input gradient through gate_up), dW_gu (its weight
gradient), o (forward).  Operands are random float32 split into bf16 hi/lo;
every launch is precision 3, as in the tuning step.
"""

from __future__ import annotations

import sys

import torch

from mround_b200 import kernels


def main(argv: list[str] | None = None) -> None:
    argv = sys.argv[1:] if argv is None else argv
    name, tokens = argv[0], int(argv[1])
    shapes = {"gate_up": (tokens, 37888, 3584, True, True),
              "dX_gu": (tokens, 3584, 37888, True, False),
              "dW_gu": (37888, 3584, tokens, False, False),
              "o": (tokens, 3584, 3584, True, True)}
    m, n, k, ak, bk = shapes[name]
    a_rows, a_cols = (m, k) if ak else (k, m)
    b_rows, b_cols = (n, k) if bk else (k, n)
    a = torch.randn(a_rows, a_cols, device="cuda")
    b = torch.randn(b_rows, b_cols, device="cuda")
    ah, al = kernels.split_bf16(a)
    bh, bl = kernels.split_bf16(b)
    del a, b
    c = torch.empty(m, n, device="cuda")
    for _ in range(3):
        kernels.gemm(ah, al, bh, bl, c, m=m, n=n, k=k, a_kmajor=ak, b_kmajor=bk, lda=a_cols,
                     ldb=b_cols, ldc=n, precision=3)
    torch.cuda.synchronize()
    print("ok", name, tokens)


if __name__ == "__main__":
    main()
