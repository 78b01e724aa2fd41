"""The tuning path refuses to run without its CUDA library or a CUDA device
(no CPU fallback), checked on a host without a GPU."""

from __future__ import annotations

import pytest
import torch

from mround_b200 import _native, kernels
from mround_b200.exceptions import NativeLibraryError, PlatformError


def test_host_tensors_are_refused_not_computed():
    w = torch.zeros(4, 64, dtype=torch.bfloat16)
    v = torch.zeros(4, 64)
    a = torch.ones(4, 1)
    b = torch.ones(4, 1)
    with pytest.raises(PlatformError, match="CUDA tensor"):
        kernels.fq_forward(w, v, a, b, bits=2, group=64, eps=1e-8,
                           wq_f32=torch.empty(4, 64))
    with pytest.raises(PlatformError, match="CUDA tensor"):
        hi = torch.zeros(128, 64, dtype=torch.bfloat16)
        kernels.gemm(hi, None, hi, None, torch.empty(128, 128), m=128, n=128, k=64,
                     a_kmajor=True, b_kmajor=True, lda=64, ldb=64, ldc=128, precision=1)


def test_a_missing_library_is_an_error(tmp_path, monkeypatch):
    monkeypatch.setattr(_native, "LIB_PATH", tmp_path / "libmround_b200.so")
    _native.lib.cache_clear()
    try:
        with pytest.raises(NativeLibraryError, match="no CPU fallback"):
            _native.lib()
    finally:
        monkeypatch.undo()
        _native.lib.cache_clear()


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the refusal on a host without a GPU")
def test_quantize_without_a_device_is_refused(tmp_path):
    from mround_b200.api import quantize
    from mround_b200.pipeline.dist import DistContext

    with pytest.raises(PlatformError, match="CUDA device"):
        quantize("synthetic:tiny-qwen2", output_dir=tmp_path, bits=2, group_size=32,
                 symmetry="asym", progress=None, dist=DistContext())
