"""The allocation-free loss entry point against the workspace one, through the C ABI.

``mr_loss_outlier_noalloc`` serves callers that cannot hand the library a
device buffer (an FFI host with no device allocator, or a pipeline that must
not call cudaMalloc because it can synchronize the device): its scratch is a
fixed array inside the library.  Two calls in a row, on different inputs,
must each give what ``mr_loss_outlier`` gives with a caller workspace: the
same threshold, the same loss to float64 summation order (the kernels are
the same, so in practice identical) and the same gradient.  This file is
collected last so that a run stopping at its first failure has already run
everything else.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _call_workspace(lib, pred, tgt, grad, loss, thr, ws, k, suppress, thr_in):
    n = pred.numel()
    st = lib.mr_loss_outlier(pred.data_ptr(), tgt.data_ptr(), n, k, int(suppress), float(n),
                             thr_in, grad.data_ptr(), loss.data_ptr(), thr.data_ptr(),
                             ws.data_ptr(), None)
    assert st == 0


def _call_noalloc(lib, pred, tgt, grad, loss, thr, k, suppress, thr_in):
    n = pred.numel()
    st = lib.mr_loss_outlier_noalloc(pred.data_ptr(), tgt.data_ptr(), n, k, int(suppress),
                                     float(n), thr_in, grad.data_ptr(), loss.data_ptr(),
                                     thr.data_ptr(), None)
    assert st == 0


def test_noalloc_loss_matches_workspace_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mround_b200._native import lib as load

    lib = load()
    assert lib.mr_loss_noalloc_scratch_bytes() >= lib.mr_loss_workspace_bytes()
    torch.cuda.synchronize()
    ws = torch.zeros(int(lib.mr_loss_workspace_bytes()), dtype=torch.uint8, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(7)
    # (shape, suppress, caller threshold): the selected threshold on two sizes,
    # plain MSE, an element count that is not a multiple of 4 (the kernels'
    # scalar tail), and a caller-given threshold that skips the selection
    cases = [((3, 129, 96), True, -1.0), ((8, 64, 576), True, -1.0), ((2, 16, 64), False, -1.0),
             ((3, 7, 13), False, -1.0), ((5, 11, 9), True, -1.0), ((4, 33, 64), True, 0.07)]
    for shape, suppress, thr_in in cases:
        pred = torch.randn(shape, device="cuda", generator=g)
        tgt = pred + 0.05 * torch.randn(shape, device="cuda", generator=g)
        n = pred.numel()
        k = max(1, int(n * 0.001))
        want = [torch.empty_like(pred), torch.zeros((), dtype=torch.float64, device="cuda"),
                torch.zeros((), device="cuda")]
        _call_workspace(lib, pred, tgt, *want, ws, k, suppress, thr_in)
        for _ in range(2):  # two calls in a row share (and overwrite) the static scratch
            got = [torch.full_like(pred, float("nan")),
                   torch.zeros((), dtype=torch.float64, device="cuda"),
                   torch.zeros((), device="cuda")]
            _call_noalloc(lib, pred, tgt, *got, k, suppress, thr_in)
            torch.cuda.synchronize()
            assert got[1].item() == pytest.approx(want[1].item(), rel=1e-12)
            assert torch.equal(got[0], want[0])
            if suppress and thr_in < 0:
                assert got[2].item() == want[2].item()


def test_noalloc_refuses_sizes_beyond_its_counters():
    from mround_b200._native import lib as load

    lib = load()
    st = lib.mr_loss_outlier_noalloc(None, None, 1 << 33, 1, 1, float(1 << 33), -1.0, None, None,
                                     None, None)
    assert st == -1
