"""The C-ABI library loads and exports every symbol the public header declares.

No compute call is made here, so these run without a GPU.
"""

from __future__ import annotations

import ctypes

import pytest

from mround_b200 import _native


def test_header_declares_the_kernels():
    names = _native.declared_symbols()
    for required in ("mr_fq_forward", "mr_ste_signsgd", "mr_pack_mlx", "mr_loss_outlier",
                     "mr_deltaloss", "mr_split_bf16"):
        assert required in names


def test_every_declared_symbol_is_exported():
    handle = ctypes.CDLL(str(_native.LIB_PATH))
    missing = [n for n in _native.declared_symbols() if not hasattr(handle, n)]
    assert not missing, f"not exported: {missing}"


def test_library_loads_and_reports_version():
    lib = _native.lib()
    assert lib.mr_version() == 100
    assert lib.mr_status_string(0).decode() == "ok"
    assert "misaligned" in lib.mr_status_string(-2).decode()
    assert lib.mr_loss_workspace_bytes() > 2048 * 4


def test_every_declared_symbol_has_a_signature():
    for name in _native.declared_symbols():
        assert name in _native._SIGNATURES, f"{name} has no ctypes signature"


def test_status_maps_to_exceptions():
    from mround_b200.exceptions import DeviceError, SchemeError

    _native.check(0, "ok")
    with pytest.raises(SchemeError):
        _native.check(-1, "x")
    with pytest.raises(DeviceError):
        _native.check(-3, "x")


def test_argument_errors_are_refused_before_any_launch():
    lib = _native.lib()
    # group 12 is not a device group: refused on the host side of the ABI
    st = lib.mr_fq_forward(None, None, None, None, 4, 48, 12, 2, 0, None, 1e-8, None, None, None,
                           None, None, None, None)
    assert st == -1
    st = lib.mr_pack_mlx(None, None, None, None, 4, 64, 64, 9, 0, None, 1e-8, None, None, None,
                         None, None)
    assert st == -1
    # a searched scale without the symmetric flag is refused before any launch
    buf = (ctypes.c_uint8 * 4096)()
    p = ctypes.addressof(buf)
    st = lib.mr_fq_forward(p, p, p, p, 4, 64, 64, 2, 0, p, 1e-8, None, None, None, None, None,
                           None, None)
    assert st == -1
    cands = (ctypes.c_float * 1)(2.0)
    st = lib.mr_scale_search(p, 4, 64, 12, 2, cands, 1, None, p, None)
    assert st == -1
    st = lib.mr_scale_search(p, 4, 64, 64, 2, cands, 0, None, p, None)
    assert st == -1


def test_selection_refuses_inputs_beyond_its_32bit_counters():
    """Every K4 entry point that selects a threshold refuses n >= 2^32 before
    touching a pointer (the histogram bins count in 32 bits); the pointers
    here are never dereferenced."""
    lib = _native.lib()
    fake = 1 << 12  # aligned, non-null stand-ins
    n = 1 << 33
    assert lib.mr_loss_outlier(fake, fake, n, 1, 1, float(n), -1.0, None, fake, None, fake,
                               None) == -1
    assert lib.mr_loss_hist_pass(fake, fake, n, 0, None, fake, None) == -1
    assert lib.mr_loss_outlier_noalloc(fake, fake, n, 1, 1, float(n), -1.0, None, fake, None,
                                       None) == -1


def test_gemm_entry_points_refuse_bad_precision_and_alignment():
    """The bf16 GEMM entry points take products 1-3 only (tf32 has its own
    entry points); float32 operands need leading dimensions in 16-byte units.
    Refused on the host, before any launch."""
    lib = _native.lib()
    p = 1 << 12
    assert lib.mr_gemm(p, p, 64, 1, p, p, 64, 1, p, 64, None, 0, 128, 128, 64, 4, None) == -1
    assert lib.mr_gemm(p, p, 64, 1, p, p, 64, 1, p, 64, None, 0, 128, 128, 64, 0, None) == -1
    assert lib.mr_gemm_tf32(p, 66, 1, p, 64, 1, p, 64, None, 0, 128, 128, 64, None) == -2
    assert lib.mr_gemm_tf32(None, 64, 1, p, 64, 1, p, 64, None, 0, 128, 128, 64, None) == -1


def test_gemm_tile_width_follows_the_persistent_schedule():
    """The tile-width query needs no GPU (148 SMs assumed without one): 224
    for tf32 products where it shortens the schedule, 256 otherwise, 128 for
    narrow outputs."""
    from mround_b200 import kernels

    def width(m, n, precision, b_kmajor=True, a_kmajor=True, batch=1, causal=0):
        return kernels.gemm_tile_n(m=m, n=n, k=3584, precision=precision, a_kmajor=a_kmajor,
                                   b_kmajor=b_kmajor, batch=batch, causal=causal)

    assert width(2048, 3584, 4) == 224           # 224 tiles of 256: 1.5 waves
    assert width(2048, 3584, 4, b_kmajor=False) == 224
    assert width(2048, 3584, 3) == 256           # the bf16 forms keep 256
    assert width(2048, 3584, 1) == 256
    assert width(2048, 3584, 4, batch=2) == 256
    assert width(16384, 37888, 4) == 256         # 128 whole waves already
    assert width(16384, 3584, 4) == 224          # 13 waves of 256 against 14 of 224
    assert width(3584, 3584, 1) == 256
    assert width(2048, 128, 4) == 128
    assert width(2048, 4608, 4) == 256           # a ragged 224 tile would lengthen it
    from mround_b200.exceptions import SchemeError

    with pytest.raises(SchemeError):
        width(0, 3584, 3)


def test_segmented_k2_refuses_bad_tables_before_any_launch():
    """mr_ste_signsgd_segments: 1 to 8 segments, one scheme per launch."""
    lib = _native.lib()
    buf = (ctypes.c_float * 4096)()
    p = ctypes.addressof(buf)
    assert p % 16 == 0

    def seg(init_scale=None, rows=4, cols=64):
        return _native.K2Segment(p, p, p, p, p, init_scale, rows, cols, 2, 0.01, 0.5, 1.5,
                                 p, p, None, None, None, None)

    table = (_native.K2Segment * 9)(*[seg() for _ in range(9)])
    assert lib.mr_ste_signsgd_segments(table, 0, 64, 1, 1e-8, None) == -1
    assert lib.mr_ste_signsgd_segments(table, 9, 64, 1, 1e-8, None) == -1
    # a searched segment beside an observed-range one: two schemes in one launch
    mixed = (_native.K2Segment * 2)(seg(), seg(init_scale=p))
    assert lib.mr_ste_signsgd_segments(mixed, 2, 64, 1, 1e-8, None) == -1
    # a width that is not whole groups
    ragged = (_native.K2Segment * 2)(seg(), seg(cols=96))
    assert lib.mr_ste_signsgd_segments(ragged, 2, 64, 1, 1e-8, None) == -1


def test_k2_segment_layout_matches_the_header(tmp_path):
    """The ctypes mirror of ``mr_k2_segment`` has the C compiler's offsets."""
    import shutil
    import subprocess

    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    fields = [name for name, _ in _native.K2Segment._fields_]
    body = "".join(f'  printf("{f} %zu\\n", offsetof(mr_k2_segment, {f}));\n' for f in fields)
    src = tmp_path / "layout.c"
    src.write_text("#include <stdio.h>\n#include <stddef.h>\n#include \"mround_b200.h\"\n"
                   "int main(void) {\n" + body +
                   '  printf("size %zu\\n", sizeof(mr_k2_segment));\n  return 0;\n}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(_native.HEADER.parent), str(src), "-o", str(exe)], check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    for f in fields:
        assert int(got[f]) == getattr(_native.K2Segment, f).offset, f
    assert int(got["size"]) == ctypes.sizeof(_native.K2Segment)


def test_gemm_tile_height_follows_the_schedule_model():
    """tf32 products take 256-row tiles where whole waves of them finish
    first and K covers their unoverlapped epilogue (the 7B backward at one
    GPU), 128 rows for small M or short K; the bf16 products keep 128."""
    from mround_b200 import kernels

    def tile(m, n, k, precision=4):
        return kernels.gemm_tile(m=m, n=n, k=k, precision=precision, a_kmajor=False,
                                 b_kmajor=False)

    assert tile(16384, 3584, 37888) == (256, 224)  # dX through gate_up, one GPU
    assert tile(2048, 3584, 37888) == (256, 224)   # the same at 2048 tokens (8 ranks)
    assert tile(37888, 3584, 16384) == (256, 256)  # dW through gate_up, one GPU
    assert tile(3584, 18944, 16384) == (256, 256)  # dW through down, one GPU
    assert tile(3584, 3584, 2048) == (128, 256)    # dW through o at 8 ranks: K too short
    assert tile(256, 3584, 4096) == (128, 224)     # one 256-row tile would leave SMs idle
    assert tile(16384, 3584, 37888, precision=3) == (128, 256)
    assert tile(2048, 128, 2048) == (128, 128)
