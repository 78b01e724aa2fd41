"""MLX uint32 code packing and the affine scale/bias form. TEST ORACLE ONLY.

Layout (reference ``mround/formats/packing.py:119-163``, oracle
``mround/reference/packing.py:73-122``): codes pack along the input axis with
element 0 in the least significant bits.  Widths dividing 32 (2, 4, 8) put
``32 // b`` codes in each word at offsets ``j * b``; the others (3, 5, 6, 7)
form a little-endian bitstream, element ``i`` at absolute bits
``[i*b, (i+1)*b)``, so 32 codes fill exactly ``b`` words.

This packer is written independently of the reference's: it lays the codes
out as a bit matrix and folds each run of 32 bits into a word, which covers
both layouts with one rule (the even layout is the bitstream layout whenever
``b`` divides 32).

Affine form (reference ``mround/formats/mlx_export.py:159-195``):
``scales = bf16(scale)``, ``biases = bf16(-scales * bf16(zp))`` with the
product taken from the already rounded scale.
"""

from __future__ import annotations

import numpy as np

__all__ = ["bf16_bits", "bf16_to_f32", "pack_codes", "packed_width", "to_affine", "unpack_codes"]


def packed_width(cols: int, bits: int) -> int:
    """Words per row (reference ``packing.py:84-116``)."""
    if 32 % bits == 0:
        per = 32 // bits
        if cols % per:
            raise ValueError(f"cols={cols} is not a multiple of {per} at {bits} bits")
        return cols // per
    if cols % 32:
        raise ValueError(f"cols={cols} is not a multiple of 32 at {bits} bits")
    return cols // 32 * bits


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """(rows, cols) integer codes in [0, 2**bits) -> (rows, words) uint32."""
    codes = np.asarray(codes)
    if codes.size and (codes.min() < 0 or codes.max() > (1 << bits) - 1):
        raise ValueError(f"codes must lie in [0, {(1 << bits) - 1}] at {bits} bits")
    rows, cols = codes.shape
    words = packed_width(cols, bits)
    c = codes.astype(np.uint64)
    # bit matrix: (rows, cols, bits), least significant bit first
    bitm = ((c[:, :, None] >> np.arange(bits, dtype=np.uint64)) & np.uint64(1)).astype(np.uint64)
    stream = bitm.reshape(rows, cols * bits)[:, : words * 32].reshape(rows, words, 32)
    out = (stream << np.arange(32, dtype=np.uint64)).sum(axis=-1)
    return out.astype(np.uint32)


def unpack_codes(packed: np.ndarray, cols: int, bits: int) -> np.ndarray:
    """Inverse of :func:`pack_codes`."""
    packed = np.asarray(packed, dtype=np.uint32)
    rows, words = packed.shape
    if words != packed_width(cols, bits):
        raise ValueError("word count does not match cols and bits")
    stream = ((packed.astype(np.uint64)[:, :, None] >> np.arange(32, dtype=np.uint64)) & np.uint64(1))
    stream = stream.reshape(rows, words * 32)[:, : cols * bits].reshape(rows, cols, bits)
    return (stream << np.arange(bits, dtype=np.uint64)).sum(axis=-1).astype(np.int64)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16, nearest-even; returns the uint16 patterns."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> np.uint64(16)) & np.uint64(1)) + np.uint64(0x7FFF)
    return (((u + rounding) >> np.uint64(16)) & np.uint64(0xFFFF)).astype(np.uint16)


def bf16_to_f32(bits16: np.ndarray) -> np.ndarray:
    """Widen bfloat16 patterns to float32 (exact)."""
    return (np.asarray(bits16, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def to_affine(scale: np.ndarray, zp, bits: int | None = None) -> tuple[np.ndarray, np.ndarray]:
    """MLX affine parameters as bf16 bit patterns ``(scales, biases)``.

    ``zp`` None means a symmetric scheme: the fixed offset ``2**(bits-1)``
    (reference ``mround/formats/mlx_export.py:186-194``).
    """
    s_bits = bf16_bits(scale)
    s = bf16_to_f32(s_bits)
    if zp is None:
        z = np.float32(2 ** (bits - 1))
    else:
        z = bf16_to_f32(bf16_bits(zp))
    prod = ((-s) * z).astype(np.float32)  # exact: two 8-bit significands
    return s_bits, bf16_bits(prod)
