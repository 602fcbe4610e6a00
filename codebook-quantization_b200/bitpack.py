"""Fixed-width index bitstream (the ``indices`` key of a ``direct_codebook`` tensor).

Layout (reference ``src/bitpack.py:32-94``): element ``e`` of the flattened
row-major ``[M, K]`` index matrix occupies bits ``[e*b, (e+1)*b)`` of a byte
stream whose bit 0 is the least-significant bit of byte 0 (LSB-first,
little-endian).  The stream is exactly ``ceil(n*b/8)`` bytes long on disk.
The reference's 4-, 8- and 16-bit fast paths are the same layout (4-bit puts
the even element in the low nibble; 16-bit is little-endian ``uint16``), so one
implementation covers every width 1..16.

These CPU routines write the format for tests and for host-side tooling; the
device path reads it with ``cbq_linear_fixed_*`` (``csrc/cbq_fixed.cu``) and
large streams are written on the GPU by ``cbq_pack_fixed``.
"""
from __future__ import annotations

import numpy as np

__all__ = ["packed_size", "pack_any_bits", "unpack_any_bits"]


def packed_size(n: int, bits: int) -> int:
    """Bytes of an ``n``-element, ``bits``-wide stream (``src/bitpack.py:184``)."""
    return (int(n) * int(bits) + 7) // 8


def _check_bits(bits: int) -> int:
    bits = int(bits)
    if not 1 <= bits <= 16:
        raise ValueError(f"bits must be in [1, 16], got {bits}")
    return bits


def pack_any_bits(indices, bits: int, chunk: int = 1 << 22) -> np.ndarray:
    """Pack ``indices`` (any integer array, flattened) into an LSB-first stream.

    Values are truncated to their low ``bits`` bits, like the reference's
    shifts into a fixed-width field.  Works on 64-bit words: element ``e``'s
    field starts at bit ``e*b``; its low part is OR-ed into word ``e*b >> 6``
    and, when it straddles, its high part into the next word.  Contributions to
    a word come from consecutive elements, so a segmented OR
    (``bitwise_or.reduceat``) assembles every word without a per-bit loop.
    """
    bits = _check_bits(bits)
    idx = np.asarray(indices).reshape(-1)
    n = idx.size
    nbytes = packed_size(n, bits)
    nwords = (n * bits + 63) // 64
    words = np.zeros(nwords + 1, dtype=np.uint64)
    mask = np.uint64((1 << bits) - 1)
    for s in range(0, n, chunk):
        v = idx[s:s + chunk].astype(np.uint64) & mask
        e = np.arange(s, s + v.size, dtype=np.int64)
        bit = e * bits
        w = bit >> 6
        sh = (bit & 63).astype(np.uint64)
        lo = v << sh                                 # bits beyond 63 drop out
        hi_shift = np.uint64(64) - sh
        spill = (sh + np.uint64(bits)) > np.uint64(64)
        # hi part only where the field crosses into the next word
        hi = np.where(spill, v >> np.where(spill, hi_shift, np.uint64(0)), np.uint64(0))
        # segmented OR over runs of equal word index (w is non-decreasing)
        starts = np.flatnonzero(np.r_[True, w[1:] != w[:-1]])
        words[w[starts]] |= np.bitwise_or.reduceat(lo, starts)
        hs = np.flatnonzero(spill)
        if hs.size:
            words[w[hs] + 1] |= hi[hs]
    out = words.view(np.uint8) if np.little_endian else words.byteswap().view(np.uint8)
    return out[:nbytes].copy()


def unpack_any_bits(packed, bits: int, original_len: int, first: int = 0) -> np.ndarray:
    """Inverse of :func:`pack_any_bits`: ``original_len`` indices as ``uint16``.

    ``first`` selects the starting element, which is the seek the reference's
    ``FastIndexManager`` performs (``src/fast_index_manager.py:115-137``).
    Bytes beyond the end of ``packed`` read as zero.
    """
    bits = _check_bits(bits)
    p = np.asarray(packed, dtype=np.uint8).reshape(-1)
    n = int(original_len)
    if n == 0:
        return np.zeros(0, dtype=np.uint16)
    e = np.arange(first, first + n, dtype=np.int64)
    bit = e * bits
    byte = bit >> 3
    pad = np.zeros(int(byte[-1]) + 4 - p.size, dtype=np.uint8) if int(byte[-1]) + 4 > p.size else None
    if pad is not None:
        p = np.concatenate([p, pad])
    win = (p[byte].astype(np.uint32)
           | (p[byte + 1].astype(np.uint32) << 8)
           | (p[byte + 2].astype(np.uint32) << 16)
           | (p[byte + 3].astype(np.uint32) << 24))
    return ((win >> (bit & 7).astype(np.uint32)) & np.uint32((1 << bits) - 1)).astype(np.uint16)
