"""Canonical-Huffman index stream (the ``--entropy-code`` variant of a tensor).

Format (reference ``src/huffman_codebook.py:126-226``):

* ``huff_lengths`` ``uint8[A]``: code length of each symbol ``0..A-1`` where
  ``A = max(index) + 1``; 0 marks an unused symbol.  Lengths come from a
  Huffman tree built with a min-heap over ``(frequency, node id)`` pairs,
  leaves numbered by symbol and internal nodes numbered from ``A`` upwards in
  creation order, each length capped at 32 (``src/huffman_codebook.py:42-86``).
  The tie-break is part of the format: a different rule gives different
  lengths, so it is kept exactly.
* canonical codes (RFC 1951 section 3.2.2): symbols sorted by (length, symbol)
  receive consecutive code values, the first code of each length being
  ``(first code of the previous length + its count) << 1``.
* ``huff_stream`` ``uint8``: codes written MSB-first, rows concatenated with no
  alignment, followed by 4 zero bytes.
* ``huff_row_bit_starts`` ``int64[M]``: bit offset of each row's first symbol.
* ``huff_lut_sym`` / ``huff_lut_len`` ``int32[4096]``: for each 12-bit prefix,
  the symbol and length of the code of length <= 12 that it starts with, or
  ``-1`` / ``0`` (``src/huffman_codebook.py:394-423``).
* ``huff_sl_first_code`` ``int64[max+2]``, ``huff_sl_base_offset``
  ``int32[max+2]``, ``huff_sl_sym`` ``int32[>=1]``: per-length first code
  (``-1`` = none), offsets into the long-code symbol list and the list itself,
  for codes longer than 12 bits (``src/huffman_codebook.py:353-391``).

The CUDA path (``csrc/cbq_huff.cu``) does not use the 12-bit tables directly;
it derives its own decode tables from ``huff_lengths`` at load time
(:func:`decode_tables`), which tests check against the stored ones.
"""
from __future__ import annotations

import heapq
from typing import Dict, Tuple

import numpy as np

GPU_LUT_BITS = 12
GPU_LUT_SIZE = 1 << GPU_LUT_BITS
MAX_CODE_LEN = 32

__all__ = [
    "code_lengths", "canonical_codes", "huffman_encode_indices", "build_gpu_lut",
    "build_slow_path_tables", "decode_tables", "GPU_LUT_BITS", "MAX_CODE_LEN",
]


def code_lengths(freq) -> np.ndarray:
    """Huffman code length per symbol from a frequency array (0 = unused).

    Follows ``src/huffman_codebook.py:42-86``: one active symbol gets length 1;
    otherwise repeatedly merge the two smallest ``(freq, id)`` entries of a
    min-heap into a new node ``id = A, A+1, ...``.  Depths are then computed
    top-down from the root over the recorded merges and capped at 32.
    """
    freq = np.asarray(freq, dtype=np.int64).reshape(-1)
    a = freq.size
    lengths = np.zeros(a, dtype=np.uint8)
    active = [(int(f), i) for i, f in enumerate(freq.tolist()) if f > 0]
    if not active:
        return lengths
    if len(active) == 1:
        lengths[active[0][1]] = 1
        return lengths
    heapq.heapify(active)
    children = []                      # children[j] = (left, right) of node a + j
    nid = a
    while len(active) > 1:
        f1, x = heapq.heappop(active)
        f2, y = heapq.heappop(active)
        children.append((x, y))
        heapq.heappush(active, (f1 + f2, nid))
        nid += 1
    depth = np.zeros(nid, dtype=np.int64)
    for j in range(len(children) - 1, -1, -1):     # root is the last node made
        d = depth[a + j] + 1
        x, y = children[j]
        depth[x] = d
        depth[y] = d
    used = freq > 0
    lengths[used] = np.minimum(depth[:a][used], MAX_CODE_LEN).astype(np.uint8)
    return lengths


def canonical_codes(lengths) -> Tuple[np.ndarray, np.ndarray]:
    """RFC 1951 canonical code values: returns ``(code uint64[A], length uint8[A])``.

    Symbols with length 0 get code 0.  Same assignment as
    ``src/huffman_codebook.py:89-119``.
    """
    lengths = np.asarray(lengths, dtype=np.uint8).reshape(-1)
    codes = np.zeros(lengths.size, dtype=np.uint64)
    if lengths.size == 0 or int(lengths.max()) == 0:
        return codes, lengths
    max_len = int(lengths.max())
    count = np.bincount(lengths, minlength=max_len + 1).astype(np.int64)
    count[0] = 0
    first = np.zeros(max_len + 2, dtype=np.int64)
    c = 0
    for L in range(1, max_len + 1):
        c = (c + int(count[L - 1])) << 1
        first[L] = c
    # rank of each symbol among the symbols of its length, in symbol order
    order = np.lexsort((np.arange(lengths.size), lengths))
    ls = lengths[order]
    used = ls > 0
    order, ls = order[used], ls[used].astype(np.int64)
    run_start = np.searchsorted(ls, ls, side="left")
    rank = np.arange(ls.size) - run_start
    codes[order] = (first[ls] + rank).astype(np.uint64)
    return codes, lengths


def _encode_stream(idx: np.ndarray, sym_code: np.ndarray, sym_len: np.ndarray):
    """Concatenate codes MSB-first; returns (stream bytes incl. 4 pad, bit starts)."""
    n = idx.size
    lens = sym_len[idx].astype(np.int64)
    starts = np.zeros(n, dtype=np.int64)
    if n > 1:
        np.cumsum(lens[:-1], out=starts[1:])
    total = int(starts[-1] + lens[-1]) if n else 0
    nbytes = (total + 7) // 8
    nwords = (total + 63) // 64
    words = np.zeros(nwords + 1, dtype=np.uint64)
    if n:
        code = sym_code[idx].astype(np.uint64)
        w = starts >> 6
        o = starts & 63
        end = o + lens                               # one past the last bit, within word w
        fits = end <= 64
        # big-endian bit numbering inside a word: bit position o maps to 1 << (63 - o)
        sh_fit = np.where(fits, 64 - end, 0).astype(np.uint64)
        sh_spl = np.where(fits, 0, end - 64).astype(np.uint64)
        first_part = np.where(fits, code << sh_fit, code >> sh_spl)
        seg = np.flatnonzero(np.r_[True, w[1:] != w[:-1]])
        words[w[seg]] |= np.bitwise_or.reduceat(first_part, seg)
        spl = np.flatnonzero(~fits)
        if spl.size:
            rest = (end[spl] - 64).astype(np.uint64)         # bits that fall into word w+1
            words[w[spl] + 1] |= code[spl] << (np.uint64(64) - rest)
    stream = words.astype(">u8").view(np.uint8)[:nbytes]
    return np.concatenate([stream, np.zeros(4, dtype=np.uint8)]), starts


def huffman_encode_indices(indices, shape: tuple = None) -> Dict[str, np.ndarray]:
    """Huffman-encode a flat index array (``src/huffman_codebook.py:126-226``).

    Returns ``huff_lengths``, ``huff_stream`` and ``huff_n``; when ``shape`` is
    ``(M, K)`` it adds ``huff_row_bit_starts`` and the 12-bit LUT / slow-path
    tables, exactly as the reference stores them in the ``.npz``.
    """
    idx = np.asarray(indices).astype(np.uint16).reshape(-1)
    n = idx.size
    a = int(idx.max()) + 1 if n else 1
    freq = np.bincount(idx, minlength=a).astype(np.int64)
    lengths = code_lengths(freq)
    codes, _ = canonical_codes(lengths)
    stream, starts = _encode_stream(idx, codes, lengths)
    out = {
        "huff_lengths": lengths,
        "huff_stream": stream,
        "huff_n": np.array([n], dtype=np.int64),
    }
    if shape is not None and len(shape) == 2:
        m, k = int(shape[0]), int(shape[1])
        if n > 0 and m * k == n:
            out["huff_row_bit_starts"] = starts[::k].astype(np.int64)
        else:
            out["huff_row_bit_starts"] = np.zeros(max(m, 1), dtype=np.int64)
        out["huff_lut_sym"], out["huff_lut_len"] = build_gpu_lut(lengths)
        (out["huff_sl_first_code"], out["huff_sl_base_offset"],
         out["huff_sl_sym"]) = build_slow_path_tables(lengths)
    return out


def build_gpu_lut(lengths) -> Tuple[np.ndarray, np.ndarray]:
    """12-bit prefix table ``(lut_sym int32[4096], lut_len int32[4096])``.

    Every prefix that starts with a code of length ``L <= 12`` maps to that
    code's symbol and length; other prefixes hold ``-1`` / ``0``
    (``src/huffman_codebook.py:394-423``).
    """
    lut_sym = np.full(GPU_LUT_SIZE, -1, dtype=np.int32)
    lut_len = np.zeros(GPU_LUT_SIZE, dtype=np.int32)
    codes, lengths = canonical_codes(lengths)
    for s in np.flatnonzero((lengths > 0) & (lengths <= GPU_LUT_BITS)):
        L = int(lengths[s])
        base = int(codes[s]) << (GPU_LUT_BITS - L)
        span = 1 << (GPU_LUT_BITS - L)
        lut_sym[base:base + span] = s
        lut_len[base:base + span] = L
    return lut_sym, lut_len


def build_slow_path_tables(lengths):
    """Long-code tables ``(sl_first_code int64, sl_base_offset int32, sl_sym int32)``.

    Sized ``max_len + 2`` (``max_len`` = 12 when no code exists); lengths
    ``13..max_len`` get their first code and the offset of their symbols in
    ``sl_sym``, which lists long-code symbols in (length, code) order;
    ``sl_base_offset[max_len+1]`` is the total (``src/huffman_codebook.py:353-391``).
    """
    codes, lengths = canonical_codes(lengths)
    max_len = int(lengths.max()) if lengths.size and int(lengths.max()) > 0 else GPU_LUT_BITS
    first = np.full(max_len + 2, -1, dtype=np.int64)
    base = np.zeros(max_len + 2, dtype=np.int32)
    syms = []
    off = 0
    for L in range(GPU_LUT_BITS + 1, max_len + 1):
        base[L] = off
        s = np.flatnonzero(lengths == L)
        if s.size:
            s = s[np.argsort(codes[s], kind="stable")]
            first[L] = int(codes[s[0]])
            syms.extend(int(v) for v in s)
            off += s.size
    base[max_len + 1] = off
    if not syms:
        syms = [0]
    return first, base, np.array(syms, dtype=np.int32)


def decode_tables(lengths) -> Dict[str, np.ndarray]:
    """Decode tables the CUDA Huffman kernels use, derived from ``huff_lengths``.

    * ``limit`` ``uint32[33]``: for length ``L``, one past the largest code of
      length ``<= L`` left-justified in 32 bits (0 when no code is that short),
      with ``limit[32]`` forced to ``2**32 - 1``-style saturation handled by the
      kernel through ``max_len``.  A 32-bit MSB-first window ``w`` starts with a
      code of length ``L`` iff ``L`` is the smallest length with
      ``w < limit[L]`` (canonical codes are ordered by length).
    * ``first`` ``uint32[33]``: first code value of each length.
    * ``offset`` ``int32[33]``: index in ``sorted_syms`` of the first symbol of
      each length.
    * ``sorted_syms`` ``uint16[n_used]``: symbols in (length, code) order.
    * ``max_len``: longest code length (0 for an empty code).
    """
    codes, lengths = canonical_codes(lengths)
    max_len = int(lengths.max()) if lengths.size else 0
    count = np.bincount(lengths, minlength=MAX_CODE_LEN + 1).astype(np.int64)
    count[0] = 0
    first = np.zeros(MAX_CODE_LEN + 1, dtype=np.int64)
    c = 0
    for L in range(1, MAX_CODE_LEN + 1):
        c = (c + int(count[L - 1])) << 1
        first[L] = c
    offset = np.zeros(MAX_CODE_LEN + 1, dtype=np.int64)
    offset[1:] = np.cumsum(count[:-1])[:MAX_CODE_LEN]
    limit = np.zeros(MAX_CODE_LEN + 1, dtype=np.uint64)
    for L in range(1, MAX_CODE_LEN + 1):
        # codes of length <= L, left-justified: (first[L] + count[L]) << (32 - L)
        limit[L] = min((first[L] + count[L]) << (MAX_CODE_LEN - L), (1 << 32))
    order = np.lexsort((codes, lengths))
    order = order[lengths[order] > 0]
    return {
        "limit": limit,
        "first": first.astype(np.uint64),
        "offset": offset.astype(np.int32),
        "sorted_syms": order.astype(np.uint16),
        "max_len": max_len,
    }
