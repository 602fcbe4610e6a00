"""Tensor-parallel shards of compressed tensors, cut at load time.

A column-parallel layer (q, k, v, gate, up, lm_head) keeps a contiguous block
of output rows on each rank; a row-parallel layer (o, down) keeps a block of
input columns and its partial products are all-reduced.  The reference has
no tensor parallelism (it runs one process on one device); these functions
cut its unchanged ``.npz`` payloads:

* fixed width, rows: the bit range of rows ``[r0, r1)`` of the LSB-first
  stream (``src/bitpack.py:32-94``) -- a byte slice when ``r0*K*bits`` is a
  multiple of 8 (always for the BASELINE shapes), else re-aligned;
* fixed width, columns: unpack, keep columns ``[c0, c1)``, pack again with
  the same width;
* Huffman, rows: the bit range ``[row_bit_starts[r0], row_bit_starts[r1])``
  of the MSB-first stream (``src/huffman_codebook.py:126-226``) shifted to
  start at bit 0, row starts re-based, the code lengths unchanged;
* Huffman, columns: the decoded index matrix's columns ``[c0, c1)``
  re-encoded with the SAME canonical code (same ``huff_lengths``), so every
  shard decodes to exactly the unsharded matrix's indices for its block.

Every shard is a complete tensor in the reference's format (plus the 4 zero
pad bytes the Huffman stream carries), so the single-device kernels run on it
unchanged.
"""
from __future__ import annotations

from typing import Dict, Tuple

import numpy as np

from . import bitpack
from . import huffman_codebook as hc

__all__ = ["shard_range", "shift_bits_msb", "shift_bits_lsb", "shard_fixed_rows", "shard_fixed_cols",
           "shard_huffman_rows", "huffman_encode_rows_with_lengths", "shard_huffman_cols"]


def shard_range(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Block ``[lo, hi)`` of ``n`` for ``rank`` of ``world`` (n must divide)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if n % world:
        raise ValueError(f"dimension {n} does not split over {world} ranks")
    s = n // world
    return rank * s, (rank + 1) * s


def _as_bytes(stream) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(stream).reshape(-1).view(np.uint8))


def shift_bits_msb(stream, bit0: int, nbits: int) -> np.ndarray:
    """Bits ``[bit0, bit0 + nbits)`` of an MSB-first byte stream, moved to
    start at bit 0 (MSB of byte 0); returns ``ceil(nbits/8)`` bytes."""
    src = _as_bytes(stream)
    nbytes = (nbits + 7) // 8
    if nbits == 0:
        return np.zeros(0, dtype=np.uint8)
    b0, s = bit0 // 8, bit0 % 8
    chunk = src[b0:b0 + nbytes + 1]
    if chunk.size < nbytes + 1:
        chunk = np.concatenate([chunk, np.zeros(nbytes + 1 - chunk.size, dtype=np.uint8)])
    if s == 0:
        out = chunk[:nbytes].copy()
    else:
        hi = chunk[:nbytes].astype(np.uint16) << s
        lo = chunk[1:nbytes + 1].astype(np.uint16) >> (8 - s)
        out = ((hi | lo) & 0xFF).astype(np.uint8)
    tail = nbits % 8
    if tail:
        out[-1] &= np.uint8((0xFF << (8 - tail)) & 0xFF)
    return out


def shift_bits_lsb(stream, bit0: int, nbits: int) -> np.ndarray:
    """Bits ``[bit0, bit0 + nbits)`` of an LSB-first byte stream, moved to
    start at bit 0 (LSB of byte 0); returns ``ceil(nbits/8)`` bytes."""
    src = _as_bytes(stream)
    nbytes = (nbits + 7) // 8
    if nbits == 0:
        return np.zeros(0, dtype=np.uint8)
    b0, s = bit0 // 8, bit0 % 8
    chunk = src[b0:b0 + nbytes + 1]
    if chunk.size < nbytes + 1:
        chunk = np.concatenate([chunk, np.zeros(nbytes + 1 - chunk.size, dtype=np.uint8)])
    if s == 0:
        out = chunk[:nbytes].copy()
    else:
        lo = chunk[:nbytes].astype(np.uint16) >> s
        hi = chunk[1:nbytes + 1].astype(np.uint16) << (8 - s)
        out = ((lo | hi) & 0xFF).astype(np.uint8)
    tail = nbits % 8
    if tail:
        out[-1] &= np.uint8((1 << tail) - 1)
    return out


def shard_fixed_rows(indices, M: int, K: int, bits: int, r0: int, r1: int) -> np.ndarray:
    """Packed stream of rows ``[r0, r1)`` of a fixed-width ``[M, K]`` stream."""
    if not 0 <= r0 <= r1 <= M:
        raise ValueError(f"rows [{r0}, {r1}) outside [0, {M})")
    return shift_bits_lsb(indices, r0 * K * bits, (r1 - r0) * K * bits)


def shard_fixed_cols(indices, M: int, K: int, bits: int, c0: int, c1: int) -> np.ndarray:
    """Packed stream of columns ``[c0, c1)`` (same width) of a fixed-width ``[M, K]`` stream."""
    if not 0 <= c0 <= c1 <= K:
        raise ValueError(f"columns [{c0}, {c1}) outside [0, {K})")
    idx = bitpack.unpack_any_bits(_as_bytes(indices), bits, M * K).reshape(M, K)
    return bitpack.pack_any_bits(np.ascontiguousarray(idx[:, c0:c1]).reshape(-1), bits)


def shard_huffman_rows(d: Dict[str, np.ndarray], M: int, K: int, r0: int, r1: int) -> Dict[str, np.ndarray]:
    """Rows ``[r0, r1)`` of a Huffman tensor (``huff_*`` keys), same code."""
    if not 0 <= r0 < r1 <= M:
        raise ValueError(f"rows [{r0}, {r1}) outside [0, {M})")
    rbs = np.asarray(d["huff_row_bit_starts"], dtype=np.int64).reshape(-1)
    stream = _as_bytes(d["huff_stream"])
    total = (stream.size - 4) * 8                     # the stream ends with 4 zero pad bytes
    end = int(rbs[r1]) if r1 < M else _huffman_end_bit(d, M, K)
    start = int(rbs[r0])
    if not start <= end <= total:
        raise ValueError("row bit starts do not fit the stream")
    body = shift_bits_msb(stream, start, end - start)
    out = {k: v for k, v in d.items() if not k.startswith("huff_")}
    out.update(_huffman_tables(d))
    out["huff_stream"] = np.concatenate([body, np.zeros(4, dtype=np.uint8)])
    out["huff_row_bit_starts"] = (rbs[r0:r1] - start).astype(np.int64)
    out["huff_n"] = np.array([(r1 - r0) * K], dtype=np.int64)
    return out


def _huffman_end_bit(d: Dict[str, np.ndarray], M: int, K: int) -> int:
    """End of the last row.  The format does not store the exact bit length;
    the stream's byte length (minus the 4 pad bytes) bounds it, and the at
    most 7 zero bits after the last code are never read (a row ends after K
    symbols)."""
    return (_as_bytes(d["huff_stream"]).size - 4) * 8


def _huffman_tables(d: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
    keep = ("huff_lengths", "huff_lut_sym", "huff_lut_len", "huff_sl_first_code", "huff_sl_base_offset",
            "huff_sl_sym", "encoding")
    return {k: d[k] for k in keep if k in d}


def huffman_encode_rows_with_lengths(idx2d: np.ndarray, lengths) -> Tuple[np.ndarray, np.ndarray]:
    """Encode an index matrix ``[m, k]`` with the canonical code of ``lengths``
    (no new code is built): returns (stream incl. 4 pad bytes, row bit starts)."""
    idx2d = np.asarray(idx2d)
    m, k = idx2d.shape
    codes, lens = hc.canonical_codes(np.asarray(lengths))
    flat = np.ascontiguousarray(idx2d).reshape(-1).astype(np.int64)
    if flat.size and (flat.max() >= lens.size or (lens[flat] == 0).any()):
        raise ValueError("an index has no code in the given code lengths")
    stream, starts = hc._encode_stream(flat, codes, lens)
    rbs = starts[::k].astype(np.int64) if k and m else np.zeros(max(m, 1), dtype=np.int64)
    return stream, rbs


def shard_huffman_cols(d: Dict[str, np.ndarray], idx2d: np.ndarray, c0: int, c1: int) -> Dict[str, np.ndarray]:
    """Columns ``[c0, c1)`` of a Huffman tensor whose decoded index matrix is
    ``idx2d`` ``[M, K]``, re-encoded with the tensor's own code lengths."""
    M, K = idx2d.shape
    if not 0 <= c0 < c1 <= K:
        raise ValueError(f"columns [{c0}, {c1}) outside [0, {K})")
    stream, rbs = huffman_encode_rows_with_lengths(idx2d[:, c0:c1], d["huff_lengths"])
    out = {k: v for k, v in d.items() if not k.startswith("huff_")}
    out.update(_huffman_tables(d))
    out["huff_stream"] = stream
    out["huff_row_bit_starts"] = rbs
    out["huff_n"] = np.array([M * (c1 - c0)], dtype=np.int64)
    return out
