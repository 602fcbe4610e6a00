"""Generate the golden fixtures in this directory from the reference itself.

Run where the reference tree is present, with ``$CBQ_REFERENCE`` naming its
root, after ``make -C oracle REF=$CBQ_REFERENCE``::

    CBQ_REFERENCE=<reference root> python tests/golden/make_golden.py

It imports the reference's own ``src/bitpack.py`` and
``src/huffman_codebook.py`` (read-only; no byte-code is written) and calls the
reference's ``src/compressed_matmul.c`` built unmodified into
``oracle/_ref/``.  The fixtures pin the oracle and the package's format code
on machines where the reference is absent.  Cases follow the reference's own
tests:

* pack/unpack for every width 1..16 (``tests/test_bitpack.py``,
  ``tests/test_compressed_roundtrip.py:59-79``);
* the 16-symbol two-row hand stream (``diagnostics/test_huffman_gpu.py:29-36``),
  the single- and two-symbol codes (``tests/test_compressed_roundtrip.py:281-300``),
  a Zipf-1.5 stream (``:261-279``), the deep-tree regression's distribution
  (``:302-334``; 18-bit codes at its size), a complete code whose lengths run
  1..32 (``deep32``), and a bf16 N(0, 0.02) lossless tensor;
* GEMV / embedding outputs of ``compressed_matmul_f32_chunk``,
  ``huffman_matmul_f32_chunk`` and ``huffman_embedding_f32_rows``.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

sys.dont_write_bytecode = True
HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
if not os.environ.get("CBQ_REFERENCE"):
    sys.exit("set CBQ_REFERENCE to the reference project's root directory")
REF = Path(os.environ["CBQ_REFERENCE"])
sys.path.insert(0, str(REF / "src"))
sys.path.insert(0, str(REPO / "oracle"))

import bitpack as ref_bitpack            # noqa: E402  (the reference's module)
import huffman_codebook as ref_huff      # noqa: E402  (the reference's module)
import oracle                            # noqa: E402

HUFF_KEYS = ("huff_lengths", "huff_stream", "huff_n", "huff_row_bit_starts", "huff_lut_sym",
             "huff_lut_len", "huff_sl_first_code", "huff_sl_base_offset", "huff_sl_sym")


def bf16_trunc(w: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit pattern by truncation (reference src/compressor.py:28-34)."""
    return (w.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)


def freq_sorted_codebook(bf: np.ndarray):
    """Distinct bf16 values by descending count, ties by bit pattern."""
    hist = np.bincount(bf.reshape(-1), minlength=65536)
    vals = np.flatnonzero(hist)
    order = np.lexsort((vals, -hist[vals]))
    vals = vals[order]
    lut = np.zeros(65536, dtype=np.uint16)
    lut[vals] = np.arange(vals.size, dtype=np.uint16)
    cb = (vals.astype(np.uint32) << 16).view(np.float32).astype(np.float32)
    return cb, lut[bf]


def pack_cases():
    out = {}
    for bits in range(1, 17):
        rng = np.random.default_rng(1000 + bits)
        n = 997 if bits != 4 else 999          # odd lengths exercise the tails
        idx = rng.integers(0, 1 << bits, size=n).astype(np.uint16)
        out[f"b{bits}_idx"] = idx
        out[f"b{bits}_packed"] = ref_bitpack.pack_any_bits(idx, bits)
        out[f"b{bits}_unpacked"] = ref_bitpack.unpack_any_bits(out[f"b{bits}_packed"], bits, n)
    return out


def huff_case(idx: np.ndarray, shape):
    enc = ref_huff.huffman_encode_indices(idx, shape=shape)
    d = {k: np.asarray(enc[k]) for k in HUFF_KEYS}
    d["indices"] = np.asarray(idx, dtype=np.uint16).reshape(-1)
    d["shape"] = np.array(shape, dtype=np.int64)
    dec = ref_huff.huffman_decode_indices(enc["huff_stream"], enc["huff_lengths"],
                                          int(enc["huff_n"][0]))
    assert np.array_equal(dec, d["indices"]), "reference round trip failed"
    return d


def deep32_case():
    """Code lengths 1, 2, ..., 31, 32, 32 (a complete code reaching 32 bits).

    Frequencies that make the reference encoder build such a tree would need
    millions of symbols, so the codes come from the reference's
    ``_canonical_codes`` and its table builders, the bits are concatenated
    MSB-first here, and the reference's ``huffman_decode_indices`` confirms
    the stream decodes back to the indices."""
    lengths = np.array(list(range(1, 33)) + [32], dtype=np.uint8)
    codes = ref_huff._canonical_codes(lengths)
    rng = np.random.default_rng(3232)
    M, K = 48, 80
    idx = rng.integers(0, lengths.size, size=M * K).astype(np.uint16)
    bits, starts, pos = [], [], 0
    for i, s in enumerate(idx.tolist()):
        if i % K == 0:
            starts.append(pos)
        c, L = codes[s]
        bits.append(format(c, f"0{L}b"))
        pos += L
    bitstr = "".join(bits)
    nbytes = (len(bitstr) + 7) // 8
    bitstr += "0" * (nbytes * 8 - len(bitstr))
    stream = np.frombuffer(int(bitstr, 2).to_bytes(nbytes, "big"), dtype=np.uint8)
    stream = np.concatenate([stream, np.zeros(4, np.uint8)])
    lut_sym, lut_len = ref_huff.build_gpu_lut(lengths)
    fc, bo, ss = ref_huff._build_slow_path_tables(lengths)
    dec = ref_huff.huffman_decode_indices(stream, lengths, idx.size)
    assert np.array_equal(dec, idx), "reference decoder disagrees on the 32-bit code"
    return {"huff_lengths": lengths, "huff_stream": stream, "huff_n": np.array([idx.size], np.int64),
            "huff_row_bit_starts": np.array(starts, np.int64), "huff_lut_sym": lut_sym,
            "huff_lut_len": lut_len, "huff_sl_first_code": fc, "huff_sl_base_offset": bo,
            "huff_sl_sym": ss, "indices": idx, "shape": np.array([M, K], np.int64),
            "codebook": rng.standard_normal(lengths.size).astype(np.float32)}


def huffman_cases():
    cases = {}
    hand = np.array([3, 1, 0, 3, 2, 1, 0, 3, 0, 1, 2, 3, 0, 1, 2, 3], dtype=np.uint16)
    cases["hand"] = huff_case(hand, (2, 8))
    cases["single"] = huff_case(np.zeros(256, dtype=np.uint16), (4, 64))
    rng = np.random.default_rng(0)
    cases["two"] = huff_case(rng.integers(0, 2, size=512, dtype=np.uint16), (8, 64))
    rng = np.random.default_rng(4096 + 10)
    maxv = (1 << 10) - 1
    p = 1.0 / (np.arange(1, maxv + 2) ** 1.5)
    p /= p.sum()
    cases["zipf"] = huff_case(rng.choice(maxv + 1, size=4096, p=p).astype(np.uint16), (64, 64))
    rng = np.random.default_rng(777)
    n_syms = 5000
    freq = np.ones(n_syms, dtype=np.int64)
    freq[:200] = rng.integers(1000, 10000, size=200)
    freq[200:500] = rng.integers(100, 1000, size=300)
    p = freq.astype(np.float64) / freq.sum()
    cases["deep"] = huff_case(rng.choice(n_syms, size=4096 * 64, p=p).astype(np.uint16), (4096, 64))
    rng = np.random.default_rng(2024)
    bf = bf16_trunc(rng.standard_normal((96, 256)).astype(np.float32) * 0.02)
    cb, idx = freq_sorted_codebook(bf)
    d = huff_case(idx.reshape(-1), (96, 256))
    d["codebook"] = cb
    d["bf16"] = bf
    cases["bf16"] = d
    cases["deep32"] = deep32_case()
    return cases


def gemv_cases(huff):
    assert oracle.ref_lib() is not None, "build the reference object first: make -C oracle"
    out = {}
    rng = np.random.default_rng(31337)
    M, K, bits = 80, 384, 13
    bf = bf16_trunc(rng.standard_normal((M, K)).astype(np.float32) * 0.02)
    cb, idx = freq_sorted_codebook(bf)
    packed = ref_bitpack.pack_any_bits(idx.reshape(-1), bits)
    x = rng.standard_normal((3, K)).astype(np.float32)
    out.update(fx_codebook=cb, fx_packed=packed, fx_x=x, fx_shape=np.array([M, K, bits]),
               fx_out=oracle.ref_linear_fixed(x, packed, cb, M, K, bits, chunk_rows=32),
               fx_bf16=bf)
    ids = np.array([0, 5, M - 1, 5], dtype=np.int64)
    out["fx_emb_ids"] = ids
    d = huff["bf16"]
    hM, hK = (int(v) for v in d["shape"])
    hx = rng.standard_normal((2, hK)).astype(np.float32)
    out["hf_x"] = hx
    out["hf_out"] = oracle.ref_huff_linear(hx, d, d["codebook"], hM, hK, chunk_rows=16)
    L = oracle.ref_lib()
    h = oracle.HuffData(d)
    stream = np.concatenate([h.stream, np.zeros(4, np.uint8)])
    hid = np.array([3, 0, hM - 1, 3], dtype=np.int32)
    emb = np.empty((hid.size, hK), dtype=np.float32)
    cbv = np.ascontiguousarray(d["codebook"], dtype=np.float32)
    P = oracle._ptr
    L.huffman_embedding_f32_rows(P(hid), P(stream), P(h.lut_sym), P(h.lut_len), P(h.sl_first),
                                 P(h.sl_base), P(h.sl_sym), P(h.rbs), P(cbv), P(emb), hid.size, hK,
                                 cbv.size, h.max_len)
    out["hf_emb_ids"] = hid.astype(np.int64)
    out["hf_emb"] = emb
    out["hf_weights"] = oracle.ref_huff_decode_weights(d, d["codebook"], hM, hK)
    return out


def main():
    np.savez_compressed(HERE / "pack.npz", **pack_cases())
    huff = huffman_cases()
    for name, d in huff.items():
        np.savez_compressed(HERE / f"huff_{name}.npz", **d)
    np.savez_compressed(HERE / "gemv.npz", **gemv_cases(huff))
    for f in sorted(HERE.glob("*.npz")):
        print(f"{f.name:24s} {f.stat().st_size:9d} B")


if __name__ == "__main__":
    main()
