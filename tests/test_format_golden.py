"""Format code and oracle against the golden fixtures made by the reference.

The fixtures (``tests/golden/*.npz``, written by ``tests/golden/make_golden.py``
from the reference's own ``bitpack.py``, ``huffman_codebook.py`` and
``compressed_matmul.c``) pin, bit for bit:

* the package's packer / unpacker and Huffman encoder and table builders;
* the oracle's decoders and GEMV / embedding loops.
"""
import glob

import numpy as np
import pytest

import oracle
from helpers import GOLDEN, cbq, golden, rel_l2

HUFF_FILES = sorted(glob.glob(str(GOLDEN / "huff_*.npz")))
HUFF_KEYS = ("huff_lengths", "huff_stream", "huff_n", "huff_row_bit_starts", "huff_lut_sym",
             "huff_lut_len", "huff_sl_first_code", "huff_sl_base_offset", "huff_sl_sym")


@pytest.mark.parametrize("bits", range(1, 17))
def test_pack_matches_reference(bits):
    g = golden("pack.npz")
    idx, packed = g[f"b{bits}_idx"], g[f"b{bits}_packed"]
    mine = cbq.bitpack.pack_any_bits(idx, bits)
    assert mine.dtype == np.uint8 and mine.size == cbq.bitpack.packed_size(idx.size, bits)
    np.testing.assert_array_equal(mine, packed)
    np.testing.assert_array_equal(cbq.bitpack.unpack_any_bits(packed, bits, idx.size), idx)
    np.testing.assert_array_equal(g[f"b{bits}_unpacked"], idx)


@pytest.mark.parametrize("bits", range(1, 17))
def test_oracle_unpack_matches_reference(bits):
    g = golden("pack.npz")
    idx, packed = g[f"b{bits}_idx"], g[f"b{bits}_packed"]
    np.testing.assert_array_equal(oracle.unpack_fixed(packed, bits, idx.size), idx)


@pytest.mark.parametrize("bits", [8, 13])
@pytest.mark.parametrize("start", [0, 3, 5, 8, 11, 24, 600])
def test_seek_equals_slice(bits, start):
    """Seeking to any element equals slicing a full unpack
    (reference tests/test_index_seek.py:46-131)."""
    g = golden("pack.npz")
    idx, packed = g[f"b{bits}_idx"], g[f"b{bits}_packed"]
    n = min(64, idx.size - start)
    np.testing.assert_array_equal(cbq.bitpack.unpack_any_bits(packed, bits, n, first=start),
                                  idx[start:start + n])
    np.testing.assert_array_equal(oracle.unpack_fixed(packed, bits, n, first=start), idx[start:start + n])


@pytest.mark.parametrize("path", HUFF_FILES, ids=lambda p: p.rsplit("/", 1)[-1])
def test_huffman_encoder_matches_reference(path):
    d = dict(np.load(path))
    if "deep32" in path:
        pytest.skip("deep32 is built from canonical codes directly, not by the encoder")
    M, K = (int(v) for v in d["shape"])
    enc = cbq.huffman_codebook.huffman_encode_indices(d["indices"], shape=(M, K))
    assert set(enc) == set(HUFF_KEYS)
    for k in HUFF_KEYS:
        a = np.asarray(enc[k])
        assert a.dtype == d[k].dtype, k
        np.testing.assert_array_equal(a, d[k], err_msg=k)


@pytest.mark.parametrize("path", HUFF_FILES, ids=lambda p: p.rsplit("/", 1)[-1])
def test_huffman_tables_match_reference(path):
    d = dict(np.load(path))
    sym, ln = cbq.huffman_codebook.build_gpu_lut(d["huff_lengths"])
    np.testing.assert_array_equal(sym, d["huff_lut_sym"])
    np.testing.assert_array_equal(ln, d["huff_lut_len"])
    for a, b in zip(cbq.huffman_codebook.build_slow_path_tables(d["huff_lengths"]),
                    (d["huff_sl_first_code"], d["huff_sl_base_offset"], d["huff_sl_sym"])):
        assert a.dtype == b.dtype
        np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("path", HUFF_FILES, ids=lambda p: p.rsplit("/", 1)[-1])
def test_oracle_huffman_decode_matches_reference(path):
    d = dict(np.load(path))
    M, K = (int(v) for v in d["shape"])
    np.testing.assert_array_equal(oracle.huff_decode_rows(d, M, K), d["indices"])


@pytest.mark.parametrize("path", HUFF_FILES, ids=lambda p: p.rsplit("/", 1)[-1])
def test_oracle_chunk_offsets_are_entry_points(path):
    """Decoding from every chunk offset reproduces the chunk's indices."""
    d = dict(np.load(path))
    M, K = (int(v) for v in d["shape"])
    offs = oracle.huff_chunk_offsets(d, M, K, 64).reshape(M, -1)
    rbs = d["huff_row_bit_starts"]
    idx = d["indices"].reshape(M, K)
    for r in (0, M // 2, M - 1):
        for c in range(offs.shape[1]):
            e = dict(d)
            e["huff_row_bit_starts"] = np.array([rbs[r] + offs[r, c]], dtype=np.int64)
            n = min(64, K - 64 * c)
            got = oracle.huff_decode_rows(e, 1, n)
            np.testing.assert_array_equal(got, idx[r, 64 * c:64 * c + n])


def test_oracle_linear_fixed_equals_reference_output():
    g = golden("gemv.npz")
    M, K, bits = (int(v) for v in g["fx_shape"])
    y = oracle.linear_fixed(g["fx_x"], g["fx_packed"], g["fx_codebook"], M, K, bits)
    np.testing.assert_array_equal(y, g["fx_out"])


def test_oracle_huffman_linear_and_embedding_equal_reference_output():
    g = golden("gemv.npz")
    d = golden("huff_bf16.npz")
    M, K = (int(v) for v in d["shape"])
    y = oracle.huff_linear(g["hf_x"], d, d["codebook"], M, K)
    np.testing.assert_array_equal(y, g["hf_out"])
    e = oracle.huff_embedding(g["hf_emb_ids"], d, d["codebook"], K)
    np.testing.assert_array_equal(e, g["hf_emb"])
    w = d["codebook"][d["indices"]].reshape(M, K)
    np.testing.assert_array_equal(w, g["hf_weights"])


def test_fixed_embedding_oracle_rows():
    g = golden("gemv.npz")
    M, K, bits = (int(v) for v in g["fx_shape"])
    cb, idx = cbq.synth.lossless_indices_np(g["fx_bf16"]) if hasattr(cbq, "synth") else (None, None)
    ids = g["fx_emb_ids"]
    e = oracle.embedding_fixed(ids, g["fx_packed"], g["fx_codebook"], K, bits)
    full = oracle.unpack_fixed(g["fx_packed"], bits, M * K).reshape(M, K)
    np.testing.assert_array_equal(e, g["fx_codebook"][full[ids]])
    # lossless: the codebook reproduces the original bf16 weights exactly
    w = (g["fx_bf16"].astype(np.uint32) << 16).view(np.float32)
    np.testing.assert_array_equal(g["fx_codebook"][full], w)


def test_huffman_single_symbol_and_guard():
    """A one-symbol code is incomplete: a '1' bit matches nothing and the
    reference's guard emits symbol 0 and advances one bit."""
    d = golden("huff_single.npz")
    e = dict(d)
    e["huff_stream"] = np.array([0b10100000, 0, 0, 0, 0], dtype=np.uint8)
    e["huff_row_bit_starts"] = np.array([0], dtype=np.int64)
    got = oracle.huff_decode_rows(e, 1, 5)
    np.testing.assert_array_equal(got, [0, 0, 0, 0, 0])


def test_synthetic_lossless_codebook_is_exact():
    bf = cbq.synth.bf16_normal_np((64, 256), seed=7)
    d = cbq.synth.compress_fixed_np(bf)
    cb, nb = d["codebook"], d["bits"]
    assert nb == int(np.ceil(np.log2(max(cb.size, 2))))
    idx = cbq.bitpack.unpack_any_bits(d["indices"], nb, bf.size)
    np.testing.assert_array_equal(cb[idx].view(np.uint32) >> 16, bf.reshape(-1))
    # descending frequency order
    counts = np.bincount(idx, minlength=cb.size)
    assert np.all(np.diff(counts) <= 0)


def test_oracle_vs_reference_object_random():
    """The oracle restatement equals the reference's compiled C on fresh data."""
    if oracle.ref_lib() is None:
        pytest.skip("reference object not built here")
    rng = np.random.default_rng(5)
    for (M, K, T, bits) in [(64, 32, 1, 8), (256, 128, 3, 13), (100, 64, 2, 13), (128, 64, 8, 11)]:
        idx = rng.integers(0, 1 << bits, size=M * K).astype(np.uint16)
        packed = cbq.bitpack.pack_any_bits(idx, bits)
        C = (1 << bits) - 5                     # some indices >= C exercise the clamp
        cb = rng.standard_normal(C).astype(np.float32)
        x = rng.standard_normal((T, K)).astype(np.float32)
        a = oracle.linear_fixed(x, packed, cb, M, K, bits)
        b = oracle.ref_linear_fixed(x, packed, cb, M, K, bits)
        np.testing.assert_array_equal(a, b)
        ref_dense = x.astype(np.float64) @ cb[np.minimum(idx, C - 1)].reshape(M, K).T.astype(np.float64)
        assert rel_l2(a, ref_dense) < 1e-5
