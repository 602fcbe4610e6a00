"""The C-ABI library loads without a GPU, exports every symbol ``include/cbq.h``
declares, and its host-only entry points behave (argument checks happen before
any CUDA call, table blobs match the Python derivation)."""
import ctypes as ct
import re
from pathlib import Path

import numpy as np
import pytest

from helpers import GOLDEN, cbq, golden

HEADER = Path(__file__).resolve().parent.parent / "include" / "cbq.h"
L = cbq._lib


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cbq_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    names = declared_functions()
    assert len(names) >= 15
    assert set(names) == set(L.SIGNATURES), set(names) ^ set(L.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.cbq_version() >= 1
    assert L.status_string(L.CBQ_ERR_ARG) == "invalid argument"


def test_size_queries():
    lib = L.lib()
    assert lib.cbq_fixed_stream_bytes(2048, 2048, 13) >= (2048 * 2048 * 13 + 7) // 8 + 16
    assert lib.cbq_fixed_stream_bytes(3, 5, 7) % 16 == 0
    assert lib.cbq_fixed_stream_bytes(1, 1, 17) == -1
    assert lib.cbq_huff_stream_bytes(100) >= 100 + 16
    assert lib.cbq_huff_chunk_count(10, 130) == 10 * 3
    assert lib.cbq_huff_chunk_table_words(10, 130) == 2 * 30       # offsets + packed quarter lengths
    assert lib.cbq_huff_tables_bytes(0) == -1


def test_argument_errors_are_detected_on_host():
    lib = L.lib()
    args = dict(x=None, xd=0, T=1, ldx=8, p=None, pb=1 << 20, cb=None, C=4, bits=4, M=8, K=8,
                bias=None, out=None, od=0, ldo=8, ws=None, wsb=0, s=None)
    base = list(args.values())

    def call(**kw):
        a = dict(args)
        a.update(kw)
        return lib.cbq_linear_fixed(*a.values())
    assert call(bits=0) == L.CBQ_ERR_ARG
    assert call(bits=17) == L.CBQ_ERR_ARG
    assert call(C=0) == L.CBQ_ERR_ARG
    assert call(xd=7) == L.CBQ_ERR_ARG
    assert call() == L.CBQ_ERR_ARG                 # null pointers
    assert call(T=0) == L.CBQ_OK                   # nothing to do
    assert call(x=1, p=16, cb=4, out=8, ldx=4) == L.CBQ_ERR_ARG       # ldx < K
    assert call(x=1, p=16, cb=4, out=8, pb=10) == L.CBQ_ERR_ARG       # stream too short
    assert call(x=1, p=16, cb=4, out=8, ws=64, wsb=1) == L.CBQ_ERR_ARG  # workspace too small
    assert lib.cbq_pack_fixed(None, 10, 0, None, 64, None) == L.CBQ_ERR_ARG
    assert len(base) == 18


def _blob_view(blob):
    """Decode the fields of a table blob (layout of cbq_huff.cu HuffTables)."""
    hdr = np.frombuffer(blob[:16].tobytes(), dtype=np.int32)
    limit = np.frombuffer(blob[16:16 + 264].tobytes(), dtype=np.uint64)
    first = np.frombuffer(blob[280:280 + 264].tobytes(), dtype=np.uint64)
    offset = np.frombuffer(blob[544:544 + 132].tobytes(), dtype=np.int32)
    lut = np.frombuffer(blob[688:688 + 16384].tobytes(), dtype=np.uint32)
    n_used = int(hdr[3])
    syms = np.frombuffer(blob[17072:17072 + 2 * n_used].tobytes(), dtype=np.uint16)
    return hdr, limit, first, offset, lut, syms


@pytest.mark.parametrize("case", ["hand", "single", "two", "zipf", "deep", "bf16", "deep32"])
def test_table_blob_matches_stored_tables(case):
    d = golden(f"huff_{case}.npz")
    blob = cbq.gpu_huffman_functions.tables_blob(d["huff_lengths"])
    hdr, limit, first, offset, lut, syms = _blob_view(blob)
    assert hdr[0] == 0x48514243 and hdr[1] == d["huff_lengths"].size
    assert hdr[2] == int(d["huff_lengths"].max())
    # the 12-bit LUT carries exactly the stored (sym, len) pairs
    ln = d["huff_lut_len"]
    expect = np.where(ln > 0, (ln.astype(np.uint32) << 16) | (d["huff_lut_sym"].astype(np.uint32) & 0xFFFF), 0)
    np.testing.assert_array_equal(lut, expect)
    # long codes: first codes and symbol order agree with the stored slow-path tables
    t = cbq.huffman_codebook.decode_tables(d["huff_lengths"])
    np.testing.assert_array_equal(first[1:], t["first"][1:])
    np.testing.assert_array_equal(offset, t["offset"])
    np.testing.assert_array_equal(syms, t["sorted_syms"])
    fc, bo, ss = d["huff_sl_first_code"], d["huff_sl_base_offset"], d["huff_sl_sym"]
    for Lc in range(13, fc.size - 1):
        if fc[Lc] >= 0:
            assert first[Lc] == fc[Lc]
            cnt = bo[Lc + 1] - bo[Lc]
            assert limit[Lc] == first[Lc] + cnt
            np.testing.assert_array_equal(syms[offset[Lc]:offset[Lc] + cnt], ss[bo[Lc]:bo[Lc] + cnt])


def test_table_build_rejects_oversubscribed_code():
    lens = np.array([1, 1, 1], dtype=np.uint8)
    n = L.lib().cbq_huff_tables_bytes(3)
    blob = np.zeros(n, dtype=np.uint8)
    rc = L.lib().cbq_huff_tables_build(lens.ctypes.data, 3, blob.ctypes.data, n)
    assert rc == L.CBQ_ERR_ARG
