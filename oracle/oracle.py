"""Python binding of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs import this module.  It checks the CUDA library's results; the product
(``codebook-quantization_b200``) never imports it.

Two native objects are loaded with ctypes:

* ``_build/libcbq_oracle.so`` -- ``cbq_oracle.c``, this repository's C
  restatement of the reference's decoders and GEMV loops (each function there
  cites the reference file:line it restates);
* ``_ref/libcompressed_matmul_ref.so`` -- the reference's own
  ``src/compressed_matmul.c`` compiled unmodified by ``oracle/Makefile`` when
  the reference tree was available.  It pins the restatement and serves as the
  "reference" CPU baseline; it may be absent.

Argument conventions mirror the reference's ctypes wrapper
(``src/compressed_matmul_cpu.py:94-215``): the C kernels accumulate into a
zero-initialised ``out``.
"""
from __future__ import annotations

import ctypes as ct
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libcbq_oracle.so"
REF_SO = HERE / "_ref" / "libcompressed_matmul_ref.so"

_P = ct.c_void_p
_I64 = ct.c_int64
_INT = ct.c_int


def build() -> None:
    """Build the oracle (and the reference object when its source exists)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_P)


_lib = None
_ref = None


def lib() -> ct.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            build()
        L = ct.CDLL(str(ORACLE_SO))
        L.orc_unpack_fixed.argtypes = [_P, _I64, _INT, _I64, _I64, _P]
        L.orc_linear_fixed_f32.argtypes = [_P, _P, _I64, _P, _I64, _INT, _I64, _I64, _I64, _P, _I64, _I64]
        L.orc_embedding_fixed_f32.argtypes = [_P, _I64, _P, _I64, _P, _I64, _INT, _I64, _P]
        huff = [_P, _I64, _P, _P, _P, _P, _P, _INT]
        L.orc_huff_decode_rows.argtypes = huff + [_P, _I64, _I64, _P]
        L.orc_huff_chunk_offsets.argtypes = huff + [_P, _I64, _I64, _I64, _P]
        L.orc_huff_linear_f32.argtypes = [_P] + huff + [_P, _P, _I64, _I64, _I64, _I64, _P, _I64, _I64]
        L.orc_huff_embedding_f32.argtypes = [_P, _I64] + huff + [_P, _P, _I64, _I64, _P]
        L.orc_max_threads.restype = _INT
        L.orc_set_threads.argtypes = [_INT]
        _lib = L
    return _lib


def ref_lib():
    """The reference's own compressed_matmul.c object, or None if not built."""
    global _ref
    if _ref is None and REF_SO.exists():
        L = ct.CDLL(str(REF_SO))
        L.compressed_matmul_f32_chunk.argtypes = [_P, _P, _P, _P] + [_INT] * 7
        L.huffman_matmul_f32_chunk.argtypes = [_P] * 10 + [_INT] * 7
        L.huffman_embedding_f32_rows.argtypes = [_P] * 10 + [_INT] * 4
        L.huffman_decode_to_weights_f32.argtypes = [_P] * 9 + [_INT] * 4
        _ref = L
    return _ref


def threads() -> int:
    return int(lib().orc_max_threads())


# ------------------------------------------------------------------ fixed width

def unpack_fixed(packed: np.ndarray, bits: int, n: int, first: int = 0) -> np.ndarray:
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    out = np.empty(int(n), dtype=np.uint16)
    lib().orc_unpack_fixed(_ptr(p), p.size, int(bits), int(first), int(n), _ptr(out))
    return out


def linear_fixed(x: np.ndarray, packed: np.ndarray, codebook: np.ndarray, M: int, K: int,
                 bits: int, C: int = None, r0: int = 0, r1: int = None) -> np.ndarray:
    """y[t, r] = sum_k x[t,k] * cb[min(idx, C-1)], fp32, rows [r0, r1) (others 0)."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32).reshape(-1, K))
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    cb = np.ascontiguousarray(codebook, dtype=np.float32)
    C = cb.size if C is None else int(C)
    out = np.zeros((x.shape[0], M), dtype=np.float32)
    lib().orc_linear_fixed_f32(_ptr(x), _ptr(p), p.size, _ptr(cb), C, int(bits), x.shape[0], int(M),
                               int(K), _ptr(out), int(r0), int(M if r1 is None else r1))
    return out


def embedding_fixed(ids: np.ndarray, packed: np.ndarray, codebook: np.ndarray, H: int,
                    bits: int) -> np.ndarray:
    ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int64).reshape(-1))
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    cb = np.ascontiguousarray(codebook, dtype=np.float32)
    out = np.empty((ids.size, H), dtype=np.float32)
    lib().orc_embedding_fixed_f32(_ptr(ids), ids.size, _ptr(p), p.size, _ptr(cb), cb.size, int(bits),
                                  int(H), _ptr(out))
    return out


# ------------------------------------------------------------------ Huffman

class HuffData:
    """The stored tables of one Huffman tensor in the dtypes the reference's C
    path uses (``src/compressed_modules.py:240-249``)."""

    def __init__(self, d: dict):
        self.stream = np.ascontiguousarray(d["huff_stream"], dtype=np.uint8)
        self.lut_sym = np.ascontiguousarray(d["huff_lut_sym"]).astype(np.uint16)
        self.lut_len = np.ascontiguousarray(d["huff_lut_len"]).astype(np.uint8)
        self.sl_first = np.ascontiguousarray(d["huff_sl_first_code"], dtype=np.int64)
        self.sl_base = np.ascontiguousarray(d["huff_sl_base_offset"], dtype=np.int32)
        self.sl_sym = np.ascontiguousarray(d["huff_sl_sym"]).astype(np.uint16)
        self.rbs = np.ascontiguousarray(d["huff_row_bit_starts"], dtype=np.int64)
        lens = np.asarray(d["huff_lengths"], dtype=np.uint8)
        self.max_len = int(lens.max()) if lens.size and lens.max() > 0 else 1

    def args(self):
        return [_ptr(self.stream), self.stream.size, _ptr(self.lut_sym), _ptr(self.lut_len),
                _ptr(self.sl_first), _ptr(self.sl_base), _ptr(self.sl_sym), self.max_len]


def huff_decode_rows(d: dict, M: int, K: int) -> np.ndarray:
    h = HuffData(d)
    out = np.empty(M * K, dtype=np.uint16)
    lib().orc_huff_decode_rows(*h.args(), _ptr(h.rbs), int(M), int(K), _ptr(out))
    return out


def huff_chunk_offsets(d: dict, M: int, K: int, S: int = 64) -> np.ndarray:
    h = HuffData(d)
    nch = (K + S - 1) // S
    out = np.zeros(M * nch, dtype=np.int64)
    lib().orc_huff_chunk_offsets(*h.args(), _ptr(h.rbs), int(M), int(K), int(S), _ptr(out))
    return out


def huff_linear(x: np.ndarray, d: dict, codebook: np.ndarray, M: int, K: int,
                C: int = None) -> np.ndarray:
    h = HuffData(d)
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32).reshape(-1, K))
    cb = np.ascontiguousarray(codebook, dtype=np.float32)
    C = cb.size if C is None else int(C)
    out = np.zeros((x.shape[0], M), dtype=np.float32)
    lib().orc_huff_linear_f32(_ptr(x), *h.args(), _ptr(h.rbs), _ptr(cb), C, x.shape[0], int(M), int(K),
                              _ptr(out), 0, int(M))
    return out


def huff_embedding(ids: np.ndarray, d: dict, codebook: np.ndarray, H: int) -> np.ndarray:
    h = HuffData(d)
    ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int64).reshape(-1))
    cb = np.ascontiguousarray(codebook, dtype=np.float32)
    out = np.empty((ids.size, H), dtype=np.float32)
    lib().orc_huff_embedding_f32(_ptr(ids), ids.size, *h.args(), _ptr(h.rbs), _ptr(cb), cb.size,
                                 int(H), _ptr(out))
    return out


# ------------------------------------------------------------------ reference object

def ref_linear_fixed(x, packed, codebook, M, K, bits, chunk_rows=None):
    """The reference's compressed_matmul_f32_chunk, called like
    src/compressed_matmul_cpu.py:279-343 (chunk_rows=None: one call)."""
    L = ref_lib()
    if L is None:
        return None
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32).reshape(-1, K))
    p = np.concatenate([np.asarray(packed, dtype=np.uint8), np.zeros(4, np.uint8)])
    cb = np.ascontiguousarray(codebook, dtype=np.float32)
    out = np.zeros((x.shape[0], M), dtype=np.float32)
    step = M if chunk_rows is None else int(chunk_rows)
    for r in range(0, M, step):
        L.compressed_matmul_f32_chunk(_ptr(x), _ptr(p), _ptr(cb), _ptr(out), x.shape[0], M, K, cb.size,
                                      int(bits), r, min(r + step, M))
    return out


def ref_huff_linear(x, d, codebook, M, K, chunk_rows=None):
    """The reference's huffman_matmul_f32_chunk (src/compressed_matmul_cpu.py:446-506)."""
    L = ref_lib()
    if L is None:
        return None
    h = HuffData(d)
    stream = np.concatenate([h.stream, np.zeros(4, np.uint8)])
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32).reshape(-1, K))
    cb = np.ascontiguousarray(codebook, dtype=np.float32)
    out = np.zeros((x.shape[0], M), dtype=np.float32)
    step = M if chunk_rows is None else int(chunk_rows)
    for r in range(0, M, step):
        L.huffman_matmul_f32_chunk(_ptr(x), _ptr(stream), _ptr(h.lut_sym), _ptr(h.lut_len),
                                   _ptr(h.sl_first), _ptr(h.sl_base), _ptr(h.sl_sym), _ptr(h.rbs),
                                   _ptr(cb), _ptr(out), x.shape[0], M, K, cb.size, r,
                                   min(r + step, M), h.max_len)
    return out


def ref_huff_decode_weights(d, codebook, M, K):
    L = ref_lib()
    if L is None:
        return None
    h = HuffData(d)
    stream = np.concatenate([h.stream, np.zeros(4, np.uint8)])
    cb = np.ascontiguousarray(codebook, dtype=np.float32)
    out = np.empty((M, K), dtype=np.float32)
    L.huffman_decode_to_weights_f32(_ptr(stream), _ptr(h.lut_sym), _ptr(h.lut_len), _ptr(h.sl_first),
                                    _ptr(h.sl_base), _ptr(h.sl_sym), _ptr(h.rbs), _ptr(cb), _ptr(out),
                                    M, K, cb.size, h.max_len)
    return out


def host_cores() -> int:
    """Cores this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def set_threads(n: int) -> int:
    """Use ``n`` OpenMP threads in the oracle and the reference object from
    now on (whatever OMP_NUM_THREADS says); returns the count now in effect."""
    os.environ["OMP_NUM_THREADS"] = str(int(n))
    lib().orc_set_threads(int(n))
    return threads()
