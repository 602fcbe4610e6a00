"""ctypes binding of ``libcbq.so`` (the C ABI declared in ``include/cbq.h``).

The library is built in-tree (``csrc/Makefile``) and loaded from the package
directory.  There is no fallback: if the library is missing or a CUDA device
is absent, every compute call raises.  Status codes other than ``CBQ_OK``
become :class:`CbqError`.
"""
from __future__ import annotations

import ctypes as ct
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libcbq.so"
CSRC = HERE / "csrc"

CBQ_OK, CBQ_ERR_CUDA, CBQ_ERR_ARG, CBQ_ERR_CORRUPT, CBQ_ERR_TIMEOUT, CBQ_ERR_UNSUPPORTED = range(6)
CBQ_F32, CBQ_BF16 = 0, 1
CBQ_HUFF_CHUNK = 64
FLAG_CORRUPT, FLAG_ROW_END, FLAG_TIMEOUT, FLAG_SPAN = 1, 2, 4, 8

_P = ct.c_void_p
_I64 = ct.c_int64
_INT = ct.c_int

# name -> (restype, argtypes); the order of include/cbq.h
SIGNATURES = {
    "cbq_status_string": (ct.c_char_p, [_INT]),
    "cbq_version": (_INT, []),
    "cbq_fixed_stream_bytes": (_I64, [_I64, _I64, _INT]),
    "cbq_linear_fixed_workspace_bytes": (_I64, [_I64, _I64, _I64]),
    "cbq_linear_fixed": (_INT, [_P, _INT, _I64, _I64, _P, _I64, _P, _I64, _INT, _I64, _I64, _P, _P,
                                _INT, _I64, _P, _I64, _P]),
    "cbq_linear_fixed_multi": (_INT, [_P, _INT, _I64, _I64, _INT, _P, _P, _P, _P, _I64, _INT, _I64, _P,
                                      _P, _P, _P, _INT, _INT, _P]),
    "cbq_linear_fixed_multi_norm": (_INT, [_P, _INT, _I64, _I64, _INT, _P, _P, _P, _P, _I64, _INT, _I64, _P,
                                           _P, _P, _P, _INT, _INT, _P, ct.c_float, _P]),
    "cbq_linear_fixed_multi_allreduce_norm": (_INT, [_P, _INT, _I64, _I64, _INT, _P, _P, _P, _P, _I64, _INT, _I64,
                                                     _P, _P, _P, _P, _INT, _INT, _P, ct.c_float, _INT, _P, _P, _P,
                                                     _P, _I64, _P, _P]),
    "cbq_linear_fixed_peer_flagged": (_INT, [_P, _INT, _I64, _I64, _P, _I64, _P, _I64, _INT, _I64, _I64, _P, _INT,
                                             _P, _P, _I64, _INT, _P]),
    "cbq_linear_fixed_peer": (_INT, [_P, _INT, _I64, _I64, _P, _I64, _P, _I64, _INT, _I64, _I64, _P, _INT,
                                     _P, _P, _I64, _INT, _P]),
    "cbq_linear_fixed_peer_norm": (_INT, [_P, _INT, _I64, _I64, _P, _I64, _P, _I64, _INT, _I64, _I64, _P, _INT,
                                          _P, _P, _I64, _INT, _P, _P, _P, _I64, _P, _I64, _P, ct.c_float, _P,
                                          _I64, _P, _P, _P]),
    "cbq_linear_fixed_residual_norm": (_INT, [_P, _INT, _I64, _I64, _P, _I64, _P, _I64, _INT, _I64, _I64, _P,
                                              _P, _I64, _INT, _P, ct.c_float, _P, _I64, _P, _P]),
    "cbq_linear_fixed_noalloc": (_INT, [_P, _INT, _I64, _I64, _P, _I64, _P, _I64, _INT, _I64, _I64, _P,
                                        _P, _INT, _I64, _P]),
    "cbq_host_register": (_INT, [_P, _I64, _INT]),
    "cbq_host_unregister": (_INT, [_P]),
    "cbq_streamed_chunk_rows": (_I64, [_I64, _I64, _INT, _I64]),
    "cbq_linear_fixed_streamed": (_INT, [_P, _INT, _I64, _I64, _P, _I64, _P, _I64, _INT, _I64, _I64, _P, _P,
                                         _INT, _I64, _P, _I64, _P, _I64, _P]),
    "cbq_embedding_fixed": (_INT, [_P, _I64, _P, _I64, _P, _I64, _INT, _I64, _I64, _P, _INT, _P, _P]),
    "cbq_unpack_fixed": (_INT, [_P, _I64, _INT, _I64, _P, _P]),
    "cbq_pack_fixed": (_INT, [_P, _I64, _INT, _P, _I64, _P]),
    "cbq_huff_tables_bytes": (_I64, [_I64]),
    "cbq_huff_tables_build": (_INT, [_P, _I64, _P, _I64]),
    "cbq_huff_tables_max_len": (_INT, [_P]),
    "cbq_huff_stream_bytes": (_I64, [_I64]),
    "cbq_huff_chunk_count": (_I64, [_I64, _I64]),
    "cbq_huff_chunk_table_words": (_I64, [_I64, _I64]),
    "cbq_huff_chunk_table": (_INT, [_P, _I64, _P, _P, _I64, _I64, _I64, _P, _P, _P]),
    "cbq_huff_decode_lut_bytes": (_I64, []),
    "cbq_huff_build_decode_lut": (_INT, [_P, _P, _I64, _P, _P]),
    "cbq_linear_huff_workspace_bytes": (_I64, [_I64, _I64, _I64]),
    "cbq_linear_huff": (_INT, [_P, _INT, _I64, _I64, _P, _I64, _P, _P, _P, _P, _I64, _P, _I64, _I64,
                               _I64, _P, _P, _INT, _I64, _P, _I64, _P, _P]),
    "cbq_embedding_huff": (_INT, [_P, _I64, _P, _I64, _P, _P, _P, _P, _I64, _I64, _I64, _P, _INT, _P,
                                  _P]),
    "cbq_huff_decode_indices": (_INT, [_P, _I64, _P, _P, _P, _I64, _I64, _P, _P, _P]),
    "cbq_huff_encode": (_INT, [_P, _I64, _P, _P, _P, _P, _I64, _P]),
    "cbq_rmsnorm": (_INT, [_P, _P, _INT, _I64, _I64, _P, ct.c_float, _P, _P]),
    "cbq_rmsnorm_allreduce": (_INT, [_P, _P, _P, _P, _I64, _INT, _INT, _I64, _I64, _P, ct.c_float, _P, _P,
                                     _P]),
    "cbq_greedy_pick": (_INT, [_P, _INT, _I64, _I64, _I64, _INT, _INT, _P, _P, _P, _P, _P, _P]),
    "cbq_qk_norm_rope": (_INT, [_P, _P, _P, _INT, _I64, _I64, _I64, _I64, ct.c_float, _P, _P, _P, _P, _P,
                                _P, _P, _P, _I64, _P]),
    "cbq_attn_decode": (_INT, [_P, _P, _P, _INT, _I64, _I64, _I64, _I64, _I64, _P, ct.c_float, _P, _P]),
    "cbq_attn_decode_rope": (_INT, [_P, _P, _P, _INT, _I64, _I64, _I64, _I64, ct.c_float, _P, _P, _P, _P, _P,
                                    _P, _P, _I64, ct.c_float, _P, _P]),
    "cbq_silu_mul": (_INT, [_P, _P, _INT, _I64, _P, _P]),
    "cbq_attn_workspace_bytes": (_I64, [_I64, _I64, _I64, _I64, _I64]),
    "cbq_attn_decode_rope_split": (_INT, [_P, _P, _P, _INT, _I64, _I64, _I64, _I64, ct.c_float, _P, _P, _P, _P,
                                          _P, _P, _P, _I64, ct.c_float, _P, _P, _I64, _P]),
    "cbq_attn_decode_split": (_INT, [_P, _P, _P, _INT, _I64, _I64, _I64, _I64, _I64, _P, ct.c_float, _P, _P,
                                     _I64, _P]),
}
CBQ_EPI_STORE, CBQ_EPI_RESIDUAL, CBQ_EPI_SILU_MUL = 0, 1, 2


class CbqError(RuntimeError):
    """A libcbq call returned a non-OK status."""

    def __init__(self, fn: str, status: int):
        self.status = status
        super().__init__(f"{fn} failed: {status_string(status)} (status {status})")


def build_library(force: bool = False) -> Path:
    """Compile ``libcbq.so`` for sm_100a with nvcc (no GPU needed)."""
    if force or not LIB_PATH.exists():
        subprocess.run(["make", "-s", "-j3", "-C", str(CSRC)], check=True)
    return LIB_PATH


_lib = None


def lib() -> ct.CDLL:
    """Load the library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C {CSRC}` "
                               "(the CUDA path has no fallback)")
        L = ct.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def status_string(status: int) -> str:
    return lib().cbq_status_string(int(status)).decode()


def call(name: str, *args) -> None:
    rc = getattr(lib(), name)(*args)
    if rc != CBQ_OK:
        raise CbqError(name, rc)


def query(name: str, *args) -> int:
    v = getattr(lib(), name)(*args)
    if v < 0:
        raise CbqError(name, CBQ_ERR_ARG)
    return int(v)
