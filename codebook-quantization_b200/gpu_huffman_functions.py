"""Huffman GPU layers: the B200 replacement of the reference's
``src/gpu_huffman_functions.py`` (``HuffmanCodebookLinear`` :715-866,
``HuffmanCodebookEmbedding`` :869-1002).

The reference's "Phase 2" decodes the whole ``[M, K]`` matrix into an int32
buffer with one thread per row and then runs a separate GEMV over it (and
decodes the entire vocabulary table for every embedding call).  Here:

* load time: the ``huff_stream`` bytes go to a zero-padded device buffer, the
  decode tables are derived from ``huff_lengths`` by ``cbq_huff_tables_build``
  and one ``cbq_huff_chunk_table`` pass records the bit offset of every 64th
  symbol of every row (checked for consistency; a corrupt stream raises);
* call time: one fused decode-GEMV launch (``cbq_linear_huff``) or a
  requested-rows-only embedding decode (``cbq_embedding_huff``).

Row bit offsets are kept as int64 (the reference's CUDA path narrows them to
int32, ``:777-784``, which breaks past 2**31 bits).  The stored 12-bit
``huff_lut_*`` / ``huff_sl_*`` tables are accepted for API compatibility and
not needed: they are a function of ``huff_lengths``.
"""
from __future__ import annotations

from typing import Optional, Tuple

import numpy as np
import torch

from . import _lib
from .gpu_accelerated_functions import (_codebook_f32, _require_cuda, as_kernel_input,
                                        device_stream, padded_device_bytes)

__all__ = ["HuffmanCodebookLinear", "HuffmanCodebookEmbedding", "HuffmanStream", "tables_blob"]


def tables_blob(huff_lengths) -> np.ndarray:
    """Host decode-table blob for ``huff_lengths`` (layout owned by libcbq)."""
    lens = np.ascontiguousarray(np.asarray(huff_lengths, dtype=np.uint8).reshape(-1))
    if lens.size == 0:
        lens = np.zeros(1, dtype=np.uint8)
    nbytes = _lib.query("cbq_huff_tables_bytes", lens.size)
    blob = np.zeros(nbytes, dtype=np.uint8)
    _lib.call("cbq_huff_tables_build", lens.ctypes.data, lens.size, blob.ctypes.data, nbytes)
    return blob


def new_status(device) -> torch.Tensor:
    """Device status word: [flags, first bad row (all ones), count, 0]."""
    return torch.tensor([0, -1, 0, 0], dtype=torch.int32, device=device)


def read_status(status: torch.Tensor) -> Tuple[int, int, int]:
    s = status.cpu().numpy().view(np.uint32)
    return int(s[0]), int(s[1]), int(s[2])


# Token count from which cbq_linear_huff transcodes the stream to fixed width
# and runs the tensor-core GEMM (bf16 activations); the per-device scratch
# that transcode lives in.
PREFILL_TOKENS = 64
_PREFILL_WS = {}


class HuffmanStream:
    """Device-resident Huffman stream of one ``[rows, cols]`` tensor plus the
    derived decode tables and chunk-entry table."""

    def __init__(self, name: str, huff_stream, huff_lengths, huff_n: int, shape,
                 huff_row_bit_starts, device):
        self.name = name
        self.rows, self.cols = (int(s) for s in shape)
        self.device = device
        n = int(huff_n)
        if n != self.rows * self.cols:
            raise ValueError(f"{name}: huff_n={n} does not match shape {shape}")
        if huff_row_bit_starts is None:
            raise NotImplementedError(
                f"{name}: .npz has no huff_row_bit_starts (written by an encoder run without the "
                "weight shape); re-encode it with shape=(M, K)")
        if isinstance(huff_stream, torch.Tensor):
            stream = huff_stream.reshape(-1)
            stream = stream if stream.dtype == torch.uint8 else stream.view(torch.uint8)
            slen = stream.numel()
        else:
            stream = np.ascontiguousarray(np.asarray(huff_stream, dtype=np.uint8).reshape(-1))
            slen = stream.size
        if slen < 4:
            raise ValueError(f"{name}: huff_stream must end with 4 pad bytes")
        self.stream_len = slen
        self.total_bits = 8 * (slen - 4)
        self.nbytes = _lib.query("cbq_huff_stream_bytes", slen)
        self.stream = padded_device_bytes(stream, self.nbytes, device)
        self.lengths = np.asarray(huff_lengths, dtype=np.uint8).reshape(-1)
        self.blob_host = tables_blob(self.lengths)
        self.max_len = _lib.lib().cbq_huff_tables_max_len(self.blob_host.ctypes.data)
        self.tables = torch.from_numpy(self.blob_host).to(device)
        if isinstance(huff_row_bit_starts, torch.Tensor):
            self.rbs = huff_row_bit_starts.reshape(-1).to(device=device, dtype=torch.int64).contiguous()
        else:
            rbs = np.ascontiguousarray(np.asarray(huff_row_bit_starts, dtype=np.int64).reshape(-1))
            self.rbs = torch.from_numpy(rbs).to(device)
        if self.rbs.numel() != self.rows:
            raise ValueError(f"{name}: {self.rbs.numel()} row bit starts for {self.rows} rows")
        self.nchunk = _lib.query("cbq_huff_chunk_count", self.rows, self.cols)
        words = _lib.query("cbq_huff_chunk_table_words", self.rows, self.cols)
        self.chunk = torch.zeros(max(words, 1), dtype=torch.int32, device=device)
        self.status = new_status(device)
        _lib.call("cbq_huff_chunk_table", self.stream.data_ptr(), self.nbytes, self.tables.data_ptr(),
                  self.rbs.data_ptr(), self.rows, self.cols, self.total_bits, self.chunk.data_ptr(),
                  self.status.data_ptr(), device_stream(device))
        flags, row, cnt = read_status(self.status)
        if flags:
            raise _lib.CbqError(f"cbq_huff_chunk_table({name}): flags={flags:#x} first row={row} "
                                f"errors={cnt}", _lib.CBQ_ERR_CORRUPT)

    def check(self) -> None:
        """Raise if any decode since construction hit a corrupt code."""
        flags, row, cnt = read_status(self.status)
        if flags:
            raise _lib.CbqError(f"{self.name}: flags={flags:#x} first row={row} errors={cnt}",
                                _lib.CBQ_ERR_CORRUPT)

    def decode_indices(self) -> torch.Tensor:
        """All indices as a ``[rows, cols]`` int32 tensor (bit-exactness checks)."""
        idx = torch.empty(self.rows * self.cols + 1, dtype=torch.int16, device=self.device)
        _lib.call("cbq_huff_decode_indices", self.stream.data_ptr(), self.nbytes, self.tables.data_ptr(),
                  self.rbs.data_ptr(), self.chunk.data_ptr(), self.rows, self.cols, idx.data_ptr(),
                  self.status.data_ptr(), device_stream(self.device))
        return (idx[:-1].to(torch.int32) & 0xFFFF).reshape(self.rows, self.cols)

    @property
    def compressed_bytes(self) -> int:
        """Algorithmic bytes one full pass reads: stream + row starts + chunk
        table (32-bit chunk offsets and 32-bit packed quarter lengths)."""
        return self.stream_len + 8 * self.rows + 8 * self.nchunk


class HuffmanCodebookLinear:
    """Linear layer over a Huffman-coded index stream (signature of
    ``src/gpu_huffman_functions.py:734-754``)."""

    def __init__(self, name: str, huff_stream, huff_lengths, huff_n: int, codebook, shape: tuple,
                 bits: int, huff_row_bit_starts=None, huff_lut_sym=None, huff_lut_len=None,
                 huff_sl_first_code=None, huff_sl_base_offset=None, huff_sl_sym=None, device=None):
        self.name = name
        self.shape = tuple(int(s) for s in shape)
        self.M, self.K = self.shape
        self.bits = int(bits)
        if device is None and isinstance(codebook, torch.Tensor) and codebook.is_cuda:
            device = codebook.device
        self.device = _require_cuda(device)
        self.codebook = _codebook_f32(codebook, self.device)
        self.C = self.codebook.numel()
        self.hs = HuffmanStream(name, huff_stream, huff_lengths, huff_n, self.shape,
                                huff_row_bit_starts, self.device)
        self.status = self.hs.status
        nl = _lib.query("cbq_huff_decode_lut_bytes")
        self.lut = torch.zeros(nl // 4, dtype=torch.int32, device=self.device)
        _lib.call("cbq_huff_build_decode_lut", self.hs.tables.data_ptr(), self.codebook.data_ptr(), self.C,
                  self.lut.data_ptr(), device_stream(self.device))
        self._ws = {}

    def workspace(self, T: int) -> torch.Tensor:
        """Zero-filled workspace for T-token calls (the kernels leave it zeroed).
        From 64 tokens it also holds the fixed-width transcode the tensor-core
        GEMM reads (2 bytes per weight at most); that buffer is one per device,
        shared by every layer, so such calls on one device must share a stream."""
        if T >= PREFILL_TOKENS:
            n = _lib.query("cbq_linear_huff_workspace_bytes", self.M, self.K, int(T))
            buf = _PREFILL_WS.get(self.device)
            if buf is None or buf.numel() < n:
                buf = torch.zeros(max(n, 16), dtype=torch.uint8, device=self.device)
                _PREFILL_WS[self.device] = buf
            return buf
        key = min(int(T), 8)
        ws = self._ws.get(key)
        if ws is None:
            n = _lib.query("cbq_linear_huff_workspace_bytes", self.M, self.K, key)
            ws = torch.zeros(max(n, 16), dtype=torch.uint8, device=self.device)
            self._ws[key] = ws
        return ws

    def __call__(self, x: torch.Tensor, bias: torch.Tensor = None, out: torch.Tensor = None,
                 out_dtype: torch.dtype = None) -> torch.Tensor:
        if x.shape[-1] != self.K:
            raise ValueError(f"{self.name}: expected last dim {self.K}, got {tuple(x.shape)}")
        if x.device != self.device:
            x = x.to(self.device)
        lead = x.shape[:-1]
        x2, xcode = as_kernel_input(x, self.K)
        T = x2.shape[0]
        want = out_dtype or x.dtype
        kdt = want if want in (torch.float32, torch.bfloat16) else torch.float32
        if out is None:
            out = torch.empty((T, self.M), dtype=kdt, device=self.device)
        ocode = _lib.CBQ_BF16 if out.dtype == torch.bfloat16 else _lib.CBQ_F32
        b = None if bias is None else bias.to(device=self.device, dtype=torch.float32).contiguous()
        hs = self.hs
        ws = self.workspace(T)
        _lib.call("cbq_linear_huff", x2.data_ptr(), xcode, T, x2.stride(0) if T > 1 else self.K,
                  hs.stream.data_ptr(), hs.nbytes, hs.tables.data_ptr(), self.lut.data_ptr(),
                  hs.rbs.data_ptr(), hs.chunk.data_ptr(), hs.total_bits, self.codebook.data_ptr(), self.C,
                  self.M, self.K, None if b is None else b.data_ptr(), out.data_ptr(), ocode,
                  out.stride(0) if T > 1 else self.M, ws.data_ptr(), ws.numel(), hs.status.data_ptr(),
                  device_stream(self.device))
        res = out.reshape(*lead, self.M)
        return res if res.dtype == want else res.to(want)


class HuffmanCodebookEmbedding:
    """Embedding over a Huffman-coded table (signature of
    ``src/gpu_huffman_functions.py:877-893``); decodes only requested rows."""

    def __init__(self, name: str, huff_stream, huff_lengths, huff_n: int, codebook, shape: tuple,
                 bits: int, huff_row_bit_starts=None, huff_lut_sym=None, huff_lut_len=None,
                 huff_sl_first_code=None, huff_sl_base_offset=None, huff_sl_sym=None, device=None):
        self.name = name
        self.shape = tuple(int(s) for s in shape)
        self.vocab, self.hidden = self.shape
        self.bits = int(bits)
        if device is None and isinstance(codebook, torch.Tensor) and codebook.is_cuda:
            device = codebook.device
        self.device = _require_cuda(device)
        self.codebook = _codebook_f32(codebook, self.device)
        self.C = self.codebook.numel()
        self.hs = HuffmanStream(name, huff_stream, huff_lengths, huff_n, self.shape,
                                huff_row_bit_starts, self.device)
        self.status = self.hs.status

    def __call__(self, ids: torch.Tensor, out_dtype: torch.dtype = torch.float32,
                 out: torch.Tensor = None) -> torch.Tensor:
        lead = ids.shape
        flat = ids.reshape(-1).to(device=self.device, dtype=torch.int64).contiguous()
        T = flat.numel()
        if out is not None:
            out_dtype = out.dtype
        kdt = out_dtype if out_dtype in (torch.float32, torch.bfloat16) else torch.float32
        if out is None or out.dtype != kdt or not out.is_contiguous():
            out = torch.empty((T, self.hidden), dtype=kdt, device=self.device)
        hs = self.hs
        _lib.call("cbq_embedding_huff", flat.data_ptr(), T, hs.stream.data_ptr(), hs.nbytes,
                  hs.tables.data_ptr(), hs.rbs.data_ptr(), hs.chunk.data_ptr(), self.codebook.data_ptr(),
                  self.C, self.vocab, self.hidden, out.data_ptr(),
                  _lib.CBQ_BF16 if kdt == torch.bfloat16 else _lib.CBQ_F32, hs.status.data_ptr(),
                  device_stream(self.device))
        res = out.reshape(*lead, self.hidden)
        return res if res.dtype == out_dtype else res.to(out_dtype)
