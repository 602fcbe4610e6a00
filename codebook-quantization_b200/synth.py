"""Seeded synthetic compressed tensors for the BASELINE configurations.

There are no checkpoints on the GPU hosts, so weights are drawn N(0, std) in
fp32 and truncated to bf16 (the reference's ``float32_to_bfloat16``,
``src/compressor.py:28-34``), then compressed losslessly the way the
reference's fast lossless path does (``src/adaptive_compressor.py:85-136``):
the codebook is the set of distinct bf16 values (here sorted by descending
frequency, ties by bit pattern, as BASELINE asks; the format is
order-agnostic), each weight becomes its value's index, ``bits =
ceil(log2(max(C, 2)))``, and the indices are either packed fixed-width or
Huffman-coded on their own frequencies.

Two generators:

* numpy (``np.random.default_rng(seed)``) for CPU-checkable sizes;
* torch on the GPU (``torch.Generator('cuda').manual_seed(seed)``) for model
  sizes, with packing and Huffman encoding done by ``libcbq``'s device
  encoders (``cbq_pack_fixed``, ``cbq_huff_encode``), so multi-GB models never
  round-trip through host memory.  The two generators give different (equally
  seeded) values.
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import numpy as np
import torch

from . import _lib, bitpack, huffman_codebook as hc
from .gpu_accelerated_functions import device_stream

__all__ = ["bf16_normal_np", "bf16_normal_gpu", "codebook_from_hist", "lossless_indices_np",
           "compress_fixed_np", "compress_huffman_np", "GpuCompressor", "bits_for"]


def bits_for(C: int) -> int:
    """``ceil(log2(max(C, 2)))`` (src/adaptive_compressor.py:109)."""
    return int(math.ceil(math.log2(max(int(C), 2))))


# ------------------------------------------------------------------ numpy side

def bf16_normal_np(shape, seed: int, std: float = 0.02) -> np.ndarray:
    """bf16 bit patterns (uint16) of ``bf16(N(0,1) * std)`` by truncation."""
    rng = np.random.default_rng(seed)
    w = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
    return (w.view(np.uint32) >> 16).astype(np.uint16)


def codebook_from_hist(hist: np.ndarray, order: str = "frequency"):
    """Codebook (fp32) and bf16-pattern -> index LUT from a 65536-bin histogram."""
    vals = np.flatnonzero(hist)
    if order == "frequency":
        vals = vals[np.lexsort((vals, -hist[vals]))]
    elif order != "bitpattern":
        raise ValueError(order)
    lut = np.zeros(65536, dtype=np.uint16)
    lut[vals] = np.arange(vals.size, dtype=np.uint16)
    cb = (vals.astype(np.uint32) << 16).view(np.float32).astype(np.float32)
    return cb, lut


def lossless_indices_np(bf: np.ndarray, order: str = "frequency"):
    hist = np.bincount(bf.reshape(-1), minlength=65536)
    cb, lut = codebook_from_hist(hist, order)
    return cb, lut[bf]


def compress_fixed_np(bf: np.ndarray, codebook=None, lut=None, codebook_type="mlp_ffn") -> dict:
    """``direct_codebook`` fixed-width tensor dict from bf16 patterns [M, K]."""
    if codebook is None:
        codebook, idx = lossless_indices_np(bf)
    else:
        idx = lut[bf]
    bits = bits_for(len(codebook))
    return {"mode": "direct_codebook", "shape": np.array(bf.shape), "bits": bits,
            "codebook": codebook, "codebook_type": codebook_type,
            "indices": bitpack.pack_any_bits(idx.reshape(-1), bits), "_idx": idx}


def compress_huffman_np(bf: np.ndarray, codebook=None, lut=None, codebook_type="mlp_ffn") -> dict:
    """``direct_codebook`` Huffman tensor dict from bf16 patterns [M, K]."""
    if codebook is None:
        codebook, idx = lossless_indices_np(bf)
    else:
        idx = lut[bf]
    enc = hc.huffman_encode_indices(idx.reshape(-1), shape=bf.shape)
    d = {"mode": "direct_codebook", "shape": np.array(bf.shape), "bits": bits_for(len(codebook)),
         "codebook": codebook, "codebook_type": codebook_type, "encoding": "huffman", "_idx": idx}
    d.update(enc)
    return d


# ------------------------------------------------------------------ GPU side

def bf16_normal_gpu(shape, seed: int, device, std: float = 0.02) -> torch.Tensor:
    """bf16 bit patterns as int32 in [0, 65536), generated on ``device``."""
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    w = torch.randn(tuple(shape), generator=g, device=device, dtype=torch.float32) * std
    return (w.view(torch.int32) >> 16) & 0xFFFF


class GpuCompressor:
    """Lossless compression of bf16 tensors on one GPU.

    Per-tensor codebooks by default; ``shared_codebook(hist)`` installs one
    codebook per category (the reference's ``codebooks/<type>_codebook.npy``).
    """

    def __init__(self, device):
        self.device = torch.device(device)

    def histogram(self, bits: torch.Tensor) -> torch.Tensor:
        return torch.bincount(bits.reshape(-1).long(), minlength=65536)

    def codebook(self, hist: torch.Tensor):
        """(codebook fp32 [C] on device, LUT int64 [65536] on device)."""
        vals = torch.nonzero(hist, as_tuple=False).reshape(-1)
        cnt = hist[vals]
        key = (cnt.max() - cnt) * 65536 + vals        # descending count, then pattern
        vals = vals[torch.argsort(key)]
        lut = torch.zeros(65536, dtype=torch.int64, device=self.device)
        lut[vals] = torch.arange(vals.numel(), device=self.device)
        cb = (vals.to(torch.int32) << 16).view(torch.float32).contiguous()
        return cb, lut

    def indices(self, bits: torch.Tensor, lut: torch.Tensor) -> torch.Tensor:
        """uint16 indices stored in an int16 tensor."""
        return lut[bits.long()].to(torch.int32).to(torch.int16)

    def pack_fixed(self, idx16: torch.Tensor, nbits: int) -> torch.Tensor:
        n = idx16.numel()
        nbytes = (n * nbits + 7) // 8
        out = torch.zeros(((nbytes + 3) // 4) * 4, dtype=torch.uint8, device=self.device)
        _lib.call("cbq_pack_fixed", idx16.data_ptr(), n, nbits, out.data_ptr(), out.numel(),
                  device_stream(self.device))
        return out[:nbytes]

    def huffman(self, idx16: torch.Tensor, shape) -> Dict[str, object]:
        """Huffman-encode on the device; stream and row starts stay on the GPU,
        the small tables come back as numpy arrays (``.npz`` dtypes)."""
        M, K = (int(s) for s in shape)
        idx = idx16.reshape(-1)
        n = idx.numel()
        idx_l = idx.to(torch.int64) & 0xFFFF
        A = int(idx_l.max().item()) + 1 if n else 1
        freq = torch.bincount(idx_l, minlength=A).cpu().numpy()
        lengths = hc.code_lengths(freq)
        codes, _ = hc.canonical_codes(lengths)
        code_d = torch.from_numpy(codes.astype(np.uint32).view(np.int32)).to(self.device)
        len_d = torch.from_numpy(lengths.astype(np.uint8)).to(self.device)
        sym_len = len_d[idx_l].to(torch.int64)
        starts = torch.cumsum(sym_len, 0) - sym_len
        total = int((starts[-1] + sym_len[-1]).item()) if n else 0
        nbytes = (total + 7) // 8
        out = torch.empty(((nbytes + 3) // 4) * 4 + 8, dtype=torch.uint8, device=self.device)
        _lib.call("cbq_huff_encode", idx.data_ptr(), n, code_d.data_ptr(), len_d.data_ptr(),
                  starts.data_ptr(), out.data_ptr(), out.numel(), device_stream(self.device))
        stream = torch.zeros(nbytes + 4, dtype=torch.uint8, device=self.device)
        stream[:nbytes].copy_(out[:nbytes])
        rbs = starts[::K].contiguous() if (n and M * K == n) else torch.zeros(max(M, 1), dtype=torch.int64,
                                                                               device=self.device)
        d = {"huff_lengths": lengths, "huff_stream": stream, "huff_n": np.array([n], dtype=np.int64),
             "huff_row_bit_starts": rbs}
        d["huff_lut_sym"], d["huff_lut_len"] = hc.build_gpu_lut(lengths)
        (d["huff_sl_first_code"], d["huff_sl_base_offset"],
         d["huff_sl_sym"]) = hc.build_slow_path_tables(lengths)
        return d

    def compress(self, bits: torch.Tensor, huffman: bool, codebook=None, lut=None,
                 codebook_type: str = "mlp_ffn", keep_codebook: bool = True) -> dict:
        """Tensor dict (device-resident payload) for bf16 patterns ``bits [M, K]``."""
        if codebook is None:
            codebook, lut = self.codebook(self.histogram(bits))
        idx16 = self.indices(bits, lut)
        nb = bits_for(codebook.numel())
        d = {"mode": "direct_codebook", "shape": np.array(tuple(bits.shape)), "bits": nb,
             "codebook_type": codebook_type}
        if keep_codebook:
            d["codebook"] = codebook
        if huffman:
            d["encoding"] = "huffman"
            d.update(self.huffman(idx16, bits.shape))
        else:
            d["indices"] = self.pack_fixed(idx16, nb)
        return d
