"""``AdaptiveCodebookLinear`` / ``AdaptiveCodebookEmbedding``: the drop-in module
API of the reference (``src/compressed_modules.py:48-490``) over the B200
kernels.

Kept from the reference: class names, constructor ``(name, shape, mode)``,
``from_compressed(name, data, global_codebooks, use_gpu=True, use_mmap=False,
idx_file=None)``, the ``data`` dict keys of an ``.npz`` tensor, codebook
priority (local ``codebook`` key first, then ``global_codebooks[codebook_type]``,
``:183-196``), ``forward`` semantics (input ``[*, K]`` of any float dtype,
output ``[*, M]`` in ``x.dtype``, ``+ bias``), the inspected attributes
(``bits``, ``codebook``, ``indices``, ``bias``, ``_gpu_func``, ``_huff_data``)
and the embedding's ``embed_scale`` and output dtype (the codebook buffer's).

Changed on purpose: ``direct_codebook`` tensors always run on the GPU through
``libcbq``.  There is no CPU or decode-at-load fallback: ``use_gpu=False`` or a
missing CUDA device raises instead of silently switching path.  ``use_mmap``
with an existing ``idx_file`` (a flat ``.idx`` of the packed indices) keeps a
fixed-width stream in host memory -- the mapped file, page-locked -- and
streams it to the GPU on every forward (``HostStreamedLinear``), where the
reference runs its CPU kernel on the mapping (``:137-140``, ``:268-274``);
otherwise the stream is copied to device memory, as the reference's GPU path
does (``:265-267``).
"""
from __future__ import annotations

from pathlib import Path
from typing import Tuple

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from .gpu_accelerated_functions import GPUAcceleratedEmbedding, GPUAcceleratedLinear
from .gpu_huffman_functions import HuffmanCodebookEmbedding, HuffmanCodebookLinear

__all__ = ["AdaptiveCodebookLinear", "AdaptiveCodebookEmbedding"]

_HUFF_TABLE_KEYS = ("huff_row_bit_starts", "huff_lut_sym", "huff_lut_len", "huff_sl_first_code",
                    "huff_sl_base_offset", "huff_sl_sym")


def _exact_weight(data: dict, shape) -> torch.Tensor:
    raw = data["data"]
    if raw.dtype == np.uint16:                       # bf16 bit patterns
        w = (raw.astype(np.uint32) << 16).view(np.float32)
    else:
        w = raw.astype(np.float32)
    return torch.from_numpy(np.ascontiguousarray(w).reshape(tuple(int(s) for s in shape)))


def _select_codebook(data: dict, global_codebooks: dict, default_type=None):
    """Local per-tensor codebook first, then the category's global codebook."""
    cb = data.get("codebook")
    if cb is not None and np.asarray(cb).size > 0:
        return torch.as_tensor(np.asarray(cb)).float()
    ttype = data.get("codebook_type") or data.get("type") or default_type
    if ttype and global_codebooks and ttype in global_codebooks:
        g = global_codebooks[ttype]
        return (g if isinstance(g, torch.Tensor) else torch.from_numpy(np.asarray(g))).float()
    return None


def _gpu_device(use_gpu: bool, name: str, device):
    if not use_gpu:
        raise RuntimeError(f"{name}: direct_codebook layers run only on the GPU (use_gpu=False has "
                           "no CPU path in this build)")
    if not torch.cuda.is_available():
        raise RuntimeError(f"{name}: no CUDA device; the codebook kernels have no CPU fallback")
    return device


class AdaptiveCodebookLinear(nn.Module):
    """Linear layer whose weight stays compressed (``src/compressed_modules.py:48``)."""

    def __init__(self, name: str, shape: Tuple[int, ...], mode: str = "exact"):
        super().__init__()
        self.name = name
        self.shape = tuple(int(s) for s in shape)
        self.mode = mode
        self.register_buffer("bias", None, persistent=False)
        self.register_buffer("indices", None, persistent=False)
        self.register_buffer("codebook", None, persistent=False)
        self.register_buffer("weight", None, persistent=False)
        self.register_buffer("scale", None, persistent=False)
        self.register_buffer("v_min", None, persistent=False)
        self.bits = 8
        self._gpu_func = None
        self._huff_data = None
        self._mmap_buf = None   # MmappedPackedBuffer of the .idx file when use_mmap=True

    @property
    def in_features(self) -> int:
        return self.shape[1]

    @property
    def out_features(self) -> int:
        return self.shape[0]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.mode == "exact":
            w = self.weight if self.weight.dtype == x.dtype else self.weight.to(x.dtype)
            return F.linear(x, w, self.bias)
        if self.mode == "direct_codebook":
            if self._gpu_func is None:
                raise RuntimeError(f"{self.name}: direct_codebook layer has no GPU kernel bound")
            return self._gpu_func(x, bias=self.bias)
        if self.mode == "linear_quant":
            w = (self.indices.float() * self.scale + self.v_min).reshape(self.shape)
            return F.linear(x, w.to(x.dtype), self.bias)
        raise ValueError(f"Unsupported mode: {self.mode}")

    @classmethod
    def from_compressed(cls, name: str, data: dict, global_codebooks: dict, use_gpu: bool = True,
                        use_mmap: bool = False, idx_file=None, device=None):
        """Build from an ``.npz`` tensor dict (``src/compressed_modules.py:167-296``)."""
        mode = data["mode"]
        shape = tuple(int(s) for s in np.asarray(data["shape"]).reshape(-1))
        layer = cls(name, shape, mode)
        layer.bits = int(data.get("bits", 8))
        if mode == "exact":
            layer.weight = nn.Parameter(_exact_weight(data, shape), requires_grad=False)
        elif mode == "direct_codebook":
            cb = _select_codebook(data, global_codebooks)
            if cb is None:
                raise ValueError(f"{name}: no local codebook and no global codebook for "
                                 f"{data.get('codebook_type')!r}")
            layer.register_buffer("codebook", cb, persistent=False)
            device = _gpu_device(use_gpu, name, device)
            if data.get("encoding") == "huffman":
                layer._gpu_func = HuffmanCodebookLinear(
                    name, data["huff_stream"], data["huff_lengths"], int(np.asarray(data["huff_n"])[0]),
                    cb, shape, layer.bits, device=device,
                    **{k: data.get(k) for k in _HUFF_TABLE_KEYS})
            elif use_mmap and idx_file is not None and Path(idx_file).exists():
                from .host_stream import HostStreamedLinear, MmappedPackedBuffer
                layer._mmap_buf = MmappedPackedBuffer(idx_file)
                layer._gpu_func = HostStreamedLinear(name, layer._mmap_buf, cb, shape, layer.bits, device=device)
            else:
                layer._gpu_func = GPUAcceleratedLinear(name, data["indices"], cb, shape, layer.bits,
                                                       device=device)
            layer.register_buffer("indices", None)
        elif mode == "linear_quant":
            layer.register_buffer("indices", torch.from_numpy(np.asarray(data["indices"])))
            layer.register_buffer("scale", torch.tensor(data["scale"], dtype=torch.float32))
            layer.register_buffer("v_min", torch.tensor(data["v_min"], dtype=torch.float32))
        else:
            raise ValueError(f"Unsupported mode: {mode}")
        return layer


class AdaptiveCodebookEmbedding(nn.Module):
    """Embedding whose table stays compressed (``src/compressed_modules.py:298``)."""

    def __init__(self, name: str, shape: Tuple[int, ...], mode: str = "exact"):
        super().__init__()
        self.name = name
        self.shape = tuple(int(s) for s in shape)
        self.mode = mode
        self.register_buffer("indices", None, persistent=False)
        self.register_buffer("codebook", None, persistent=False)
        self.register_buffer("weight", None, persistent=False)
        self.bits = 8
        self._gpu_func = None
        self._huff_data = None
        self.embed_scale: float = 1.0

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.mode == "exact":
            out = F.embedding(x, self.weight)
            return out * self.embed_scale if self.embed_scale != 1.0 else out
        if self.mode == "direct_codebook":
            if self._gpu_func is None:
                raise RuntimeError(f"{self.name}: direct_codebook embedding has no GPU kernel bound")
            target = self.codebook.dtype if self.codebook is not None else torch.bfloat16
            out = self._gpu_func(x, out_dtype=target)
            return out * self.embed_scale if self.embed_scale != 1.0 else out
        raise ValueError(f"Unsupported mode: {self.mode}")

    @classmethod
    def from_compressed(cls, name: str, data: dict, global_codebooks: dict, use_gpu: bool = True,
                        use_mmap: bool = False, idx_file=None, device=None):
        """Build from an ``.npz`` tensor dict (``src/compressed_modules.py:378-490``)."""
        mode = data["mode"]
        shape = tuple(int(s) for s in np.asarray(data["shape"]).reshape(-1))
        layer = cls(name, shape, mode)
        layer.bits = int(data.get("bits", 8))
        if mode == "exact":
            layer.weight = nn.Parameter(_exact_weight(data, shape), requires_grad=False)
        elif mode == "direct_codebook":
            cb = _select_codebook(data, global_codebooks, default_type="embedding")
            if cb is None:
                raise ValueError(f"{name}: no codebook available")
            layer.register_buffer("codebook", cb, persistent=False)
            device = _gpu_device(use_gpu, name, device)
            if data.get("encoding") == "huffman":
                layer._gpu_func = HuffmanCodebookEmbedding(
                    name, data["huff_stream"], data["huff_lengths"], int(np.asarray(data["huff_n"])[0]),
                    cb, shape, layer.bits, device=device,
                    **{k: data.get(k) for k in _HUFF_TABLE_KEYS})
            else:
                layer._gpu_func = GPUAcceleratedEmbedding(name, data["indices"], cb, shape, layer.bits,
                                                          device=device)
            layer.register_buffer("indices", None)
        else:
            raise ValueError(f"Unsupported mode: {mode}")
        return layer
