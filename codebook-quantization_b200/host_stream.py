"""Host-resident packed streams: flat ``.idx`` files, their memory maps, and a
linear layer whose stream stays in host memory and is streamed to the GPU
per call.

The reference's path for models whose packed indices do not fit in memory
(``README.md:8-9``): ``export_flat_idx`` writes each tensor's raw
``indices`` bytes to ``<name>.idx`` next to its ``.npz``
(``src/adaptive_compressor.py:1254-1316``), ``MmappedPackedBuffer`` maps such
a file read-only (``src/compressed_matmul_cpu.py:23-63``) and the CPU kernel
reads the mapping, so the OS pages the stream in on demand.

Here the same files and the same ``MmappedPackedBuffer`` interface feed
:class:`HostStreamedLinear`: the mapping (or any host array) is page-locked
once (``cbq_host_register``) and every call copies it to the device in row
chunks through a two-buffer staging area while the previous chunk's GEMV
runs (``cbq_linear_fixed_streamed``), so device memory holds only the
staging buffers and the call runs at the host link's bandwidth.
"""
from __future__ import annotations

import mmap
from pathlib import Path

import numpy as np
import torch

from . import _lib
from .gpu_accelerated_functions import _codebook_f32, _require_cuda, as_kernel_input, device_stream

__all__ = ["MmappedPackedBuffer", "export_flat_idx", "HostStreamedLinear"]


class MmappedPackedBuffer:
    """Read-only mmap of a flat ``.idx`` file (raw uint8 bytes); ``as_numpy()``
    is a zero-copy uint8 view, so opening the file reads nothing."""

    def __init__(self, path):
        self.path = Path(path)
        self._f = open(self.path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self._arr = np.frombuffer(self._mm, dtype=np.uint8)

    def as_numpy(self) -> np.ndarray:
        return self._arr

    def __len__(self) -> int:
        return 0 if self._arr is None else len(self._arr)

    def close(self) -> None:
        self._arr = None
        if self._mm is not None:
            try:
                self._mm.close()
            except BufferError:               # views still alive; the OS unmaps when they go
                pass
            self._mm = None
        if self._f is not None:
            self._f.close()
            self._f = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def export_flat_idx(model_dir, tensors_subdir: str = "codebook-lossless/tensors", verbose: bool = False) -> int:
    """Write ``<name>.idx`` (the raw ``indices`` bytes) next to every fixed-width
    ``.npz`` under ``model_dir/tensors_subdir`` that has none yet; returns the
    number written."""
    tdir = Path(model_dir) / tensors_subdir
    if not tdir.exists():
        raise FileNotFoundError(f"tensors directory not found: {tdir}")
    written = 0
    for npz in sorted(tdir.glob("*.npz")):
        idx = npz.with_suffix(".idx")
        if idx.exists():
            continue
        with np.load(npz) as z:
            if "indices" not in z.files:
                continue
            np.asarray(z["indices"], dtype=np.uint8).tofile(idx)
        written += 1
        if verbose:
            print(f"{npz.stem}: {idx.stat().st_size / 1024:.0f} KB -> {idx.name}")
    return written


class HostStreamedLinear:
    """Fixed-width linear layer whose packed stream stays in host memory.

    ``indices``: a host uint8 array, an :class:`MmappedPackedBuffer` or a path
    to an ``.idx`` file.  A mapping is page-locked in place (read-only); any
    other array is copied once into pinned memory.  ``staging_bytes`` of
    device memory hold two row chunks.  Same call signature as
    ``GPUAcceleratedLinear``; K must be a multiple of 128.
    """

    def __init__(self, name: str, indices, codebook, shape: tuple, bits: int, device=None,
                 staging_bytes: int = 64 << 20):
        self.name = name
        self.shape = tuple(int(s) for s in shape)
        self.M, self.K = self.shape
        self.bits = int(bits)
        self.device = _require_cuda(device)
        self.codebook = _codebook_f32(codebook, self.device)
        self.C = self.codebook.numel()
        self.nbytes = (self.M * self.K * self.bits + 7) // 8
        if isinstance(indices, (str, Path)):
            indices = MmappedPackedBuffer(indices)
        self._buf = indices if isinstance(indices, MmappedPackedBuffer) else None
        self._registered = None
        self._pinned = None
        torch.cuda.set_device(self.device)
        if self._buf is not None:
            arr = self._buf.as_numpy()
            if arr.size < self.nbytes:
                raise ValueError(f"{name}: {arr.size}-byte .idx file, needs {self.nbytes}")
            rc = _lib.lib().cbq_host_register(arr.ctypes.data, arr.size, 1)
            if rc == _lib.CBQ_OK:
                self._registered = arr.ctypes.data
                self.host_ptr = arr.ctypes.data
            else:                                       # read-only registration unavailable: pinned copy
                self._pinned = torch.from_numpy(np.array(arr[:self.nbytes])).pin_memory()
                self.host_ptr = self._pinned.data_ptr()
        else:
            arr = np.ascontiguousarray(np.asarray(indices).reshape(-1).view(np.uint8))
            if arr.size < self.nbytes:
                raise ValueError(f"{name}: packed stream has {arr.size} bytes, needs {self.nbytes}")
            self._pinned = torch.from_numpy(arr[:self.nbytes].copy()).pin_memory()
            self.host_ptr = self._pinned.data_ptr()
        self.chunk_rows = _lib.query("cbq_streamed_chunk_rows", self.M, self.K, self.bits, int(staging_bytes))
        self.staging = torch.empty(int(staging_bytes), dtype=torch.uint8, device=self.device)
        self._ws = {}

    def workspace(self, T: int) -> torch.Tensor:
        key = min(int(T), 8)
        ws = self._ws.get(key)
        if ws is None:
            n = _lib.query("cbq_linear_fixed_workspace_bytes", self.chunk_rows, self.K, key)
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
        ws = self.workspace(T)
        _lib.call("cbq_linear_fixed_streamed", x2.data_ptr(), xcode, T, x2.stride(0) if T > 1 else self.K,
                  self.host_ptr, self.nbytes, self.codebook.data_ptr(), self.C, self.bits, self.M, self.K,
                  None if b is None else b.data_ptr(), out.data_ptr(), ocode, out.stride(0) if T > 1 else self.M,
                  self.staging.data_ptr(), self.staging.numel(), ws.data_ptr(), ws.numel(),
                  device_stream(self.device))
        res = out.reshape(*lead, self.M)
        return res if res.dtype == want else res.to(want)

    def close(self) -> None:
        """Unregister the page-locked mapping (after the device work that reads it)."""
        if self._registered is not None:
            torch.cuda.synchronize(self.device)
            _lib.lib().cbq_host_unregister(self._registered)
            self._registered = None
        self._pinned = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
