"""Fixed-width GPU layers: the B200 replacement of the reference's
``src/gpu_accelerated_functions.py`` (``GPUAcceleratedLinear`` :871-950,
``GPUAcceleratedEmbedding`` :953-1029).

The reference JIT-compiles an inline CUDA string on first use and launches a
one-block-per-output kernel on the default stream, with a cast, a memset and a
cast-back around it (4 launches per call).  Here each call is one launch of the
prebuilt sm_100a kernel in ``libcbq.so`` on the caller's current stream,
reading fp32 or bf16 activations directly and writing the output dtype
directly.

Device memory: the packed stream is copied once into a zero-padded, 16-byte
aligned buffer of ``cbq_fixed_stream_bytes(M, K, bits)`` bytes (the reference
pads +4 bytes, ``:860-864``) and the codebook is kept as fp32.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib

__all__ = ["GPUAcceleratedLinear", "GPUAcceleratedEmbedding", "device_stream", "as_kernel_input",
           "linear_fixed_multi"]


def device_stream(device: torch.device) -> int:
    """Raw cudaStream_t of torch's current stream on ``device``."""
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(device) -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("codebook kernels need a CUDA device; there is no CPU fallback")
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.type != "cuda":
        raise RuntimeError(f"codebook kernels run on CUDA devices only, got {dev}")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return dev


def as_kernel_input(x: torch.Tensor, K: int):
    """Flatten ``x [*, K]`` to ``[T, K]`` in a dtype the kernels read (fp32/bf16)."""
    x2 = x.reshape(-1, K)
    if x2.dtype not in (torch.float32, torch.bfloat16):
        x2 = x2.float()
    if x2.stride(-1) != 1 or (x2.shape[0] > 1 and x2.stride(0) < K):
        x2 = x2.contiguous()
    code = _lib.CBQ_BF16 if x2.dtype == torch.bfloat16 else _lib.CBQ_F32
    return x2, code


def padded_device_bytes(data, nbytes: int, device: torch.device) -> torch.Tensor:
    """Copy a byte stream (host array or CUDA uint8 tensor) into a zero-filled
    device buffer of ``nbytes`` bytes."""
    buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
    if isinstance(data, torch.Tensor):
        src = data.reshape(-1)
        if src.dtype != torch.uint8:
            src = src.view(torch.uint8)
        if src.numel() > nbytes:
            raise ValueError(f"stream of {src.numel()} bytes exceeds its {nbytes}-byte buffer")
        buf[:src.numel()].copy_(src)
        return buf
    host = np.ascontiguousarray(np.asarray(data, dtype=np.uint8).reshape(-1))
    if host.size > nbytes:
        raise ValueError(f"stream of {host.size} bytes exceeds its {nbytes}-byte buffer")
    if host.size:
        buf[:host.size].copy_(torch.from_numpy(host))
    return buf


def _codebook_f32(codebook, device) -> torch.Tensor:
    cb = codebook if isinstance(codebook, torch.Tensor) else torch.from_numpy(np.asarray(codebook))
    cb = cb.detach().reshape(-1).to(device=device, dtype=torch.float32).contiguous()
    if cb.numel() < 1:
        raise ValueError("empty codebook")
    return cb


def _stream_prefix(indices, need: int, name: str):
    """The first ``need`` bytes of a packed stream given as an array or tensor."""
    if isinstance(indices, torch.Tensor):
        flat = indices.reshape(-1)
        flat = flat if flat.dtype == torch.uint8 else flat.view(torch.uint8)
    else:
        flat = np.asarray(indices).reshape(-1).view(np.uint8)
    n = flat.numel() if isinstance(flat, torch.Tensor) else flat.size
    if n < need:
        raise ValueError(f"{name}: packed stream has {n} bytes, needs {need}")
    return flat[:need]


class GPUAcceleratedLinear:
    """Packed fixed-width indices resident on the GPU; ``__call__`` runs the
    fused decode-GEMV.  Never materialises the weight matrix.

    ``indices_np`` is the ``.npz`` ``indices`` array (uint8 LSB-first stream),
    a host array or a CUDA uint8 tensor already holding the stream.
    """

    def __init__(self, name: str, indices_np, codebook, shape: tuple, bits: int, device=None):
        self.name = name
        self.shape = tuple(int(s) for s in shape)
        self.M, self.K = self.shape
        self.bits = int(bits)
        if not 1 <= self.bits <= 16:
            raise ValueError(f"{name}: bits must be in [1, 16], got {bits}")
        if device is None and isinstance(codebook, torch.Tensor) and codebook.is_cuda:
            device = codebook.device
        self.device = _require_cuda(device)
        self.codebook = _codebook_f32(codebook, self.device)
        self.C = self.codebook.numel()
        self.nbytes = _lib.query("cbq_fixed_stream_bytes", self.M, self.K, self.bits)
        need = (self.M * self.K * self.bits + 7) // 8
        self.packed = padded_device_bytes(_stream_prefix(indices_np, need, name), self.nbytes,
                                          self.device)
        self._ws = {}                      # token-block size -> zero-filled workspace

    def workspace(self, T: int) -> torch.Tensor:
        """Zero-filled workspace for T-token calls (the kernels leave it zeroed);
        3..63 tokens size it for the split-K tensor-core path too."""
        key = int(T) if 3 <= int(T) < 64 else min(int(T), 8)
        ws = self._ws.get(key)
        if ws is None:
            n = _lib.query("cbq_linear_fixed_workspace_bytes", self.M, self.K, key)
            ws = torch.zeros(max(n, 16), dtype=torch.uint8, device=self.device)
            self._ws[key] = ws
        return ws

    def __call__(self, x: torch.Tensor, bias: torch.Tensor = None, out: torch.Tensor = None,
                 out_dtype: torch.dtype = None) -> torch.Tensor:
        """``x [..., K]`` (any float dtype) -> ``[..., M]`` in ``x.dtype``
        (or ``out_dtype``), ``+ bias`` fused when given (fp32 ``[M]``)."""
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
        b = None
        if bias is not None:
            b = bias.to(device=self.device, dtype=torch.float32).contiguous()
        ws = self.workspace(T)
        _lib.call("cbq_linear_fixed", x2.data_ptr(), xcode, T, x2.stride(0) if T > 1 else self.K,
                  self.packed.data_ptr(), self.nbytes, self.codebook.data_ptr(), self.C, self.bits,
                  self.M, self.K, None if b is None else b.data_ptr(), out.data_ptr(), ocode,
                  out.stride(0) if T > 1 else self.M, ws.data_ptr(), ws.numel(),
                  device_stream(self.device))
        res = out.reshape(*lead, self.M)
        return res if res.dtype == want else res.to(want)


def linear_fixed_multi(mats, x: torch.Tensor, outs, epilogue: int = 0, resids=None, norm=None,
                       allreduce=None) -> bool:
    """One launch of ``cbq_linear_fixed_multi`` over ``mats`` (GPUAcceleratedLinear
    objects sharing K, bits and codebook) for ``x [T, K]``.  ``outs[i]`` are
    ``[T, M_i]`` tensors (for ``CBQ_EPI_SILU_MUL`` only ``outs[0]`` is
    written); ``resids[i]`` the residual inputs of ``CBQ_EPI_RESIDUAL`` (may be
    ``outs[i]`` itself).  ``norm=(weight or None, eps)``: ``x`` is the
    un-normalised residual stream and the launch applies the RMSNorm as it
    loads it (``cbq_linear_fixed_multi_norm``).  Returns False, having
    launched nothing, when the shape is outside what the fused kernel supports
    (T > 2, unaligned rows); the caller then runs the matrices one by one.
    ``allreduce=(world, resid_in, slots_ptr, counts_ptr, epoch_ptr, expect,
    status_ptr)`` (with ``norm``): ``x`` receives round(resid_in + the
    all-reduced partial rows) before the normalised GEMV reads it
    (``cbq_linear_fixed_multi_allreduce_norm``)."""
    import ctypes as ct
    n = len(mats)
    m0 = mats[0]
    if any(m.K != m0.K or m.bits != m0.bits or m.codebook.data_ptr() != m0.codebook.data_ptr()
           or m.device != m0.device for m in mats):
        raise ValueError("linear_fixed_multi: matrices must share K, bits, codebook and device")
    x2, xcode = as_kernel_input(x, m0.K)
    T = x2.shape[0]
    outs = list(outs)
    if epilogue == _lib.CBQ_EPI_SILU_MUL:
        outs = outs[:1] * n                  # both rows of a pair land in outs[0]
    if len(outs) != n:
        raise ValueError(f"linear_fixed_multi: {n} matrices but {len(outs)} outputs")
    odt = outs[0].dtype
    ocode = _lib.CBQ_BF16 if odt == torch.bfloat16 else _lib.CBQ_F32
    P, I64 = ct.c_void_p, ct.c_int64
    packed = (P * n)(*[m.packed.data_ptr() for m in mats])
    nbytes = (I64 * n)(*[m.nbytes for m in mats])
    Ms = (I64 * n)(*[m.M for m in mats])
    optrs = (P * n)(*[o.data_ptr() for o in outs])
    ldo = (I64 * n)(*[o.stride(0) if o.dim() > 1 and T > 1 else o.shape[-1] for o in outs])
    rp = None if resids is None else (P * n)(*[r.data_ptr() for r in resids])
    common = (x2.data_ptr(), xcode, T, x2.stride(0) if T > 1 else m0.K, n, packed, nbytes, Ms,
              m0.codebook.data_ptr(), m0.C, m0.bits, m0.K, None, optrs, ldo, rp, ocode, int(epilogue))
    if allreduce is not None:
        fn = "cbq_linear_fixed_multi_allreduce_norm"
        w, eps = norm
        world, resid_in, slots, counts, epoch, expect, status = allreduce
        rc = _lib.lib().cbq_linear_fixed_multi_allreduce_norm(
            *common, None if w is None else w.data_ptr(), float(eps), int(world), resid_in.data_ptr(), slots,
            counts, epoch, int(expect), status, device_stream(m0.device))
    elif norm is None:
        fn = "cbq_linear_fixed_multi"
        rc = _lib.lib().cbq_linear_fixed_multi(*common, device_stream(m0.device))
    else:
        fn = "cbq_linear_fixed_multi_norm"
        w, eps = norm
        rc = _lib.lib().cbq_linear_fixed_multi_norm(*common, None if w is None else w.data_ptr(), float(eps),
                                                    device_stream(m0.device))
    if rc == _lib.CBQ_ERR_UNSUPPORTED:
        return False
    if rc != _lib.CBQ_OK:
        raise _lib.CbqError(fn, rc)
    return True


class GPUAcceleratedEmbedding:
    """Packed fixed-width embedding table on the GPU; ``__call__(ids)`` decodes
    only the requested rows (``src/gpu_accelerated_functions.py:109-126``)."""

    def __init__(self, name: str, indices_np, codebook, shape: tuple, bits: int, device=None):
        self.name = name
        self.shape = tuple(int(s) for s in shape)
        self.vocab, self.hidden = self.shape
        self.bits = int(bits)
        if device is None and isinstance(codebook, torch.Tensor) and codebook.is_cuda:
            device = codebook.device
        self.device = _require_cuda(device)
        self.codebook = _codebook_f32(codebook, self.device)
        self.C = self.codebook.numel()
        self.nbytes = _lib.query("cbq_fixed_stream_bytes", self.vocab, self.hidden, self.bits)
        need = (self.vocab * self.hidden * self.bits + 7) // 8
        self.packed = padded_device_bytes(_stream_prefix(indices_np, need, name), self.nbytes,
                                          self.device)
        self.status = torch.tensor([0, -1, 0, 0], dtype=torch.int32, device=self.device)

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
        _lib.call("cbq_embedding_fixed", flat.data_ptr(), T, self.packed.data_ptr(), self.nbytes,
                  self.codebook.data_ptr(), self.C, self.bits, self.vocab, self.hidden,
                  out.data_ptr(), _lib.CBQ_BF16 if kdt == torch.bfloat16 else _lib.CBQ_F32,
                  self.status.data_ptr(), device_stream(self.device))
        res = out.reshape(*lead, self.hidden)
        return res if res.dtype == out_dtype else res.to(out_dtype)
