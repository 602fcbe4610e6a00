"""cbq_linear_fixed_noalloc: the decode-GEMV entry point that allocates nothing.

Callers such as a plugin inside a host framework that owns all device memory
(and passes the plugin only its input and output buffers) cannot hand the
library a workspace; this entry point uses an array built into the library
instead.  Checked here through the C ABI against cbq_linear_fixed given a
normal workspace, on two calls in a row (the array keeps the previous call's
contents, so the second call shows that reuse is handled), within the
tolerance the other GEMV tests use (rel-L2 1e-5).  This file is collected last
so a failure here does not stop the rest of a `-x` run.
"""
import ctypes as ct

import numpy as np
import pytest
import torch

from helpers import cbq, need_cuda, rel_l2

pytestmark = pytest.mark.gpu
L = cbq._lib


def _case(M, K, bits, seed):
    rng = np.random.default_rng(seed)
    idx = rng.integers(0, 1 << bits, size=M * K).astype(np.uint16)
    cb = rng.standard_normal((1 << bits) - 3).astype(np.float32)
    return cbq.bitpack.pack_any_bits(idx, bits), cb


def _existing(dev, x, packed, nbytes, cb, bits, M, K, dtype_code, out_dtype):
    T = x.shape[0]
    n = L.query("cbq_linear_fixed_workspace_bytes", M, K, T)
    ws = torch.zeros(n, dtype=torch.uint8, device=dev)
    out = torch.empty(T, M, dtype=out_dtype, device=dev)
    L.call("cbq_linear_fixed", x.data_ptr(), dtype_code, T, K, packed.data_ptr(), nbytes, cb.data_ptr(),
           cb.numel(), bits, M, K, None, out.data_ptr(), dtype_code, M, ws.data_ptr(), n,
           torch.cuda.current_stream(dev).cuda_stream)
    return out


def _noalloc(dev, x, packed, nbytes, cb, bits, M, K, dtype_code, out_dtype):
    T = x.shape[0]
    out = torch.empty(T, M, dtype=out_dtype, device=dev)
    L.call("cbq_linear_fixed_noalloc", x.data_ptr(), dtype_code, T, K, packed.data_ptr(), nbytes,
           cb.data_ptr(), cb.numel(), bits, M, K, None, out.data_ptr(), dtype_code, M,
           torch.cuda.current_stream(dev).cuda_stream)
    return out


@pytest.mark.parametrize("M,K,T,bits,dt", [(1000, 4096, 1, 13, torch.float32),
                                           (777, 2048, 4, 12, torch.bfloat16),
                                           (96, 12288, 2, 13, torch.float32)])
def test_noalloc_matches_workspace_entry_point_twice(M, K, T, bits, dt):
    dev = need_cuda()
    packed_np, cb_np = _case(M, K, bits, seed=M + K)
    nbytes = L.query("cbq_fixed_stream_bytes", M, K, bits)
    packed = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    packed[:packed_np.size].copy_(torch.from_numpy(packed_np))
    cb = torch.from_numpy(cb_np).to(dev)
    code = L.CBQ_BF16 if dt == torch.bfloat16 else L.CBQ_F32
    tol = 1e-5
    for call in range(2):
        x = torch.randn(T, K, device=dev).to(dt)
        ref = _existing(dev, x, packed, nbytes, cb, bits, M, K, code, dt)
        got = _noalloc(dev, x, packed, nbytes, cb, bits, M, K, code, dt)
        torch.cuda.synchronize()
        assert rel_l2(got.float().cpu().numpy(), ref.float().cpu().numpy()) < tol, f"call {call}"


def test_noalloc_rejects_matrices_beyond_its_scratch():
    dev = need_cuda()
    M, K, T = 300000, 8192, 8
    assert L.query("cbq_linear_fixed_workspace_bytes", M, K, T) > (8 << 20)
    dummy = ct.c_void_p(16)
    rc = L.lib().cbq_linear_fixed_noalloc(dummy, L.CBQ_F32, T, K, dummy, 1 << 40, dummy, 8192, 13, M, K,
                                          None, dummy, L.CBQ_F32, M,
                                          torch.cuda.current_stream(dev).cuda_stream)
    assert rc == L.CBQ_ERR_ARG
