"""cbq_linear_fixed_noalloc: the decode-GEMV entry point that allocates nothing.

Callers such as a plugin inside a host framework that owns all device memory
(and passes the plugin only its input and output buffers) cannot hand the
library a workspace; this entry point uses an array built into the library
instead.  Checked here through the C ABI against cbq_linear_fixed given a
normal workspace and against the C oracle, on two calls in a row (the array
keeps the previous call's contents, so the second call shows that reuse is
handled), within the tolerance the other GEMV tests use (rel-L2 1e-5).  The
cases take every dispatch: the one/two-token GEMV (no scratch), the 3..63
token kernel with one and with two token blocks (scratch), and a matrix whose
scratch nearly fills the array.  This file is collected last so a failure
here does not stop the rest of a `-x` run.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import cbq, need_cuda, rel_l2

pytestmark = pytest.mark.gpu
L = cbq._lib
LIMIT = 8 << 20           # CBQ_NOALLOC_SCRATCH_BYTES


def _case(dev, M, K, bits, seed):
    """Random stream bytes (every bit pattern is a valid fixed-width stream;
    indices at or above C exercise the clamp) and a codebook of 2^bits - 3."""
    rng = np.random.default_rng(seed)
    packed_np = rng.integers(0, 256, size=(M * K * bits + 7) // 8, dtype=np.uint8)
    cb = rng.standard_normal(max(1, (1 << bits) - 3)).astype(np.float32)
    nbytes = L.query("cbq_fixed_stream_bytes", M, K, bits)
    packed = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    packed[:packed_np.size].copy_(torch.from_numpy(packed_np))
    return packed_np, packed, nbytes, cb, torch.from_numpy(cb).to(dev)


def _existing(dev, x, packed, nbytes, cb, bits, M, K, code, out_dtype):
    T = x.shape[0]
    n = L.query("cbq_linear_fixed_workspace_bytes", M, K, T)
    ws = torch.zeros(n, dtype=torch.uint8, device=dev)
    out = torch.empty(T, M, dtype=out_dtype, device=dev)
    L.call("cbq_linear_fixed", x.data_ptr(), code, T, K, packed.data_ptr(), nbytes, cb.data_ptr(),
           cb.numel(), bits, M, K, None, out.data_ptr(), code, M, ws.data_ptr(), n,
           torch.cuda.current_stream(dev).cuda_stream)
    return out


def _noalloc(dev, x, packed, nbytes, cb, bits, M, K, code, out):
    T = x.shape[0]
    return L.lib().cbq_linear_fixed_noalloc(x.data_ptr(), code, T, K, packed.data_ptr(), nbytes, cb.data_ptr(),
                                            cb.numel(), bits, M, K, None, out.data_ptr(), code, M,
                                            torch.cuda.current_stream(dev).cuda_stream)


@pytest.mark.parametrize("M,K,T,bits,dt", [(1000, 4096, 1, 13, torch.float32),      # one-token GEMV
                                           (96, 12288, 2, 13, torch.float32),       # two-token GEMV
                                           (777, 2048, 4, 12, torch.bfloat16),      # 3..63 kernel
                                           (512, 1024, 8, 13, torch.bfloat16),
                                           (300, 2048, 5, 11, torch.float32),       # two token blocks
                                           (230000, 1024, 8, 4, torch.float32)],    # scratch near the limit
                         ids=["t1", "t2", "t4", "t8", "t5-two-blocks", "t8-near-limit"])
def test_noalloc_matches_workspace_entry_point_twice(M, K, T, bits, dt):
    dev = need_cuda()
    packed_np, packed, nbytes, cb_np, cb = _case(dev, M, K, bits, seed=M + K)
    if M == 230000:
        assert 0.9 * LIMIT < L.query("cbq_linear_fixed_workspace_bytes", M, K, T) <= LIMIT
    code = L.CBQ_BF16 if dt == torch.bfloat16 else L.CBQ_F32
    tol = 1e-5
    for call in range(2):
        x = torch.randn(T, K, device=dev).to(dt)
        ref = _existing(dev, x, packed, nbytes, cb, bits, M, K, code, dt)
        got = torch.full((T, M), float("nan"), dtype=dt, device=dev)
        assert _noalloc(dev, x, packed, nbytes, cb, bits, M, K, code, got) == L.CBQ_OK
        torch.cuda.synchronize()
        g = got.float().cpu().numpy()
        assert rel_l2(g, ref.float().cpu().numpy()) < tol, f"call {call} vs cbq_linear_fixed"
        if dt == torch.float32:
            want = oracle.linear_fixed(x.cpu().numpy(), packed_np, cb_np, M, K, bits)
            assert rel_l2(g, want) < tol, f"call {call} vs the oracle"


def test_noalloc_rejects_matrices_beyond_its_scratch():
    """Real buffers of the declared sizes: a regression in the size check
    would compute (and fail the assert) rather than touch memory it was not
    given.  The same matrix at one token needs no scratch and is served."""
    dev = need_cuda()
    M, K, bits = 240000, 1024, 1
    assert L.query("cbq_linear_fixed_workspace_bytes", M, K, 8) > LIMIT
    packed_np, packed, nbytes, cb_np, cb = _case(dev, M, K, bits, seed=7)
    x = torch.randn(8, K, device=dev)
    out = torch.zeros(8, M, device=dev)
    assert _noalloc(dev, x, packed, nbytes, cb, bits, M, K, L.CBQ_F32, out) == L.CBQ_ERR_ARG
    torch.cuda.synchronize()
    assert not bool(out.any())                                 # nothing was launched
    x1 = x[:1].contiguous()
    out1 = torch.empty(1, M, device=dev)
    assert _noalloc(dev, x1, packed, nbytes, cb, bits, M, K, L.CBQ_F32, out1) == L.CBQ_OK
    ref = _existing(dev, x1, packed, nbytes, cb, bits, M, K, L.CBQ_F32, torch.float32)
    torch.cuda.synchronize()
    assert rel_l2(out1.cpu().numpy(), ref.cpu().numpy()) < 1e-5
