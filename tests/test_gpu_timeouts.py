"""The bounded device-side waits of the tensor-parallel all-reduce run out
cleanly on one GPU.

The consumers of the peer-memory all-reduce (``cbq_rmsnorm_allreduce``, the
last CTA of ``cbq_linear_fixed_peer_norm``, and every CTA of
``cbq_linear_fixed_multi_allreduce_norm``) poll per-rank arrival
counters until they reach ``epoch * expect``.  Here no rank ever adds to the
counters, so the wait must give up after its bound (2 s of %globaltimer),
record ``CBQ_FLAG_TIMEOUT`` in the status word, write nothing, and leave the
context usable: later calls see the flag and return without waiting.  This is
the failure a rank that died between steps would cause; it is made on the
host (a counter that nothing sets), not by faulting the GPU.
"""
import ctypes as ct
import time

import numpy as np
import pytest
import torch

from helpers import cbq, need_cuda

pytestmark = pytest.mark.gpu
L = cbq._lib


def _status(dev):
    return torch.tensor([0, -1, 0, 0], dtype=torch.int32, device=dev)


def _timed(fn):
    torch.cuda.synchronize()
    t0 = time.monotonic()
    fn()
    torch.cuda.synchronize()
    return time.monotonic() - t0


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
def test_allreduce_norm_wait_runs_out(dt):
    dev = need_cuda()
    world, B, H = 2, 1, 512
    code = L.CBQ_BF16 if dt == torch.bfloat16 else L.CBQ_F32
    x = torch.randn(B, H, device=dev).to(dt)
    x0 = x.clone()
    slots = torch.randn(world * B * H, device=dev).to(dt)
    counts = torch.zeros(world, dtype=torch.int32, device=dev)     # nobody ever arrives
    epoch = torch.ones(1, dtype=torch.int32, device=dev)
    out = torch.full((B, H), 7.0, device=dev).to(dt)
    status = _status(dev)
    s = torch.cuda.current_stream(dev).cuda_stream

    def call():
        L.call("cbq_rmsnorm_allreduce", x.data_ptr(), slots.data_ptr(), counts.data_ptr(), epoch.data_ptr(), H,
               world, code, B, H, None, 1e-6, out.data_ptr(), status.data_ptr(), s)
    dt1 = _timed(call)
    st = status.cpu().numpy()
    assert st[0] & L.FLAG_TIMEOUT, st
    assert 1.5 < dt1 < 30.0, dt1                      # waited for its bound, then returned
    assert torch.equal(x, x0)                         # nothing written after giving up
    assert bool((out.float() == 7.0).all())
    dt2 = _timed(call)                                # the flag is seen: no second wait
    assert dt2 < 1.0, dt2
    # the context still runs ordinary work
    y = (x.float() * 2).sum()
    torch.cuda.synchronize()
    assert torch.isfinite(y)


def test_peer_norm_gemv_wait_runs_out():
    """cbq_linear_fixed_peer_norm with both 'ranks' on this GPU: its own
    partial rows and counter increments arrive (M rows per counter per call),
    but the epoch asks for five calls' worth, so the last CTA's wait runs out."""
    dev = need_cuda()
    world, T, M, K, bits = 2, 1, 512, 1024, 13
    rng = np.random.default_rng(3)
    idx = rng.integers(0, 1 << bits, size=M * K).astype(np.uint16)
    cb = torch.from_numpy(rng.standard_normal(1 << bits).astype(np.float32)).to(dev)
    nbytes = L.query("cbq_fixed_stream_bytes", M, K, bits)
    packed = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    p = cbq.bitpack.pack_any_bits(idx, bits)
    packed[:p.size].copy_(torch.from_numpy(p))
    x = torch.randn(T, K, device=dev).to(torch.bfloat16)
    slots = torch.zeros(world * T * M, device=dev, dtype=torch.bfloat16)
    counts = torch.zeros(world, dtype=torch.int32, device=dev)
    epoch = torch.full((1,), 5, dtype=torch.int32, device=dev)
    resid = torch.randn(T, M, device=dev).to(torch.bfloat16)
    resid0 = resid.clone()
    norm_out = torch.zeros(T, M, device=dev, dtype=torch.bfloat16)
    arrive = torch.zeros(1, dtype=torch.int32, device=dev)
    status = _status(dev)
    P = ct.c_void_p
    slot_ptrs = (P * world)(*[slots.data_ptr() + r * T * M * 2 for r in range(world)])
    count_ptrs = (P * world)(*[counts.data_ptr() + r * 4 for r in range(world)])
    s = torch.cuda.current_stream(dev).cuda_stream

    def call():
        rc = L.lib().cbq_linear_fixed_peer_norm(
            x.data_ptr(), L.CBQ_BF16, T, K, packed.data_ptr(), nbytes, cb.data_ptr(), cb.numel(), bits, M, K,
            None, world, slot_ptrs, count_ptrs, M, L.CBQ_BF16, slots.data_ptr(), counts.data_ptr(),
            epoch.data_ptr(), M, resid.data_ptr(), M, None, 1e-6, norm_out.data_ptr(), M, arrive.data_ptr(),
            status.data_ptr(), s)
        assert rc == L.CBQ_OK, rc
    dt1 = _timed(call)
    st = status.cpu().numpy()
    assert st[0] & L.FLAG_TIMEOUT, st
    assert 1.5 < dt1 < 30.0, dt1
    assert torch.equal(resid, resid0)                 # the residual stream is untouched
    assert int(arrive.item()) == 0                    # the arrival count is left reset
    assert counts.cpu().tolist() == [M, M]            # its own rows were delivered
    dt2 = _timed(call)
    assert dt2 < 1.0, dt2


def test_allreduce_consuming_gemv_wait_runs_out():
    """cbq_linear_fixed_multi_allreduce_norm (the GEMV that consumes the
    previous layer's peer all-reduce): its CTAs' wait gives up, the updated
    residual stream is not written, and a later call does not wait."""
    dev = need_cuda()
    world, T, M, K, bits = 2, 1, 384, 512, 13
    rng = np.random.default_rng(5)
    idx = rng.integers(0, 1 << bits, size=M * K).astype(np.uint16)
    cb = torch.from_numpy(rng.standard_normal(1 << bits).astype(np.float32)).to(dev)
    lin = cbq.GPUAcceleratedLinear("w", cbq.bitpack.pack_any_bits(idx, bits), cb, (M, K), bits, device=dev)
    resid_in = torch.randn(T, K, device=dev).to(torch.bfloat16)
    x = torch.full((T, K), 3.0, device=dev).to(torch.bfloat16)
    slots = torch.randn(world * T * K, device=dev).to(torch.bfloat16)
    counts = torch.zeros(world, dtype=torch.int32, device=dev)       # no rank ever arrives
    epoch = torch.ones(1, dtype=torch.int32, device=dev)
    out = torch.empty(T, M, device=dev, dtype=torch.bfloat16)
    status = _status(dev)
    ar = (world, resid_in, slots.data_ptr(), counts.data_ptr(), epoch.data_ptr(), K, status.data_ptr())

    def call():
        assert cbq.gpu_accelerated_functions.linear_fixed_multi([lin], x, [out], norm=(None, 1e-6), allreduce=ar)
    dt1 = _timed(call)
    st = status.cpu().numpy()
    assert st[0] & L.FLAG_TIMEOUT, st
    assert 1.5 < dt1 < 30.0, dt1
    assert bool((x.float() == 3.0).all())                            # the residual stream is not written
    dt2 = _timed(call)
    assert dt2 < 1.0, dt2


def test_flagged_slot_read_runs_out():
    """The flagged-slot form of the consuming GEMV: slot words that never
    carry the step's epoch make every CTA's read give up within the bound."""
    dev = need_cuda()
    world, T, M, K, bits = 2, 1, 256, 512, 13
    rng = np.random.default_rng(6)
    idx = rng.integers(0, 1 << bits, size=M * K).astype(np.uint16)
    cb = torch.from_numpy(rng.standard_normal(1 << bits).astype(np.float32)).to(dev)
    lin = cbq.GPUAcceleratedLinear("w", cbq.bitpack.pack_any_bits(idx, bits), cb, (M, K), bits, device=dev)
    resid_in = torch.randn(T, K, device=dev).to(torch.bfloat16)
    x = torch.full((T, K), 3.0, device=dev).to(torch.bfloat16)
    slots = torch.zeros(world * T * K * 4, dtype=torch.uint8, device=dev)   # epoch 0 everywhere
    epoch = torch.ones(1, dtype=torch.int32, device=dev)
    out = torch.empty(T, M, device=dev, dtype=torch.bfloat16)
    status = _status(dev)
    ar = (world, resid_in, slots.data_ptr(), None, epoch.data_ptr(), K, status.data_ptr())

    def call():
        assert cbq.gpu_accelerated_functions.linear_fixed_multi([lin], x, [out], norm=(None, 1e-6), allreduce=ar)
    dt1 = _timed(call)
    st = status.cpu().numpy()
    assert st[0] & L.FLAG_TIMEOUT, st
    assert 1.5 < dt1 < 30.0, dt1
    dt2 = _timed(call)
    assert dt2 < 1.0, dt2
