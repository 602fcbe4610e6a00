"""Fixed-width decode-GEMV / embedding / packer on the GPU against the oracle.

Tolerances: fp32 GEMV outputs within rel-L2 1e-5 of the oracle (the bar is
1e-4; only the fp32 summation order differs), bf16-output paths within rel-L2
5e-3 (one bf16 rounding of each output), gathers and packed bytes bit-exact.
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import cbq, golden, need_cuda, rel_l2

pytestmark = pytest.mark.gpu


def make_case(M, K, bits, C=None, seed=0):
    rng = np.random.default_rng(seed + 1000 * bits + M + K)
    C = (1 << bits) if C is None else C
    hi = min(1 << bits, C + 3)                        # a few indices >= C exercise the clamp
    idx = rng.integers(0, hi, size=M * K).astype(np.uint16)
    cb = rng.standard_normal(C).astype(np.float32)
    packed = cbq.bitpack.pack_any_bits(idx, bits)
    return idx, cb, packed


SHAPES = [
    (64, 128, 1, 13), (257, 256, 3, 13), (96, 384, 2, 7), (128, 1024, 4, 12), (64, 640, 8, 16),
    (33, 128, 5, 8), (16, 4096, 16, 13), (200, 12288, 1, 13), (8, 2048, 9, 13),
    (100, 64, 2, 13), (7, 100, 3, 5), (1, 128, 1, 1),             # generic path: K % 128 != 0
]


@pytest.mark.parametrize("M,K,T,bits", SHAPES)
def test_linear_fixed_matches_oracle(M, K, T, bits):
    dev = need_cuda()
    idx, cb, packed = make_case(M, K, bits)
    x = np.random.default_rng(M * K + T).standard_normal((T, K)).astype(np.float32)
    lin = cbq.GPUAcceleratedLinear("t", packed, cb, (M, K), bits, device=dev)
    y = lin(torch.from_numpy(x).to(dev)).cpu().numpy()
    ref = oracle.linear_fixed(x, packed, cb, M, K, bits)
    assert y.shape == (T, M)
    assert rel_l2(y, ref) < 1e-5


@pytest.mark.parametrize("bits", range(1, 17))
def test_linear_fixed_every_width(bits):
    dev = need_cuda()
    M, K, T = 96, 512, 2
    idx, cb, packed = make_case(M, K, bits, C=max(1, (1 << bits) - 1))
    x = np.random.default_rng(bits).standard_normal((T, K)).astype(np.float32)
    y = cbq.GPUAcceleratedLinear("w", packed, cb, (M, K), bits, device=dev)(
        torch.from_numpy(x).to(dev)).cpu().numpy()
    assert rel_l2(y, oracle.linear_fixed(x, packed, cb, M, K, bits)) < 1e-5


def test_large_codebook_and_int64_offsets():
    """C > 16384 takes the generic kernel; M*K*bits > 2**31 bits exercises
    64-bit offsets (reference tests/test_c_kernel.py:109-138)."""
    dev = need_cuda()
    idx, cb, packed = make_case(300, 256, 16, C=40000)
    x = np.random.default_rng(1).standard_normal((2, 256)).astype(np.float32)
    y = cbq.GPUAcceleratedLinear("big", packed, cb, (300, 256), 16, device=dev)(
        torch.from_numpy(x).to(dev)).cpu().numpy()
    assert rel_l2(y, oracle.linear_fixed(x, packed, cb, 300, 256, 16)) < 1e-5
    M, K, bits = 165200, 1, 13
    idx, cb, packed = make_case(M, K, bits)
    x = np.ones((1, 1), np.float32)
    y = cbq.GPUAcceleratedLinear("tall", packed, cb, (M, K), bits, device=dev)(
        torch.from_numpy(x).to(dev)).cpu().numpy()
    np.testing.assert_array_equal(y[0], cb[np.minimum(idx, cb.size - 1)])
    M, K = 8192, 20480                                # 2.2e9 bits
    rng = np.random.default_rng(9)
    idx = rng.integers(0, 1 << 13, size=M * K, dtype=np.uint16)
    cb = rng.standard_normal(1 << 13).astype(np.float32)
    comp = cbq.synth.GpuCompressor(dev)
    packed_d = comp.pack_fixed(torch.from_numpy(idx.view(np.int16)).to(dev), 13)
    x = rng.standard_normal((1, K)).astype(np.float32)
    y = cbq.GPUAcceleratedLinear("deep", packed_d, cb, (M, K), 13, device=dev)(
        torch.from_numpy(x).to(dev)).cpu().numpy()
    rows = np.arange(M - 40, M)                       # rows past bit 2**31
    ref = x @ cb[idx.reshape(M, K)[rows]].T
    assert rel_l2(y[0, rows], ref[0]) < 1e-5


def test_bf16_io_bias_and_determinism():
    dev = need_cuda()
    M, K, bits = 512, 2048, 13
    idx, cb, packed = make_case(M, K, bits)
    lin = cbq.GPUAcceleratedLinear("b", packed, cb, (M, K), bits, device=dev)
    xb = torch.randn(4, K, device=dev).to(torch.bfloat16)
    bias = torch.randn(M, device=dev)
    y = lin(xb, bias=bias)
    assert y.dtype == torch.bfloat16 and y.shape == (4, M)
    ref = oracle.linear_fixed(xb.float().cpu().numpy(), packed, cb, M, K, bits) + bias.cpu().numpy()
    assert rel_l2(y.float().cpu().numpy(), ref) < 5e-3
    # 3..63 bf16 tokens run on the tensor cores with the codebook rounded to
    # bf16 (this codebook is not bf16-exact): the tensor-core tolerance
    y32 = lin(xb, bias=bias, out_dtype=torch.float32)
    assert rel_l2(y32.cpu().numpy(), ref) < 1e-2
    x = torch.randn(3, K, device=dev)
    a, b = lin(x), lin(x)
    assert torch.equal(a, b)                          # fixed reduction order
    x3 = torch.randn(2, 5, K, device=dev)
    np.testing.assert_array_equal(lin(x3).reshape(10, M).cpu().numpy(),
                                  lin(x3.reshape(10, K)).cpu().numpy())


def test_golden_fixture_through_gpu():
    dev = need_cuda()
    g = golden("gemv.npz")
    M, K, bits = (int(v) for v in g["fx_shape"])
    y = cbq.GPUAcceleratedLinear("g", g["fx_packed"], g["fx_codebook"], (M, K), bits, device=dev)(
        torch.from_numpy(g["fx_x"]).to(dev)).cpu().numpy()
    assert rel_l2(y, g["fx_out"]) < 1e-5


def test_config1_lossless_2048():
    """2048x2048 bf16 N(0, 0.02), frequency-sorted codebook."""
    dev = need_cuda()
    bf = cbq.synth.bf16_normal_np((2048, 2048), seed=0)
    d = cbq.synth.compress_fixed_np(bf)
    assert d["bits"] == 13
    x = np.random.default_rng(0).standard_normal((1, 2048)).astype(np.float32)
    y = cbq.GPUAcceleratedLinear("c1", d["indices"], d["codebook"], (2048, 2048), d["bits"], device=dev)(
        torch.from_numpy(x).to(dev)).cpu().numpy()
    ref = oracle.linear_fixed(x, d["indices"], d["codebook"], 2048, 2048, d["bits"])
    assert rel_l2(y, ref) < 1e-5
    r = oracle.ref_linear_fixed(x, d["indices"], d["codebook"], 2048, 2048, d["bits"])
    if r is not None:
        assert rel_l2(y, r) < 1e-4


@pytest.mark.parametrize("bits", [4, 8, 13, 16])
def test_embedding_fixed_exact(bits):
    dev = need_cuda()
    V, H = 300, 200
    idx, cb, packed = make_case(V, H, bits)
    emb = cbq.GPUAcceleratedEmbedding("e", packed, cb, (V, H), bits, device=dev)
    ids = np.array([[0, 5, 299], [5, 17, 1]], dtype=np.int64)
    y = emb(torch.from_numpy(ids).to(dev))
    assert y.shape == (2, 3, H)
    np.testing.assert_array_equal(y.cpu().numpy().reshape(-1, H),
                                  oracle.embedding_fixed(ids, packed, cb, H, bits))
    yb = emb(torch.from_numpy(ids).to(dev), out_dtype=torch.bfloat16)
    assert yb.dtype == torch.bfloat16


def test_embedding_out_of_range_id_is_reported_not_faulted():
    dev = need_cuda()
    idx, cb, packed = make_case(10, 64, 8)
    emb = cbq.GPUAcceleratedEmbedding("e", packed, cb, (10, 64), 8, device=dev)
    y = emb(torch.tensor([3, 10, -1], device=dev))
    torch.cuda.synchronize()
    assert torch.all(y[1:] == 0)
    flags = int(emb.status[0].item())
    assert flags & cbq._lib.FLAG_CORRUPT


@pytest.mark.parametrize("bits", range(1, 17))
def test_device_packer_matches_cpu_packer(bits):
    dev = need_cuda()
    rng = np.random.default_rng(bits)
    idx = rng.integers(0, 1 << bits, size=10007).astype(np.uint16)
    comp = cbq.synth.GpuCompressor(dev)
    got = comp.pack_fixed(torch.from_numpy(idx.view(np.int16)).to(dev), bits).cpu().numpy()
    np.testing.assert_array_equal(got, cbq.bitpack.pack_any_bits(idx, bits))


def test_gpu_lossless_compressor_roundtrip():
    dev = need_cuda()
    comp = cbq.synth.GpuCompressor(dev)
    bits = cbq.synth.bf16_normal_gpu((256, 512), seed=3, device=dev)
    d = comp.compress(bits, huffman=False)
    cb = d["codebook"].cpu().numpy()
    idx = cbq.bitpack.unpack_any_bits(d["indices"].cpu().numpy(), d["bits"], 256 * 512)
    np.testing.assert_array_equal(cb[idx].view(np.uint32) >> 16, bits.cpu().numpy().reshape(-1))


def test_workspace_shared_by_calls_of_different_shapes():
    """One workspace passed to 3..63-token calls of several row counts in turn:
    every call leaves it zero-filled, so a later call whose counters fall where
    an earlier call kept its piece sums still combines its rows correctly."""
    dev = need_cuda()
    L = cbq._lib
    K, T, bits = 2048, 8, 13
    n = L.query("cbq_linear_fixed_workspace_bytes", 1000, K, T)
    ws = torch.zeros(n, dtype=torch.uint8, device=dev)
    for M in (1000, 777, 1000, 301, 999):
        idx, cb, packed = make_case(M, K, bits, seed=M)
        lin = cbq.GPUAcceleratedLinear("w", packed, cb, (M, K), bits, device=dev)
        x = np.random.default_rng(M).standard_normal((T, K)).astype(np.float32)
        xd = torch.from_numpy(x).to(dev)
        out = torch.empty(T, M, device=dev)
        L.call("cbq_linear_fixed", xd.data_ptr(), L.CBQ_F32, T, K, lin.packed.data_ptr(), lin.nbytes,
               lin.codebook.data_ptr(), lin.C, bits, M, K, None, out.data_ptr(), L.CBQ_F32, M, ws.data_ptr(), n,
               torch.cuda.current_stream(dev).cuda_stream)
        torch.cuda.synchronize()
        assert rel_l2(out.cpu().numpy(), oracle.linear_fixed(x, packed, cb, M, K, bits)) < 1e-5, M
    assert not bool(ws.any())
