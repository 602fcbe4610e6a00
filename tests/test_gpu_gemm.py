"""Tensor-core prefill GEMM (cbq_gemm.cu): many tokens through cbq_linear_fixed.

bf16 activations times weights decoded to bf16 in shared memory, fp32
accumulation in TMEM.  Lossless codebooks hold bf16 values exactly, so the
only difference from the fp32 oracle on the same (bf16) activations is the
accumulation order: rel-L2 <= 1e-5.  A codebook that is not bf16-exact is
rounded to bf16 first: rel-L2 <= 1e-2 (the tensor-core tolerance)."""
import numpy as np
import pytest
import torch

import oracle
from helpers import cbq, need_cuda, rel_l2

pytestmark = pytest.mark.gpu
G = cbq.gpu_accelerated_functions


def _lin(dev, M, K, bits, seed, bf16_exact=True):
    rng = np.random.default_rng(seed)
    C = (1 << bits) - 3
    cb = (rng.standard_normal(C) * 0.02).astype(np.float32)
    if bf16_exact:
        cb = (cb.view(np.uint32) & 0xFFFF0000).view(np.float32)
    idx = rng.integers(0, 1 << bits, size=M * K).astype(np.uint16)      # some >= C: clamped
    packed = cbq.bitpack.pack_any_bits(idx, bits)
    return G.GPUAcceleratedLinear("w", packed, cb, (M, K), bits, device=dev), packed, cb


@pytest.mark.parametrize("M,K,T,bits", [(128, 128, 64, 13), (256, 512, 300, 13), (512, 1024, 256, 8),
                                        (384, 256, 520, 4), (128, 4096, 96, 14)])
def test_gemm_matches_oracle(M, K, T, bits):
    dev = need_cuda()
    lin, packed, cb = _lin(dev, M, K, bits, seed=M + T)
    x = torch.randn(T, K, device=dev).to(torch.bfloat16)
    y = lin(x).float().cpu().numpy()
    ref = oracle.linear_fixed(x.float().cpu().numpy(), packed, cb, M, K, bits)
    assert rel_l2(y, ref) < 1e-2                            # bf16 output rounding
    y32 = lin(x, out_dtype=torch.float32).cpu().numpy()
    assert rel_l2(y32, ref) < 1e-5


def test_gemm_bias_and_rounded_codebook():
    dev = need_cuda()
    M, K, T, bits = 256, 256, 128, 12
    lin, packed, cb = _lin(dev, M, K, bits, seed=3, bf16_exact=False)
    x = torch.randn(T, K, device=dev).to(torch.bfloat16)
    bias = torch.randn(M, device=dev)
    y = lin(x, bias=bias, out_dtype=torch.float32).cpu().numpy()
    ref = oracle.linear_fixed(x.float().cpu().numpy(), packed, cb, M, K, bits) + bias.cpu().numpy()
    assert rel_l2(y, ref) < 1e-2


def test_gemm_is_deterministic():
    dev = need_cuda()
    lin, _, _ = _lin(dev, 256, 512, 13, seed=9)
    x = torch.randn(200, 512, device=dev).to(torch.bfloat16)
    assert torch.equal(lin(x), lin(x))


@pytest.mark.parametrize("M,K,T,bits", [(128, 128, 64, 13), (256, 512, 300, 12), (384, 1024, 256, 8),
                                        (128, 4096, 96, 14), (256, 256, 70, 5)])
def test_huffman_prefill_transcode_gemm_matches_oracle(M, K, T, bits):
    """Huffman streams with 64 or more bf16 tokens: transcoded once to fixed
    width in the workspace, then the tensor-core GEMM (rel-L2 1e-5 with a
    bf16-exact codebook; indices at or above C clamp)."""
    dev = need_cuda()
    rng = np.random.default_rng(M + K + T)
    C = (1 << bits) - 3
    cb = ((rng.standard_normal(C) * 0.02).astype(np.float32).view(np.uint32) & 0xFFFF0000).view(np.float32)
    idx = np.minimum(rng.zipf(1.3, size=(M, K)) - 1, (1 << bits) - 1).astype(np.uint16)   # skewed, some >= C
    d = cbq.huffman_codebook.huffman_encode_indices(idx.reshape(-1), shape=(M, K))
    lin = cbq.HuffmanCodebookLinear("h", d["huff_stream"], d["huff_lengths"], int(d["huff_n"][0]), cb, (M, K), bits,
                                    huff_row_bit_starts=d["huff_row_bit_starts"], device=dev)
    x = torch.randn(T, K, device=dev).to(torch.bfloat16)
    y = lin(x, out_dtype=torch.float32).cpu().numpy()
    lin.hs.check()
    ref = oracle.huff_linear(x.float().cpu().numpy(), d, cb, M, K)
    assert rel_l2(y, ref) < 1e-5
    y16 = lin(x).float().cpu().numpy()
    assert rel_l2(y16, ref) < 1e-2


@pytest.mark.parametrize("M,K,T,bits", [(128, 256, 3, 13), (1024, 4096, 8, 13), (384, 1024, 5, 8), (12288, 4096, 8, 13),
                                        (4096, 12288, 8, 13), (256, 512, 33, 12), (640, 2048, 63, 14),
                                        (2048, 2048, 16, 4)])
def test_small_batch_tensor_core_gemm_matches_oracle(M, K, T, bits):
    """3..63 bf16 tokens (decode batches): the split-K tensor-core GEMM (one
    32/64-token tile, each row tile's K range over several CTAs, partial tiles
    combined in split order by the last one), two calls in a row (the arrival
    counters are reused): rel-L2 1e-5 against the oracle with a bf16-exact
    codebook, bit-identical between the calls."""
    dev = need_cuda()
    lin, packed, cb = _lin(dev, M, K, bits, seed=M + K + T)
    outs = []
    for _ in range(2):
        x = torch.randn(T, K, device=dev, generator=torch.Generator(device=dev).manual_seed(T)).to(torch.bfloat16)
        y = lin(x, out_dtype=torch.float32)
        outs.append(y)
    ref = oracle.linear_fixed(x.float().cpu().numpy(), packed, cb, M, K, bits)
    assert rel_l2(outs[1].cpu().numpy(), ref) < 1e-5
    assert torch.equal(outs[0], outs[1])
