"""Huffman decode / fused decode-GEMV / embedding / encoder on the GPU.

Decoded indices, chunk-entry offsets, embedding rows and encoded bytes are
compared bit for bit; fp32 GEMV outputs within rel-L2 1e-5 of the oracle (bar
1e-4); bf16 outputs within 5e-3.
"""
import glob

import numpy as np
import pytest
import torch

import oracle
from helpers import GOLDEN, cbq, golden, need_cuda, rel_l2

pytestmark = pytest.mark.gpu

CASES = ["hand", "single", "two", "zipf", "deep", "bf16", "deep32"]
HS = cbq.gpu_huffman_functions


def stream_of(d, dev, name="h"):
    M, K = (int(v) for v in d["shape"])
    return HS.HuffmanStream(name, d["huff_stream"], d["huff_lengths"], int(d["huff_n"][0]), (M, K),
                            d["huff_row_bit_starts"], dev)


def codebook_for(d, seed=0):
    if "codebook" in d:
        return d["codebook"]
    A = d["huff_lengths"].size
    return np.random.default_rng(seed).standard_normal(max(1, A - 1)).astype(np.float32)  # clamp top symbol


@pytest.mark.parametrize("case", CASES)
def test_decode_indices_bit_exact(case):
    dev = need_cuda()
    d = golden(f"huff_{case}.npz")
    hs = stream_of(d, dev)
    got = hs.decode_indices().cpu().numpy().reshape(-1)
    np.testing.assert_array_equal(got, d["indices"].astype(np.int64))
    hs.check()


@pytest.mark.parametrize("case", CASES)
def test_chunk_table_matches_oracle(case):
    dev = need_cuda()
    d = golden(f"huff_{case}.npz")
    M, K = (int(v) for v in d["shape"])
    hs = stream_of(d, dev)
    raw = hs.chunk.cpu().numpy()
    got = raw.view(np.uint32)[:hs.nchunk].astype(np.int64)
    np.testing.assert_array_equal(got, oracle.huff_chunk_offsets(d, M, K, 64))
    # quarter lengths: bits 10j..10j+9 = bit length of codes 16j..16j+15 of the
    # chunk (j = 0, 1, 2), 0 unless code 16j+16 is in the row
    qw = raw.view(np.uint32)[hs.nchunk:2 * hs.nchunk].astype(np.int64).reshape(M, -1)
    o16 = oracle.huff_chunk_offsets(d, M, K, 16).reshape(M, -1)
    for c in range(qw.shape[1]):
        for j in range(3):
            k0, k1 = 64 * c + 16 * j, 64 * c + 16 * (j + 1)
            want = o16[:, k1 // 16] - o16[:, k0 // 16] if k1 < K else np.zeros(M, np.int64)
            np.testing.assert_array_equal((qw[:, c] >> (10 * j)) & 1023, want, err_msg=f"chunk {c} quarter {j}")


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("T", [1, 3, 8, 16])
def test_linear_huff_matches_oracle(case, T):
    dev = need_cuda()
    d = golden(f"huff_{case}.npz")
    M, K = (int(v) for v in d["shape"])
    cb = codebook_for(d)
    lin = HS.HuffmanCodebookLinear("h", d["huff_stream"], d["huff_lengths"], int(d["huff_n"][0]), cb,
                                   (M, K), 13, huff_row_bit_starts=d["huff_row_bit_starts"], device=dev)
    x = np.random.default_rng(T).standard_normal((T, K)).astype(np.float32)
    y = lin(torch.from_numpy(x).to(dev)).cpu().numpy()
    ref = oracle.huff_linear(x, d, cb, M, K)
    assert rel_l2(y, ref) < 1e-5
    lin.hs.check()


@pytest.mark.parametrize("case", CASES)
def test_linear_huff_value_mode_matches_oracle(case):
    """bf16-exact codebook values: the decode table carries the weights
    themselves, which the one-token kernel decodes with four branch-free decoders
    per chunk (guards, second-level codes and 32-bit codes included)."""
    dev = need_cuda()
    d = golden(f"huff_{case}.npz")
    M, K = (int(v) for v in d["shape"])
    cb = torch.from_numpy(codebook_for(d, 2)).to(torch.bfloat16).float().numpy()
    lin = HS.HuffmanCodebookLinear("v", d["huff_stream"], d["huff_lengths"], int(d["huff_n"][0]), cb,
                                   (M, K), 13, huff_row_bit_starts=d["huff_row_bit_starts"], device=dev)
    for T, xdt in ((1, torch.float32), (1, torch.bfloat16), (2, torch.float32)):
        x = torch.from_numpy(np.random.default_rng(T).standard_normal((T, K)).astype(np.float32)).to(xdt)
        y = lin(x.to(dev)).float().cpu().numpy()
        ref = oracle.huff_linear(x.float().numpy(), d, cb, M, K)
        assert rel_l2(y, ref) < (1e-5 if xdt == torch.float32 else 5e-3), (T, xdt)
    lin.hs.check()


def test_golden_huffman_outputs_through_gpu():
    dev = need_cuda()
    g = golden("gemv.npz")
    d = golden("huff_bf16.npz")
    M, K = (int(v) for v in d["shape"])
    lin = HS.HuffmanCodebookLinear("g", d["huff_stream"], d["huff_lengths"], int(d["huff_n"][0]),
                                   d["codebook"], (M, K), 12,
                                   huff_row_bit_starts=d["huff_row_bit_starts"], device=dev)
    y = lin(torch.from_numpy(g["hf_x"]).to(dev)).cpu().numpy()
    assert rel_l2(y, g["hf_out"]) < 1e-5
    emb = HS.HuffmanCodebookEmbedding("ge", d["huff_stream"], d["huff_lengths"], int(d["huff_n"][0]),
                                      d["codebook"], (M, K), 12,
                                      huff_row_bit_starts=d["huff_row_bit_starts"], device=dev)
    e = emb(torch.from_numpy(g["hf_emb_ids"]).to(dev)).cpu().numpy()
    np.testing.assert_array_equal(e, g["hf_emb"])


@pytest.mark.parametrize("case", CASES)
def test_embedding_huff_exact(case):
    dev = need_cuda()
    d = golden(f"huff_{case}.npz")
    M, K = (int(v) for v in d["shape"])
    cb = codebook_for(d, 1)
    emb = HS.HuffmanCodebookEmbedding("e", d["huff_stream"], d["huff_lengths"], int(d["huff_n"][0]), cb,
                                      (M, K), 13, huff_row_bit_starts=d["huff_row_bit_starts"], device=dev)
    ids = np.array([0, M - 1, M // 2, 0], dtype=np.int64)
    got = emb(torch.from_numpy(ids).to(dev)).cpu().numpy()
    np.testing.assert_array_equal(got, oracle.huff_embedding(ids, d, cb, K))


def test_bf16_io_and_bias():
    dev = need_cuda()
    d = golden("huff_bf16.npz")
    M, K = (int(v) for v in d["shape"])
    lin = HS.HuffmanCodebookLinear("b", d["huff_stream"], d["huff_lengths"], int(d["huff_n"][0]),
                                   d["codebook"], (M, K), 12,
                                   huff_row_bit_starts=d["huff_row_bit_starts"], device=dev)
    xb = torch.randn(5, K, device=dev).to(torch.bfloat16)
    bias = torch.randn(M, device=dev)
    y = lin(xb, bias=bias)
    assert y.dtype == torch.bfloat16
    ref = oracle.huff_linear(xb.float().cpu().numpy(), d, d["codebook"], M, K) + bias.cpu().numpy()
    assert rel_l2(y.float().cpu().numpy(), ref) < 5e-3
    x = torch.randn(2, K, device=dev)
    assert torch.equal(lin(x), lin(x))


@pytest.mark.parametrize("shape", [(6144, 2048), (2048, 6144)])
def test_config2_mlp_shapes(shape):
    """Huffman-coded bf16 N(0, 0.02) at Qwen3-1.7B MLP shapes."""
    dev = need_cuda()
    M, K = shape
    bf = cbq.synth.bf16_normal_np(shape, seed=M + 7 * K)
    d = cbq.synth.compress_huffman_np(bf)
    bps = (d["huff_stream"].size - 4) * 8 / (M * K)
    assert 9.5 < bps < 11.5
    lin = HS.HuffmanCodebookLinear("c2", d["huff_stream"], d["huff_lengths"], int(d["huff_n"][0]),
                                   d["codebook"], shape, d["bits"],
                                   huff_row_bit_starts=d["huff_row_bit_starts"], device=dev)
    np.testing.assert_array_equal(lin.hs.decode_indices().cpu().numpy().reshape(-1),
                                  d["_idx"].reshape(-1).astype(np.int64))
    x = np.random.default_rng(2).standard_normal((1, K)).astype(np.float32)
    y = lin(torch.from_numpy(x).to(dev)).cpu().numpy()
    assert rel_l2(y, oracle.huff_linear(x, d, d["codebook"], M, K)) < 1e-5
    r = oracle.ref_huff_linear(x, d, d["codebook"], M, K)
    if r is not None:
        assert rel_l2(y, r) < 1e-4


@pytest.mark.parametrize("case", ["zipf", "deep", "bf16"])
def test_device_encoder_matches_cpu_encoder(case):
    dev = need_cuda()
    d = golden(f"huff_{case}.npz")
    M, K = (int(v) for v in d["shape"])
    comp = cbq.synth.GpuCompressor(dev)
    enc = comp.huffman(torch.from_numpy(d["indices"].view(np.int16)).to(dev), (M, K))
    np.testing.assert_array_equal(enc["huff_stream"].cpu().numpy(), d["huff_stream"])
    np.testing.assert_array_equal(enc["huff_row_bit_starts"].cpu().numpy(), d["huff_row_bit_starts"])
    for k in ("huff_lengths", "huff_lut_sym", "huff_lut_len", "huff_sl_first_code",
              "huff_sl_base_offset", "huff_sl_sym"):
        np.testing.assert_array_equal(enc[k], d[k])


def test_corrupt_stream_is_reported():
    """Errors in the stream are reported through the status word; every read
    stays inside the buffers (bounded bit reader), nothing faults."""
    dev = need_cuda()
    d = golden("huff_single.npz")       # incomplete code: a '1' bit matches nothing
    bad = dict(d)
    s = d["huff_stream"].copy()
    s[5] = 0xFF
    bad["huff_stream"] = s
    with pytest.raises(cbq._lib.CbqError):
        stream_of(bad, dev)
    d = golden("huff_bf16.npz")
    bad = dict(d)
    bad["huff_row_bit_starts"] = d["huff_row_bit_starts"].copy()
    bad["huff_row_bit_starts"][7] += 3                     # rows no longer tile the stream
    with pytest.raises(cbq._lib.CbqError):
        stream_of(bad, dev)
    bad["huff_row_bit_starts"][7] = 1 << 40                # offset far past the end
    with pytest.raises(cbq._lib.CbqError):
        stream_of(bad, dev)
