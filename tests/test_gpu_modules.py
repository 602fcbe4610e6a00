"""Module API (AdaptiveCodebookLinear / AdaptiveCodebookEmbedding) on the GPU,
fed from ``.npz`` files with the reference's key set; mirrors the checks of the
reference's ``tests/test_compressed_roundtrip.py:937-1250``."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from helpers import cbq, need_cuda, rel_l2

pytestmark = pytest.mark.gpu
NPZ = cbq.npz_format


def roundtrip(tmp_path, name, data):
    f = NPZ.tensor_file(tmp_path, name)
    NPZ.save_cached_tensor(f, name, {k: v for k, v in data.items() if not k.startswith("_")})
    n, d = NPZ.load_cached_tensor(f)
    assert n == name
    return d


@pytest.mark.parametrize("huffman", [False, True])
def test_linear_from_npz_matches_dense(tmp_path, huffman):
    dev = need_cuda()
    M, K = 384, 1024
    bf = cbq.synth.bf16_normal_np((M, K), seed=11)
    comp = cbq.synth.compress_huffman_np if huffman else cbq.synth.compress_fixed_np
    d = roundtrip(tmp_path, "model.layers.0.mlp.up_proj.weight", comp(bf, codebook_type="mlp_ffn"))
    layer = cbq.AdaptiveCodebookLinear.from_compressed("up", d, {}, use_gpu=True, device=dev)
    assert layer._gpu_func is not None and layer.indices is None and layer._huff_data is None
    assert layer.bits == d["bits"] and layer.codebook.dtype == torch.float32
    assert isinstance(layer._gpu_func, cbq.HuffmanCodebookLinear if huffman else cbq.GPUAcceleratedLinear)
    # no resident dense weight anywhere in the module
    assert all(t.numel() < M * K for t in list(layer.buffers()) + list(layer.parameters()))
    w = torch.from_numpy((bf.astype(np.uint32) << 16).view(np.float32))
    x = torch.randn(2, 3, K)
    y = layer(x.to(dev))
    assert y.shape == (2, 3, M) and y.dtype == torch.float32
    assert rel_l2(y.cpu().numpy(), F.linear(x.double(), w.double()).numpy()) < 1e-5
    xb = x.to(torch.bfloat16)
    yb = layer(xb.to(dev))
    assert yb.dtype == torch.bfloat16
    assert rel_l2(yb.float().cpu().numpy(), F.linear(xb.double(), w.double()).numpy()) < 5e-3
    layer.bias = torch.randn(M, device=dev)
    yb2 = layer(x.to(dev))
    assert rel_l2(yb2.cpu().numpy(), (F.linear(x.double(), w.double()) + layer.bias.cpu().double()).numpy()) < 1e-5


def test_global_codebook_selection(tmp_path):
    dev = need_cuda()
    M, K = 128, 256
    bf = cbq.synth.bf16_normal_np((M, K), seed=4)
    cb, lut = cbq.synth.codebook_from_hist(np.bincount(bf.reshape(-1), minlength=65536))
    d = cbq.synth.compress_fixed_np(bf, codebook=cb, lut=lut, codebook_type="attention")
    d.pop("codebook")
    NPZ.save_global_codebooks(tmp_path, {"attention": cb})
    gcb = NPZ.load_global_codebooks(tmp_path)
    d = roundtrip(tmp_path, "model.layers.0.self_attn.q_proj.weight", d)
    assert "codebook" not in d and d["codebook_type"] == "attention"
    layer = cbq.AdaptiveCodebookLinear.from_compressed("q", d, gcb, device=dev)
    x = np.random.default_rng(0).standard_normal((1, K)).astype(np.float32)
    y = layer(torch.from_numpy(x).to(dev)).cpu().numpy()
    assert rel_l2(y, oracle.linear_fixed(x, d["indices"], cb, M, K, d["bits"])) < 1e-5


@pytest.mark.parametrize("huffman", [False, True])
def test_embedding_from_npz(tmp_path, huffman):
    dev = need_cuda()
    V, H = 1000, 256
    bf = cbq.synth.bf16_normal_np((V, H), seed=5)
    comp = cbq.synth.compress_huffman_np if huffman else cbq.synth.compress_fixed_np
    d = roundtrip(tmp_path, "model.embed_tokens.weight", comp(bf, codebook_type="embedding"))
    emb = cbq.AdaptiveCodebookEmbedding.from_compressed("embed", d, {}, device=dev)
    ids = torch.tensor([[1, 999, 3], [3, 0, 500]], device=dev)
    out = emb(ids)
    w = (bf.astype(np.uint32) << 16).view(np.float32)
    np.testing.assert_array_equal(out.cpu().numpy(), w[ids.cpu().numpy()])
    emb.embed_scale = 2.0
    np.testing.assert_array_equal(emb(ids).cpu().numpy(), 2.0 * w[ids.cpu().numpy()])
    emb.codebook = emb.codebook.to(torch.bfloat16)
    assert emb(ids).dtype == torch.bfloat16


def test_no_cpu_fallback():
    need_cuda()
    bf = cbq.synth.bf16_normal_np((8, 128), seed=1)
    d = cbq.synth.compress_fixed_np(bf)
    with pytest.raises(RuntimeError):
        cbq.AdaptiveCodebookLinear.from_compressed("x", d, {}, use_gpu=False)
    layer = cbq.AdaptiveCodebookLinear("y", (8, 128), "direct_codebook")
    with pytest.raises(RuntimeError):
        layer(torch.randn(1, 128))
