"""Host-side module logic that needs no GPU: ``.npz`` schema round trip, exact
and linear_quant modes, codebook priority, and the loud failure of
``direct_codebook`` layers when no CUDA device exists."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helpers import cbq

NPZ = cbq.npz_format


def test_npz_roundtrip_fixed_and_huffman(tmp_path):
    bf = cbq.synth.bf16_normal_np((32, 128), seed=2)
    for comp in (cbq.synth.compress_fixed_np, cbq.synth.compress_huffman_np):
        d = comp(bf, codebook_type="attention")
        f = NPZ.tensor_file(tmp_path, "model.layers.3.self_attn.o_proj.weight")
        assert f.name == "model_layers_3_self_attn_o_proj_weight.npz"
        NPZ.save_cached_tensor(f, "model.layers.3.self_attn.o_proj.weight",
                               {k: v for k, v in d.items() if not k.startswith("_")})
        z = np.load(f)
        assert str(z["mode"]) == "direct_codebook" and z["codebook_type"][0] == "attention"
        assert z["bits"].dtype.kind == "i" and z["codebook"].dtype == np.float32
        name, back = NPZ.load_cached_tensor(f)
        assert back["bits"] == d["bits"] and back["codebook_type"] == "attention"
        if "encoding" in d:
            assert back["encoding"] == "huffman"
            for k in NPZ.HUFF_KEYS:
                np.testing.assert_array_equal(back[k], d[k])
        else:
            np.testing.assert_array_equal(back["indices"], d["indices"])


def test_exact_and_linear_quant_modes():
    w = np.random.default_rng(0).standard_normal((6, 10)).astype(np.float32)
    bf = (w.view(np.uint32) >> 16).astype(np.uint16)
    layer = cbq.AdaptiveCodebookLinear.from_compressed("e", {"mode": "exact", "shape": (6, 10), "data": bf}, {})
    x = torch.randn(3, 10)
    ref = F.linear(x, torch.from_numpy((bf.astype(np.uint32) << 16).view(np.float32)))
    torch.testing.assert_close(layer(x), ref)
    lq = {"mode": "linear_quant", "shape": (6, 10), "indices": np.arange(60, dtype=np.uint8),
          "scale": 0.5, "v_min": -1.0, "bits": 8}
    layer = cbq.AdaptiveCodebookLinear.from_compressed("q", lq, {})
    wq = torch.arange(60, dtype=torch.float32).reshape(6, 10) * 0.5 - 1.0
    torch.testing.assert_close(layer(x), F.linear(x, wq))


def test_codebook_priority_local_then_global():
    sel = cbq.compressed_modules._select_codebook
    local = np.array([1.0, 2.0], np.float32)
    glob = {"mlp_ffn": torch.tensor([3.0, 4.0, 5.0])}
    assert sel({"codebook": local, "codebook_type": "mlp_ffn"}, glob).numel() == 2
    assert sel({"codebook_type": "mlp_ffn"}, glob).numel() == 3
    assert sel({"codebook_type": "attention"}, glob) is None
    assert sel({}, {"embedding": torch.zeros(4)}, default_type="embedding").numel() == 4


def test_direct_codebook_without_cuda_raises():
    if torch.cuda.is_available():
        pytest.skip("CUDA present")
    d = cbq.synth.compress_fixed_np(cbq.synth.bf16_normal_np((8, 128), seed=1))
    with pytest.raises(RuntimeError):
        cbq.AdaptiveCodebookLinear.from_compressed("x", d, {})
    with pytest.raises(RuntimeError):
        cbq.GPUAcceleratedLinear("x", d["indices"], d["codebook"], (8, 128), d["bits"])


def test_model_dir_config_and_layout(tmp_path):
    """The HF config.json of a compressed model directory maps onto the
    decoder shape, and the cache directory names follow the reference's."""
    import json
    md = cbq.model_dir
    cfg = cbq.qwen3.QWEN3_8B
    (tmp_path / "config.json").write_text(json.dumps(md._config_json(cfg)))
    assert md.read_qwen3_config(tmp_path) == cfg
    assert md.cache_dir_for(tmp_path, False).name == "codebook-lossless"
    assert md.cache_dir_for(tmp_path, True).name == "codebook-lossless-huffman"


def test_mmapped_packed_buffer_and_idx_export(tmp_path):
    """Flat .idx files (the reference's export_flat_idx / MmappedPackedBuffer
    contract, tests/test_mmap_inference.py): the exported bytes are the
    .npz's `indices`, the mapping reads them back as a zero-copy view."""
    hs = cbq.host_stream
    rng = np.random.default_rng(7)
    M, K, bits = 64, 32, 13
    packed = cbq.bitpack.pack_any_bits(rng.integers(0, 1 << bits, size=M * K).astype(np.uint16), bits)
    tdir = tmp_path / "codebook-lossless" / "tensors"
    NPZ.save_cached_tensor(tdir / "model_layers_0_mlp_weight.npz", "model.layers.0.mlp.weight",
                           {"mode": "direct_codebook", "shape": np.array([M, K]), "bits": bits,
                            "codebook_type": "mlp_ffn", "indices": packed})
    assert hs.export_flat_idx(tmp_path) == 1
    assert hs.export_flat_idx(tmp_path) == 0                    # already exported
    buf = hs.MmappedPackedBuffer(tdir / "model_layers_0_mlp_weight.idx")
    arr = buf.as_numpy()
    assert arr.base is not None and len(buf) == packed.size
    np.testing.assert_array_equal(arr, packed)
    np.testing.assert_array_equal(arr[100:200], packed[100:200])
    del arr
    buf.close()
