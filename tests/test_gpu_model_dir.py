"""Compressed model directories (``<model>/codebook-lossless[-huffman]/``
``tensors/*.npz`` + ``codebooks/*.npy`` + ``config.json``) read into the
decoder, the reference's loader path (``src/model_loader.py:205-281``).

* A directory written from seeded synthetic weights loads into device
  objects whose greedy tokens (fp32 activations) equal those of the same
  model built in memory, fixed width and Huffman, tied lm_head included.
* Tensor-parallel shards cut by the loader decode to exactly the matching
  slice of the full tensor's indices (rows for column-parallel layers,
  columns for row-parallel ones), and a second load reads them back from the
  shard cache instead of re-cutting them.
"""
import importlib
import json

import numpy as np
import pytest
import torch

from helpers import cbq, need_cuda

pytestmark = pytest.mark.gpu
q3 = cbq.qwen3
md = cbq.model_dir
qd = importlib.import_module("codebook-quantization_b200.qwen3_decode")
L = cbq._lib

TINY = q3.Qwen3Config("tiny-dir", 2, 256, 512, 4, 2, 64, 1000, 1e6, False)
TINY_TIED = q3.Qwen3Config("tiny-dir-tied", 2, 256, 768, 4, 2, 64, 1024, 1e6, True)


def _indices(obj, dev):
    """Decoded index matrix of a fixed-width or Huffman device object."""
    if hasattr(obj, "hs"):
        return obj.hs.decode_indices().to(torch.int64)
    M, K = obj.shape
    idx = torch.empty(M * K + 1, dtype=torch.int16, device=dev)
    L.call("cbq_unpack_fixed", obj.packed.data_ptr(), obj.nbytes, obj.bits, M * K, idx.data_ptr(),
           torch.cuda.current_stream(dev).cuda_stream)
    return (idx[:M * K].to(torch.int64) & 0xFFFF).view(M, K)


@pytest.mark.parametrize("cfg", [TINY, TINY_TIED], ids=lambda c: c.name)
@pytest.mark.parametrize("huffman", [False, True], ids=["fixed", "huffman"])
def test_model_dir_decodes_like_the_in_memory_model(tmp_path, cfg, huffman):
    dev = need_cuda()
    md.write_qwen3_model_dir(cfg, tmp_path / "m", huffman=huffman, seed=4, device=dev)
    cache = md.cache_dir_for(tmp_path / "m", huffman)
    assert (cache / "codebooks" / "attention_codebook.npy").exists()
    assert json.loads((tmp_path / "m" / "config.json").read_text())["num_hidden_layers"] == cfg.layers
    assert md.read_qwen3_config(tmp_path / "m") == q3.Qwen3Config(cfg.name, *[getattr(cfg, f) for f in (
        "layers", "hidden", "inter", "heads", "kv_heads", "head_dim", "vocab", "rope_theta", "tie_embeddings",
        "rms_eps")])
    Wd = md.ModelDirWeights(tmp_path / "m", dev)
    assert Wd.huffman == huffman
    Wm = q3.CompressedQwen3Weights(cfg, dev, huffman=huffman, seed=4)
    for name, obj in Wm.layers.items():
        assert torch.equal(_indices(Wd.layers[name], dev), _indices(obj, dev)), name
    prompt = torch.randint(0, cfg.vocab, (2, 10), generator=torch.Generator().manual_seed(2))
    toks = [qd.Qwen3Decoder(W, batch=2, max_len=40, act_dtype=torch.float32).generate(prompt, 16).cpu()
            for W in (Wd, Wm)]
    assert torch.equal(toks[0], toks[1])


@pytest.mark.parametrize("huffman", [False, True], ids=["fixed", "huffman"])
def test_model_dir_tensor_parallel_shards_and_cache(tmp_path, huffman):
    dev = need_cuda()
    md.write_qwen3_model_dir(TINY, tmp_path / "m", huffman=huffman, seed=6, device=dev)
    full = md.ModelDirWeights(tmp_path / "m", dev)
    world = 2
    specs = {s.name: s for s in q3.linear_specs(TINY)}
    for rank in range(world):
        W = md.ModelDirWeights(tmp_path / "m", dev, rank=rank, world=world)
        assert W.shard_builds > 0 and W.shard_hits == 0
        for name, obj in W.layers.items():
            ref = _indices(full.layers[name], dev)
            sp = specs[name]
            if sp.split == "col":
                lo, hi = q3.shard_range(ref.shape[0], rank, world)
                ref = ref[lo:hi]
            elif sp.split == "row":
                lo, hi = q3.shard_range(ref.shape[1], rank, world)
                ref = ref[:, lo:hi]
            assert torch.equal(_indices(obj, dev), ref), (rank, name)
        again = md.ModelDirWeights(tmp_path / "m", dev, rank=rank, world=world)
        assert again.shard_builds == 0 and again.shard_hits == W.shard_builds
        for name, obj in again.layers.items():
            assert torch.equal(_indices(obj, dev), _indices(W.layers[name], dev)), (rank, name)
