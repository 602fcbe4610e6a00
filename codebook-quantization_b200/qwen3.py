"""Qwen3-architecture compressed models: configuration, seeded synthetic
weights (compressed on the GPU) and tensor-parallel sharding.

Weights follow BASELINE configs 3 and 5: every linear and the embedding is
bf16 N(0, 0.02) compressed losslessly with ONE codebook per category
(``attention`` for q/k/v/o, ``mlp_ffn`` for gate/up/down, ``embedding`` for
embed_tokens and lm_head -- the reference's ``classify_tensor``,
``src/compressor.py:37-92``); norms stay exact (ones).  Each tensor is seeded
by its name, so every rank regenerates identical full tensors and keeps its
shard.

Tensor parallelism (``world > 1``): q, k, v, gate, up and lm_head are split by
output rows (column-parallel), o and down by input columns (row-parallel,
followed by an all-reduce).  Both splits act on the index matrix before
packing, so each shard's stream decodes to exactly the unsharded model's
indices for its slice.
"""
from __future__ import annotations

import zlib
from dataclasses import dataclass
from typing import Dict, List, Tuple

import torch

from . import synth
from .gpu_accelerated_functions import GPUAcceleratedEmbedding, GPUAcceleratedLinear
from .gpu_huffman_functions import HuffmanCodebookEmbedding, HuffmanCodebookLinear

__all__ = ["Qwen3Config", "QWEN3_1_7B", "QWEN3_8B", "LinearSpec", "linear_specs", "tensor_seed",
           "CompressedQwen3Weights"]


@dataclass(frozen=True)
class Qwen3Config:
    name: str
    layers: int
    hidden: int
    inter: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    rope_theta: float = 1e6
    tie_embeddings: bool = False
    rms_eps: float = 1e-6


QWEN3_1_7B = Qwen3Config("qwen3-1.7b", 28, 2048, 6144, 16, 8, 128, 151936, 1e6, True)
QWEN3_8B = Qwen3Config("qwen3-8b", 36, 4096, 12288, 32, 8, 128, 151936, 1e6, False)


@dataclass(frozen=True)
class LinearSpec:
    name: str
    shape: Tuple[int, int]          # full (out, in)
    category: str
    split: str                      # "col" (rows split), "row" (cols split) or "rep"
    seed_name: str = ""             # tensor whose seed generates the weights (tied lm_head)

    @property
    def source(self) -> str:
        return self.seed_name or self.name


def linear_specs(cfg: Qwen3Config) -> List[LinearSpec]:
    """Every compressed matrix of the model, in forward order."""
    h, q, kv = cfg.hidden, cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    out = [LinearSpec("model.embed_tokens.weight", (cfg.vocab, h), "embedding", "rep")]
    for i in range(cfg.layers):
        p = f"model.layers.{i}."
        out += [
            LinearSpec(p + "self_attn.q_proj.weight", (q, h), "attention", "col"),
            LinearSpec(p + "self_attn.k_proj.weight", (kv, h), "attention", "col"),
            LinearSpec(p + "self_attn.v_proj.weight", (kv, h), "attention", "col"),
            LinearSpec(p + "self_attn.o_proj.weight", (h, q), "attention", "row"),
            LinearSpec(p + "mlp.gate_proj.weight", (cfg.inter, h), "mlp_ffn", "col"),
            LinearSpec(p + "mlp.up_proj.weight", (cfg.inter, h), "mlp_ffn", "col"),
            LinearSpec(p + "mlp.down_proj.weight", (h, cfg.inter), "mlp_ffn", "row"),
        ]
    out.append(LinearSpec("lm_head.weight", (cfg.vocab, h), "embedding", "col",
                          "model.embed_tokens.weight" if cfg.tie_embeddings else ""))
    return out


def tensor_seed(name: str, base: int = 0) -> int:
    return (zlib.crc32(name.encode()) ^ (base * 0x9E3779B1)) & 0x7FFFFFFF


def shard_range(n: int, rank: int, world: int) -> Tuple[int, int]:
    if n % world:
        raise ValueError(f"dimension {n} does not split over {world} ranks")
    s = n // world
    return rank * s, (rank + 1) * s


class CompressedQwen3Weights:
    """All compressed matrices of one rank, resident on its GPU.

    ``layers[name]`` is a GPUAccelerated*/Huffman* object holding this rank's
    shard; ``codebooks[category]`` the shared fp32 codebook (on the device);
    ``stream_bytes[name]`` the algorithmic bytes one pass over it reads.
    """

    def __init__(self, cfg: Qwen3Config, device, huffman: bool = False, rank: int = 0, world: int = 1,
                 seed: int = 0, std: float = 0.02, keep_indices: bool = False):
        self.cfg, self.device, self.huffman = cfg, torch.device(device), huffman
        self.rank, self.world = rank, world
        comp = synth.GpuCompressor(self.device)
        specs = linear_specs(cfg)
        hist: Dict[str, torch.Tensor] = {}
        for sp in specs:                                     # pass 1: category histograms
            if sp.seed_name:
                continue                                     # tied: same values as its source
            bits = synth.bf16_normal_gpu(sp.shape, tensor_seed(sp.source, seed), self.device, std)
            h = comp.histogram(bits)
            hist[sp.category] = h if sp.category not in hist else hist[sp.category] + h
            del bits
        self.codebooks, luts = {}, {}
        for cat, h in hist.items():
            self.codebooks[cat], luts[cat] = comp.codebook(h)
        self.layers: Dict[str, object] = {}
        self.stream_bytes: Dict[str, int] = {}
        self.indices: Dict[str, torch.Tensor] = {}
        for sp in specs:                                     # pass 2: shard + compress
            bits = synth.bf16_normal_gpu(sp.shape, tensor_seed(sp.source, seed), self.device, std)
            M, K = sp.shape
            if sp.split == "col" and world > 1:
                r0, r1 = shard_range(M, rank, world)
                bits = bits[r0:r1]
            elif sp.split == "row" and world > 1:
                c0, c1 = shard_range(K, rank, world)
                bits = bits[:, c0:c1]
            bits = bits.contiguous()
            cb = self.codebooks[sp.category]
            d = comp.compress(bits, huffman=huffman, codebook=cb, lut=luts[sp.category],
                              codebook_type=sp.category, keep_codebook=False)
            if keep_indices:
                self.indices[sp.name] = comp.indices(bits, luts[sp.category])
            shape = tuple(bits.shape)
            is_emb = sp.name == "model.embed_tokens.weight"
            if huffman:
                cls = HuffmanCodebookEmbedding if is_emb else HuffmanCodebookLinear
                obj = cls(sp.name, d["huff_stream"], d["huff_lengths"], int(d["huff_n"][0]), cb, shape,
                          d["bits"], huff_row_bit_starts=d["huff_row_bit_starts"], device=self.device)
                self.stream_bytes[sp.name] = obj.hs.compressed_bytes
            else:
                cls = GPUAcceleratedEmbedding if is_emb else GPUAcceleratedLinear
                obj = cls(sp.name, d["indices"], cb, shape, d["bits"], device=self.device)
                self.stream_bytes[sp.name] = (shape[0] * shape[1] * d["bits"] + 7) // 8
            self.layers[sp.name] = obj
            del bits, d
        torch.cuda.synchronize(self.device)

    def total_stream_bytes(self, include_embedding: bool = False) -> int:
        return sum(v for k, v in self.stream_bytes.items()
                   if include_embedding or k != "model.embed_tokens.weight")
