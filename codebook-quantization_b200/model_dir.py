"""Compressed model directories: the loader path of the reference, B200 side.

The reference stores a compressed model as
``<model>/codebook-lossless[-huffman]/`` with ``tensors/<name with '.' ->
'_'>.npz`` (one file per tensor, ``src/compressor.py:199-243``),
``codebooks/<type>_codebook.npy`` (one global codebook per category, read as
bf16, ``src/adaptive_compressor.py:1225-1247``) and ``metadata.json``, next
to the HF ``config.json``; ``CompressedModelLoader`` walks the model and
replaces each ``nn.Linear`` / ``nn.Embedding`` with a compressed module built
from its ``.npz`` (``src/model_loader.py:205-281``; a tied ``lm_head`` with no
file of its own reuses ``model.embed_tokens``'s, ``:233-236``).

Here :class:`ModelDirWeights` reads such a directory straight into the
device-resident objects the decoder runs (``Qwen3Decoder`` takes it in place
of the synthetic ``CompressedQwen3Weights``), and
:func:`write_qwen3_model_dir` writes one from seeded synthetic weights.

Derived data never changes the ``.npz`` files.  Under tensor parallelism each
rank cuts its shard on the GPU (fixed width: unpack, slice, re-pack; Huffman
rows: re-based bit range; Huffman columns: decode and re-encode with the
tensor's own code lengths) and caches the result in
``<cache>/derived/tp<W>/rank<r>/<file>.npz`` (uncompressed), keyed by the
source file's size and modification time, so a second load of the same
shard reads it back instead of re-cutting it.
"""
from __future__ import annotations

import json
import os
from pathlib import Path
from typing import Dict, Optional

import numpy as np
import torch

from . import _lib, huffman_codebook as hc, npz_format, qwen3, synth, tp_shard
from .compressed_modules import _select_codebook
from .gpu_accelerated_functions import (GPUAcceleratedEmbedding, GPUAcceleratedLinear, device_stream,
                                        padded_device_bytes)
from .gpu_huffman_functions import HuffmanCodebookEmbedding, HuffmanCodebookLinear

__all__ = ["cache_dir_for", "read_qwen3_config", "write_qwen3_model_dir", "ModelDirWeights"]

_HF_KEYS = {"layers": "num_hidden_layers", "hidden": "hidden_size", "inter": "intermediate_size",
            "heads": "num_attention_heads", "kv_heads": "num_key_value_heads", "head_dim": "head_dim",
            "vocab": "vocab_size", "rope_theta": "rope_theta", "tie_embeddings": "tie_word_embeddings",
            "rms_eps": "rms_norm_eps"}


def cache_dir_for(model_dir, huffman: bool) -> Path:
    """``<model>/codebook-lossless`` or ``<model>/codebook-lossless-huffman``
    (the reference appends ``-huffman`` for entropy-coded caches,
    ``src/adaptive_compressor.py:434-435``)."""
    return Path(model_dir) / ("codebook-lossless-huffman" if huffman else "codebook-lossless")


def read_qwen3_config(model_dir) -> qwen3.Qwen3Config:
    """The decoder shape from an HF ``config.json``."""
    c = json.loads((Path(model_dir) / "config.json").read_text())
    kw = {f: c[k] for f, k in _HF_KEYS.items() if k in c}
    if "head_dim" not in kw:
        kw["head_dim"] = c["hidden_size"] // c["num_attention_heads"]
    return qwen3.Qwen3Config(name=str(c.get("_name_or_path") or Path(model_dir).name), **kw)


def _config_json(cfg: qwen3.Qwen3Config) -> dict:
    d = {k: getattr(cfg, f) for f, k in _HF_KEYS.items()}
    d.update(model_type="qwen3", architectures=["Qwen3ForCausalLM"], torch_dtype="bfloat16",
             _name_or_path=cfg.name)
    return d


def _np(v):
    return v.cpu().numpy() if isinstance(v, torch.Tensor) else v


def write_qwen3_model_dir(cfg: qwen3.Qwen3Config, model_dir, huffman: bool = False, seed: int = 0,
                          device=None, std: float = 0.02) -> Path:
    """Write a compressed Qwen3-architecture model directory from seeded
    synthetic bf16 N(0, std) weights (the values ``CompressedQwen3Weights``
    builds with the same seed): one global codebook per category, no
    per-tensor codebook key, norms exact (not stored: unit weights)."""
    device = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    model_dir = Path(model_dir)
    model_dir.mkdir(parents=True, exist_ok=True)
    (model_dir / "config.json").write_text(json.dumps(_config_json(cfg), indent=1))
    out = cache_dir_for(model_dir, huffman)
    comp = synth.GpuCompressor(device)
    specs = qwen3.linear_specs(cfg)
    hist: Dict[str, torch.Tensor] = {}
    for sp in specs:
        if sp.seed_name:
            continue
        bits = synth.bf16_normal_gpu(sp.shape, qwen3.tensor_seed(sp.source, seed), device, std)
        h = comp.histogram(bits)
        hist[sp.category] = h if sp.category not in hist else hist[sp.category] + h
    cbs, luts = {}, {}
    for cat, h in hist.items():
        cbs[cat], luts[cat] = comp.codebook(h)
    npz_format.save_global_codebooks(out, {k: v.cpu().numpy() for k, v in cbs.items()})
    info = {}
    for sp in specs:
        if sp.seed_name:
            continue                                     # tied lm_head: the loader reuses embed_tokens
        bits = synth.bf16_normal_gpu(sp.shape, qwen3.tensor_seed(sp.source, seed), device, std)
        d = comp.compress(bits, huffman=huffman, codebook=cbs[sp.category], lut=luts[sp.category],
                          codebook_type=sp.category, keep_codebook=False)
        d = {k: _np(v) for k, v in d.items()}
        npz_format.save_cached_tensor(npz_format.tensor_file(out, sp.name), sp.name, d)
        info[sp.name] = {"shape": list(sp.shape), "mode": "direct_codebook", "codebook_type": sp.category,
                         "bits": int(d["bits"])}
    meta = {"compression_method": "adaptive_v2", "compression_mode": "lossless", "tensor_count": len(info),
            "codebook_sizes": {k: int(v.numel()) for k, v in cbs.items()}, "tensor_info": info,
            "entropy_code": bool(huffman)}
    (out / "metadata.json").write_text(json.dumps(meta, indent=1))
    return model_dir


def _source_key(path: Path) -> str:
    st = os.stat(path)
    return f"{st.st_size}:{st.st_mtime_ns}"


class ModelDirWeights:
    """Every compressed matrix of one rank, read from a model directory and
    resident on its GPU; the interface ``Qwen3Decoder`` uses
    (``cfg, device, huffman, rank, world, layers, codebooks, stream_bytes``).

    ``huffman=None`` picks ``codebook-lossless`` when present, else the
    ``-huffman`` directory.  ``derived_cache=False`` re-cuts tensor-parallel
    shards on every load instead of reading and writing the shard cache.
    """

    def __init__(self, model_dir, device, rank: int = 0, world: int = 1, huffman: Optional[bool] = None,
                 cfg: Optional[qwen3.Qwen3Config] = None, derived_cache: bool = True):
        model_dir = Path(model_dir)
        if huffman is None:
            huffman = not cache_dir_for(model_dir, False).exists()
        self.cache = cache_dir_for(model_dir, huffman)
        if not self.cache.exists():
            raise FileNotFoundError(f"no compressed cache at {self.cache}")
        self.cfg = cfg or read_qwen3_config(model_dir)
        self.device = torch.device(device)
        self.huffman, self.rank, self.world = huffman, rank, world
        self.derived_cache = derived_cache
        self.shard_hits = 0
        self.shard_builds = 0
        gcb = npz_format.load_global_codebooks(self.cache)
        self.codebooks: Dict[str, torch.Tensor] = {}
        self.layers: Dict[str, object] = {}
        self.stream_bytes: Dict[str, int] = {}
        for sp in qwen3.linear_specs(self.cfg):
            path = npz_format.tensor_file(self.cache, sp.name)
            if not path.exists() and sp.name == "lm_head.weight":
                path = npz_format.tensor_file(self.cache, "model.embed_tokens.weight")
            if not path.exists():
                raise FileNotFoundError(f"{sp.name}: missing {path}")
            data = self._shard(sp, path)
            cb = _select_codebook(data, gcb, default_type=sp.category)
            if cb is None:
                raise ValueError(f"{sp.name}: no codebook for {data.get('codebook_type')!r}")
            key = data.get("codebook_type") or sp.category
            if key not in self.codebooks or data.get("codebook") is not None:
                cbd = cb.to(self.device)
                if data.get("codebook") is None:
                    self.codebooks[key] = cbd
            else:
                cbd = self.codebooks[key]
            shape = tuple(int(s) for s in np.asarray(data["shape"]).reshape(-1))
            is_emb = sp.name == "model.embed_tokens.weight"
            if data.get("encoding") == "huffman":
                cls = HuffmanCodebookEmbedding if is_emb else HuffmanCodebookLinear
                obj = cls(sp.name, data["huff_stream"], data["huff_lengths"], int(np.asarray(data["huff_n"])[0]),
                          cbd, shape, int(data["bits"]), huff_row_bit_starts=data["huff_row_bit_starts"],
                          device=self.device)
                self.stream_bytes[sp.name] = obj.hs.compressed_bytes
            else:
                cls = GPUAcceleratedEmbedding if is_emb else GPUAcceleratedLinear
                obj = cls(sp.name, data["indices"], cbd, shape, int(data["bits"]), device=self.device)
                self.stream_bytes[sp.name] = (shape[0] * shape[1] * int(data["bits"]) + 7) // 8
            self.layers[sp.name] = obj
        torch.cuda.synchronize(self.device)

    def total_stream_bytes(self, include_embedding: bool = False) -> int:
        return sum(v for k, v in self.stream_bytes.items()
                   if include_embedding or k != "model.embed_tokens.weight")

    # ------------------------------------------------------------ sharding
    def _shard(self, sp: qwen3.LinearSpec, path: Path) -> dict:
        """This rank's part of the tensor in ``path`` (the whole tensor at TP = 1
        or for replicated tensors); cut once and cached."""
        _, data = npz_format.load_cached_tensor(path)
        if self.world == 1 or sp.split == "rep":
            return data
        if data["mode"] != "direct_codebook":
            raise ValueError(f"{sp.name}: mode {data['mode']!r} is not served by the compressed kernels")
        derived = self.cache / "derived" / f"tp{self.world}" / f"rank{self.rank}" / path.name
        src_key = f"{_source_key(path)}:{sp.split}"
        if self.derived_cache and derived.exists():
            z = np.load(derived, allow_pickle=False)
            if str(z["source_key"]) == src_key:
                self.shard_hits += 1
                out = dict(data)
                for k in list(out):
                    if k == "indices" or k.startswith("huff_"):
                        del out[k]
                for k in z.files:
                    if k != "source_key":
                        out[k] = z[k]
                out["shape"] = z["shape"]
                return out
        out = self._cut(sp, data)
        self.shard_builds += 1
        if self.derived_cache:
            derived.parent.mkdir(parents=True, exist_ok=True)
            keep = {k: np.asarray(v) for k, v in out.items()
                    if k == "indices" or k == "shape" or k.startswith("huff_")}
            tmp = derived.with_name(derived.stem + f".tmp{os.getpid()}.npz")
            np.savez(tmp, source_key=np.array(src_key), **keep)
            os.replace(tmp, derived)
        return out

    def _cut(self, sp: qwen3.LinearSpec, data: dict) -> dict:
        M, K = (int(s) for s in np.asarray(data["shape"]).reshape(-1))
        rows = sp.split == "col"
        lo, hi = tp_shard.shard_range(M if rows else K, self.rank, self.world)
        out = dict(data)
        if data.get("encoding") == "huffman":
            if rows:
                out.update(tp_shard.shard_huffman_rows(data, M, K, lo, hi))
            else:
                idx = _gpu_huffman_indices(data, M, K, self.device)[:, lo:hi].contiguous()
                out.update(_gpu_huffman_encode(idx, data["huff_lengths"], self.device))
            out["shape"] = np.array([hi - lo, K] if rows else [M, hi - lo])
            return out
        bits = int(data["bits"])
        if rows:
            out["indices"] = tp_shard.shard_fixed_rows(data["indices"], M, K, bits, lo, hi)
        else:
            out["indices"] = _gpu_fixed_cols(data["indices"], M, K, bits, lo, hi, self.device)
        out["shape"] = np.array([hi - lo, K] if rows else [M, hi - lo])
        return out


def _gpu_fixed_cols(indices, M: int, K: int, bits: int, c0: int, c1: int, device) -> np.ndarray:
    """Columns [c0, c1) of a fixed-width stream, re-packed at the same width on the GPU."""
    nbytes = _lib.query("cbq_fixed_stream_bytes", M, K, bits)
    packed = padded_device_bytes(np.asarray(indices, dtype=np.uint8)[:(M * K * bits + 7) // 8], nbytes, device)
    idx = torch.empty(M * K + 1, dtype=torch.int16, device=device)
    _lib.call("cbq_unpack_fixed", packed.data_ptr(), nbytes, bits, M * K, idx.data_ptr(), device_stream(device))
    sub = idx[:M * K].view(M, K)[:, c0:c1].contiguous()
    return synth.GpuCompressor(device).pack_fixed(sub, bits).cpu().numpy()


def _gpu_huffman_indices(data: dict, M: int, K: int, device) -> torch.Tensor:
    """The decoded index matrix [M, K] (int16 holding uint16) of a Huffman tensor."""
    from .gpu_huffman_functions import HuffmanStream
    hs = HuffmanStream("shard", data["huff_stream"], data["huff_lengths"], int(np.asarray(data["huff_n"])[0]),
                       (M, K), data["huff_row_bit_starts"], device)
    idx = hs.decode_indices()
    hs.check()
    return idx.to(torch.int16)


def _gpu_huffman_encode(idx: torch.Tensor, lengths, device) -> dict:
    """Encode an index matrix with the canonical code of ``lengths`` on the
    GPU (the tensor's own code, so decoded indices stay identical)."""
    m, k = idx.shape
    lengths = np.asarray(lengths, dtype=np.uint8)
    codes, _ = hc.canonical_codes(lengths)
    flat = idx.reshape(-1)
    sym = flat.to(torch.int64) & 0xFFFF
    len_d = torch.from_numpy(lengths).to(device)
    code_d = torch.from_numpy(codes.astype(np.uint32).view(np.int32)).to(device)
    n = flat.numel()
    if n and (int(sym.max().item()) >= lengths.size or bool((len_d[sym] == 0).any().item())):
        raise ValueError("an index has no code in the tensor's code lengths")
    sym_len = len_d[sym].to(torch.int64)
    starts = torch.cumsum(sym_len, 0) - sym_len
    total = int((starts[-1] + sym_len[-1]).item()) if n else 0
    nbytes = (total + 7) // 8
    buf = torch.empty(((nbytes + 3) // 4) * 4 + 8, dtype=torch.uint8, device=device)
    _lib.call("cbq_huff_encode", flat.data_ptr(), n, code_d.data_ptr(), len_d.data_ptr(), starts.data_ptr(),
              buf.data_ptr(), buf.numel(), device_stream(device))
    stream = np.zeros(nbytes + 4, dtype=np.uint8)
    stream[:nbytes] = buf[:nbytes].cpu().numpy()
    rbs = starts[::k].cpu().numpy().astype(np.int64) if n else np.zeros(max(m, 1), dtype=np.int64)
    return {"huff_stream": stream, "huff_row_bit_starts": rbs, "huff_n": np.array([n], dtype=np.int64)}
