"""On-disk ``.npz`` layout of compressed tensors (reader and writer).

Keys and dtypes follow the reference's ``_save_cached_tensor`` /
``_load_cached_tensor`` (``src/compressor.py:144-243``):

* all modes: ``name`` (str), ``mode`` (str), ``shape`` (int array);
* ``direct_codebook``: ``codebook_type`` (``[str]``, default ``'mlp_ffn'``),
  ``bits`` (``[int]``), optional ``codebook`` (fp32 ``[C]``; absent when a
  global per-category codebook is used) and either ``indices`` (uint8
  fixed-width stream) or ``encoding=['huffman']`` with ``huff_lengths``,
  ``huff_stream``, ``huff_n`` and the six table keys;
* ``exact``: ``data`` (uint16 bf16 patterns);
* ``linear_quant``: ``indices``, ``scale``, ``v_min``, ``bits``.

A compressed model directory is ``<model>/codebook-lossless[-huffman]/`` with
``tensors/<name with '.' -> '_'>.npz``, ``codebooks/<type>_codebook.npy`` and
``metadata.json`` (``compress.py:91-97``, ``src/adaptive_compressor.py:1182-1247``).
Global codebooks are read as bf16 and widened to fp32, as the reference does.
"""
from __future__ import annotations

from pathlib import Path
from typing import Dict, Tuple

import numpy as np
import torch

__all__ = ["save_cached_tensor", "load_cached_tensor", "load_global_codebooks",
           "save_global_codebooks", "tensor_file", "HUFF_KEYS", "HUFF_TABLE_KEYS"]

HUFF_TABLE_KEYS = ("huff_row_bit_starts", "huff_lut_sym", "huff_lut_len", "huff_sl_first_code",
                   "huff_sl_base_offset", "huff_sl_sym")
HUFF_KEYS = ("huff_lengths", "huff_stream", "huff_n") + HUFF_TABLE_KEYS


def tensor_file(cache_dir, name: str) -> Path:
    """``tensors/<name with . replaced by _>.npz`` (src/adaptive_compressor.py:1041-1043)."""
    return Path(cache_dir) / "tensors" / (name.replace(".", "_") + ".npz")


def save_cached_tensor(npz_file, name: str, data: dict) -> None:
    """Write one tensor (``src/compressor.py:199-243``)."""
    d = {"name": name, "mode": data["mode"], "shape": np.asarray(data["shape"])}
    mode = data["mode"]
    if mode == "exact":
        d["data"] = data["data"]
    elif mode == "direct_codebook":
        d["codebook_type"] = np.array([data.get("codebook_type") or "mlp_ffn"])
        d["bits"] = np.array([int(data.get("bits", 8))])
        if data.get("codebook") is not None:
            d["codebook"] = np.asarray(data["codebook"], dtype=np.float32)
        if data.get("encoding") == "huffman":
            d["encoding"] = np.array(["huffman"])
            for k in HUFF_KEYS:
                if k in data and data[k] is not None:
                    d[k] = np.asarray(data[k])
        else:
            d["indices"] = np.asarray(data["indices"], dtype=np.uint8)
    elif mode == "linear_quant":
        d["indices"] = data["indices"]
        d["scale"] = np.array([data["scale"]])
        d["v_min"] = np.array([data["v_min"]])
        d["bits"] = np.array([int(data.get("bits", 8))])
    else:
        raise ValueError(f"unsupported mode {mode!r}")
    Path(npz_file).parent.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(npz_file, **d)


def load_cached_tensor(npz_file) -> Tuple[str, dict]:
    """Read one tensor (``src/compressor.py:144-196``): ``(name, data dict)``."""
    z = np.load(npz_file)
    mode = str(z["mode"])
    name = str(z["name"])
    out = {"mode": mode, "name": name, "shape": z["shape"]}
    if mode == "exact":
        out["data"] = z["data"]
    elif mode == "direct_codebook":
        out["codebook_type"] = str(z["codebook_type"][0])
        out["bits"] = int(z["bits"][0]) if "bits" in z.files else 8
        if "codebook" in z.files:
            out["codebook"] = z["codebook"]
        if "encoding" in z.files and str(z["encoding"][0]) == "huffman":
            out["encoding"] = "huffman"
            for k in HUFF_KEYS:
                if k in z.files:
                    out[k] = z[k]
        else:
            out["indices"] = z["indices"]
    elif mode == "linear_quant":
        out["indices"] = z["indices"]
        out["scale"] = float(z["scale"][0])
        out["v_min"] = float(z["v_min"][0])
        out["bits"] = int(z["bits"][0]) if "bits" in z.files else 8
    return name, out


def save_global_codebooks(cache_dir, codebooks: Dict[str, np.ndarray]) -> None:
    d = Path(cache_dir) / "codebooks"
    d.mkdir(parents=True, exist_ok=True)
    for ttype, cb in codebooks.items():
        np.save(d / f"{ttype}_codebook.npy", np.asarray(cb, dtype=np.float32))


def load_global_codebooks(cache_dir) -> Dict[str, torch.Tensor]:
    """``codebooks/*.npy`` -> {type: tensor}; read as bf16 then widened to fp32,
    like ``src/adaptive_compressor.py:1225-1247`` and ``chat.py:143-146``."""
    out = {}
    d = Path(cache_dir) / "codebooks"
    if not d.exists():
        return out
    for f in sorted(d.glob("*.npy")):
        out[f.stem.replace("_codebook", "")] = torch.from_numpy(np.load(f)).to(torch.bfloat16).float()
    return out
