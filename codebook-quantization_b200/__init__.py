"""B200-native codebook decode-matmul (drop-in for the compressed linear-layer
path of bigattichouse/Codebook-Quantization).

The directory name is not a Python identifier, so import it with
``importlib.import_module("codebook-quantization_b200")``.

Public API (mirrors the reference's module and binding names):

* ``AdaptiveCodebookLinear``, ``AdaptiveCodebookEmbedding`` -- nn.Modules with
  ``from_compressed(name, data, global_codebooks, ...)``;
* ``GPUAcceleratedLinear`` / ``GPUAcceleratedEmbedding`` (fixed width) and
  ``HuffmanCodebookLinear`` / ``HuffmanCodebookEmbedding`` (canonical Huffman);
* ``bitpack``, ``huffman_codebook``, ``npz_format`` -- the on-disk format;
* ``host_stream`` -- flat ``.idx`` files, ``MmappedPackedBuffer`` and
  ``HostStreamedLinear`` (stream kept in host memory, copied per call);
* ``model_dir`` -- compressed model directories (``codebook-lossless[-huffman]/``
  ``tensors/*.npz`` + ``codebooks/*.npy``): reader into the decoder, writer;
* ``synth`` -- seeded synthetic tensors; ``_lib`` -- the ctypes binding of
  ``libcbq.so`` (C ABI in ``include/cbq.h``).
"""
from . import _lib, bitpack, huffman_codebook, npz_format, qwen3, synth, tp_shard  # noqa: F401
from . import host_stream, model_dir  # noqa: F401
from .host_stream import HostStreamedLinear, MmappedPackedBuffer, export_flat_idx  # noqa: F401
from .compressed_modules import AdaptiveCodebookEmbedding, AdaptiveCodebookLinear  # noqa: F401
from .gpu_accelerated_functions import GPUAcceleratedEmbedding, GPUAcceleratedLinear  # noqa: F401
from .gpu_huffman_functions import HuffmanCodebookEmbedding, HuffmanCodebookLinear  # noqa: F401

build_library = _lib.build_library
__version__ = "0.1.0"
