"""Host-resident streams on the GPU: HostStreamedLinear keeps the packed
indices in host memory (a pinned copy, or a memory-mapped flat .idx file
page-locked in place) and copies them to the device in row chunks per call
(cbq_linear_fixed_streamed), the B200 form of the reference's mmap path
(tests/test_mmap_inference.py: mmap output equals RAM output).

Checked against the device-resident GPUAcceleratedLinear and the C oracle
(rel-L2 1e-5: the chunks run the same kernels, only the one/two-token
kernel's unit size can differ with the chunk's row count), with staging
buffers small enough to force many chunks, on two calls in a row, inside a
CUDA graph, and through AdaptiveCodebookLinear.from_compressed(use_mmap=True).
"""
import numpy as np
import pytest
import torch

import oracle
from helpers import cbq, need_cuda, rel_l2

pytestmark = pytest.mark.gpu
HS = cbq.host_stream


def _case(M, K, bits, seed):
    rng = np.random.default_rng(seed)
    packed = rng.integers(0, 256, size=(M * K * bits + 7) // 8, dtype=np.uint8)
    cb = (rng.standard_normal((1 << bits) - 5) * 0.02).astype(np.float32)
    return packed, cb


@pytest.mark.parametrize("src", ["ram", "mmap"])
@pytest.mark.parametrize("M,K,bits,T,dt,staging", [(3000, 1024, 13, 1, torch.bfloat16, 1 << 20),
                                                   (1000, 4096, 12, 2, torch.float32, 3 << 20),
                                                   (777, 2048, 13, 8, torch.bfloat16, 1 << 20),
                                                   (900, 512, 8, 64, torch.bfloat16, 1 << 18)])
def test_host_streamed_matches_device_resident(tmp_path, src, M, K, bits, T, dt, staging):
    dev = need_cuda()
    packed, cb = _case(M, K, bits, seed=M + K + T)
    if src == "mmap":
        f = tmp_path / "w.idx"
        packed.tofile(f)
        host = HS.MmappedPackedBuffer(f)
    else:
        host = packed
    lin = HS.HostStreamedLinear("w", host, cb, (M, K), bits, device=dev, staging_bytes=staging)
    assert (M + lin.chunk_rows - 1) // lin.chunk_rows >= 3           # several chunks, both buffers reused
    ref_lin = cbq.GPUAcceleratedLinear("w", packed, cb, (M, K), bits, device=dev)
    for call in range(2):
        x = torch.randn(T, K, device=dev).to(dt)
        got = lin(x, out_dtype=torch.float32)
        ref = ref_lin(x, out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert rel_l2(got.cpu().numpy(), ref.cpu().numpy()) < 1e-5, call
        if T <= 8:
            want = oracle.linear_fixed(x.float().cpu().numpy(), packed, cb, M, K, bits)
            assert rel_l2(got.cpu().numpy(), want) < 1e-5, call
    lin.close()


def test_host_streamed_in_a_cuda_graph():
    dev = need_cuda()
    M, K, bits = 2048, 2048, 13
    packed, cb = _case(M, K, bits, seed=5)
    lin = HS.HostStreamedLinear("w", packed, cb, (M, K), bits, device=dev, staging_bytes=2 << 20)
    x = torch.randn(1, K, device=dev).to(torch.bfloat16)
    out = torch.empty(1, M, device=dev, dtype=torch.bfloat16)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        lin(x, out=out)
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        lin(x, out=out)
    x.copy_(torch.randn(1, K, device=dev).to(torch.bfloat16))
    g.replay()
    torch.cuda.synchronize()
    want = oracle.linear_fixed(x.float().cpu().numpy(), packed, cb, M, K, bits)
    assert rel_l2(out.float().cpu().numpy(), want) < 1e-2                # bf16 output rounding
    del g
    lin.close()


def test_adaptive_linear_use_mmap_streams_from_the_idx_file(tmp_path):
    dev = need_cuda()
    M, K, bits = 1536, 1024, 13
    packed, cb = _case(M, K, bits, seed=9)
    name = "model.layers.0.mlp.down_proj.weight"
    data = {"mode": "direct_codebook", "shape": np.array([M, K]), "bits": bits, "codebook_type": "mlp_ffn",
            "codebook": cb, "indices": packed}
    cbq.npz_format.save_cached_tensor(cbq.npz_format.tensor_file(tmp_path, name), name, data)
    assert HS.export_flat_idx(tmp_path, "tensors") == 1
    idx_file = tmp_path / "tensors" / (name.replace(".", "_") + ".idx")
    _, loaded = cbq.npz_format.load_cached_tensor(cbq.npz_format.tensor_file(tmp_path, name))
    layer = cbq.AdaptiveCodebookLinear.from_compressed(name, loaded, {}, use_mmap=True, idx_file=idx_file, device=dev)
    assert isinstance(layer._gpu_func, HS.HostStreamedLinear) and layer._mmap_buf is not None
    resident = cbq.AdaptiveCodebookLinear.from_compressed(name, loaded, {}, device=dev)
    x = torch.randn(3, K, device=dev)
    y, y_ref = layer(x), resident(x)
    torch.cuda.synchronize()
    assert rel_l2(y.cpu().numpy(), y_ref.cpu().numpy()) < 1e-5
    layer._gpu_func.close()
