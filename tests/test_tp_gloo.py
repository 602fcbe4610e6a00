"""Tensor-parallel sharding of compressed tensors, world size 2 over gloo (CPU).

Each rank cuts its shard of a compressed matrix with ``tp_shard`` (rows for a
column-parallel layer, columns for a row-parallel one, fixed-width and
Huffman), checks the shard decodes to exactly its block of the unsharded
indices, multiplies it with the CPU oracle, and the ranks combine the results
the way the decoder does on NCCL: rows are gathered (bit-identical to the
unsharded product), column partials are all-reduced (fp32 tolerance 1e-6).
"""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]
M, K, BITS_SEED = 192, 768, 21


def _free_port() -> int:
    """A bindable port below the kernel's ephemeral range, so that a port an
    earlier test's connections still hold (TIME_WAIT) is not handed out."""
    import random
    for _ in range(100):
        port = random.randrange(20000, 30000)
        with socket.socket() as s:
            try:
                s.bind(("127.0.0.1", port))
            except OSError:
                continue
            return port
    raise RuntimeError("no free port")


def _matrix(kind: str):
    from helpers import cbq
    bf = cbq.synth.bf16_normal_np((M, K), seed=BITS_SEED)
    if kind == "fixed":
        return cbq.synth.compress_fixed_np(bf)
    return cbq.synth.compress_huffman_np(bf)


def _rank_main(rank: int, world: int, port: int, kind: str, split: str, q):
    try:
        sys.path[:0] = [str(REPO / "oracle"), str(REPO), str(REPO / "tests")]
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch
        import torch.distributed as dist
        import oracle
        from helpers import cbq
        tp = cbq.tp_shard
        dist.init_process_group("gloo", rank=rank, world_size=world)
        d = _matrix(kind)
        cb, bits, idx = d["codebook"], int(d["bits"]), d["_idx"].reshape(M, K)
        x = np.random.default_rng(5).standard_normal((2, K)).astype(np.float32)
        if kind == "fixed":
            full = oracle.linear_fixed(x, d["indices"], cb, M, K, bits)
        else:
            full = oracle.huff_linear(x, d, cb, M, K)
        if split == "rows":
            r0, r1 = tp.shard_range(M, rank, world)
            Ms, Ks, xs, blk = r1 - r0, K, x, idx[r0:r1]
            if kind == "fixed":
                packed = tp.shard_fixed_rows(d["indices"], M, K, bits, r0, r1)
            else:
                sd = tp.shard_huffman_rows(d, M, K, r0, r1)
        else:
            c0, c1 = tp.shard_range(K, rank, world)
            Ms, Ks, xs, blk = M, c1 - c0, np.ascontiguousarray(x[:, c0:c1]), idx[:, c0:c1]
            if kind == "fixed":
                packed = tp.shard_fixed_cols(d["indices"], M, K, bits, c0, c1)
            else:
                dec = oracle.huff_decode_rows(d, M, K).reshape(M, K)
                sd = tp.shard_huffman_cols(d, dec, c0, c1)
        if kind == "fixed":
            got_idx = oracle.unpack_fixed(packed, bits, Ms * Ks).reshape(Ms, Ks)
            part = oracle.linear_fixed(xs, packed, cb, Ms, Ks, bits)
        else:
            got_idx = oracle.huff_decode_rows(sd, Ms, Ks).reshape(Ms, Ks)
            part = oracle.huff_linear(xs, sd, cb, Ms, Ks)
        assert np.array_equal(got_idx, blk), "shard does not decode to its block"
        t = torch.from_numpy(part)
        if split == "rows":
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            got = torch.cat(parts, dim=1).numpy()
            assert np.array_equal(got, full), "gathered rows differ from the unsharded product"
        else:
            dist.all_reduce(t)
            got = t.numpy()
            rel = np.linalg.norm(got - full) / np.linalg.norm(full)
            assert rel < 1e-6, f"all-reduced partials off by {rel:.2e}"
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except BaseException as e:                                 # report to the parent, never hang it
        q.put((rank, f"{type(e).__name__}: {e}"))


@pytest.mark.parametrize("kind", ["fixed", "huffman"])
@pytest.mark.parametrize("split", ["rows", "cols"])
def test_tp2_shards_reproduce_the_unsharded_product(kind, split):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, kind, split, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        r, msg = q.get(timeout=120)
        results[r] = msg
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert results == {0: "ok", 1: "ok"}, results


def test_bit_shifts_move_ranges_exactly():
    from helpers import cbq
    tp = cbq.tp_shard
    rng = np.random.default_rng(0)
    src = rng.integers(0, 256, size=64, dtype=np.uint8)
    bits_msb = np.unpackbits(src)                              # MSB-first bit order
    bits_lsb = np.unpackbits(src, bitorder="little")
    for b0, n in [(0, 0), (0, 13), (3, 100), (7, 1), (9, 400), (31, 33)]:
        got = np.unpackbits(tp.shift_bits_msb(src, b0, n))[:n]
        assert np.array_equal(got, bits_msb[b0:b0 + n])
        got = np.unpackbits(tp.shift_bits_lsb(src, b0, n), bitorder="little")[:n]
        assert np.array_equal(got, bits_lsb[b0:b0 + n])


def test_shard_range_rejects_uneven_splits():
    from helpers import cbq
    with pytest.raises(ValueError):
        cbq.tp_shard.shard_range(10, 0, 3)
    assert cbq.tp_shard.shard_range(12, 2, 3) == (8, 12)
