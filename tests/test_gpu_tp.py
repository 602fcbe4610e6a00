"""Tensor-parallel decode on two GPUs: the greedy tokens of a TP=2 model equal
those of the same model on one GPU (fp32 activations; only the summation order
of the all-reduced partial products differs), with the row-parallel layers'
all-reduce done by the fused peer-memory path (GEMV epilogue writes into every
rank's slot; the RMSNorm kernel, or the GEMV's last CTA, sums) or by NCCL.  Skipped on machines with
fewer than two GPUs."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

from helpers import cbq

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parents[1]
CFG = cbq.qwen3.Qwen3Config("tiny-tp", 2, 256, 512, 4, 2, 64, 1000, 1e6, False)


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


def _prompt():
    return torch.randint(0, CFG.vocab, (2, 12), generator=torch.Generator().manual_seed(8))


def _rank_main(rank, world, port, fused, huffman, q, allreduce="peer", fuse_norm=False):
    try:
        sys.path[:0] = [str(REPO), str(REPO / "tests")]
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        from datetime import timedelta
        import importlib
        import torch.distributed as dist
        from helpers import cbq as pkg
        qd = importlib.import_module("codebook-quantization_b200.qwen3_decode")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=timedelta(seconds=60))
        W = pkg.qwen3.CompressedQwen3Weights(CFG, dev, huffman=huffman, rank=rank, world=world, seed=3)
        dec = qd.Qwen3Decoder(W, batch=2, max_len=40, act_dtype=torch.float32, group=dist.group.WORLD,
                              fused=fused, allreduce=allreduce, fuse_norm=fuse_norm)
        peer = dec.peer is not None
        eager = dec.generate(_prompt(), 12).cpu()
        dec.reset()
        dec.capture()
        dec.reset()
        graphed = dec.generate(_prompt(), 12).cpu()
        dec.release()
        if peer and int(dec.peer.status[0].item()) != 0:
            raise RuntimeError(f"peer all-reduce reported status {dec.peer.status.tolist()}")
        del dec
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok" if (peer or allreduce != "peer" or not fused or huffman) else "peer path not used",
               eager.tolist(), graphed.tolist()))
    except BaseException as e:
        q.put((rank, f"{type(e).__name__}: {e}", None, None))


@pytest.mark.parametrize("fused,allreduce,fuse_norm", [(True, "peer", False), (True, "peer", True),
                                                      (True, "nccl", False), (False, "nccl", False)],
                         ids=["fused-peer", "fused-peer-norm", "fused-nccl", "torch-ops"])
@pytest.mark.parametrize("huffman", [False, True], ids=["fixed", "huffman"])
def test_tp2_decode_matches_one_gpu(fused, allreduce, fuse_norm, huffman):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import importlib
    qd = importlib.import_module("codebook-quantization_b200.qwen3_decode")
    W = cbq.qwen3.CompressedQwen3Weights(CFG, torch.device("cuda", 0), huffman=huffman, seed=3)
    ref = qd.Qwen3Decoder(W, batch=2, max_len=40, act_dtype=torch.float32, fused=fused).generate(
        _prompt(), 12).cpu().tolist()
    del W
    ctx = mp.get_context("spawn")
    for attempt in range(3):                    # a rendezvous port taken meanwhile: another port
        q = ctx.Queue()
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, 2, port, fused, huffman, q, allreduce, fuse_norm))
                 for r in range(2)]
        for p in procs:
            p.start()
        res = {}
        for _ in procs:
            r, msg, eager, graphed = q.get(timeout=300)
            res[r] = (msg, eager, graphed)
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
        if not any("EADDRINUSE" in str(m[0]) for m in res.values()):
            break
    for r in range(2):
        msg, eager, graphed = res[r]
        assert msg == "ok", (r, msg)
        assert eager == graphed, r
        assert eager == ref, (r, eager, ref)
