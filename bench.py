"""Benchmark: compressed greedy decode throughput at Qwen3-8B shape, batch 1.

One step = one greedy decode token of a Qwen3-8B-architecture model whose
every matrix stays compressed (36 layers x q,k,v,o,gate,up,down + lm_head +
embedding; 12.3 GB of 13-bit streams), bf16 activations, KV cache, the whole
step replayed from one CUDA graph, with an NCCL all-reduce after o_proj and
down_proj when tensor-parallel (N > 1).
Weights are seeded synthetic bf16 N(0, 0.02) compressed losslessly on the GPU
with one codebook per category.  The 12.3 GB of inputs is
~100x the 126 MB L2, so no flush is needed between steps.

Reported (one JSON line on rank 0): ``value`` tok/s (device-timed, max over
ranks), ``e2e`` (host-pinned input copied in and the lm_head output copied out
every step, through the same public API), ``roofline`` of the dominant kernel
(gate_proj's decode-GEMV, timed with CUDA events over all 36 layers' weights),
``cpu_baseline`` (the reference's own compressed_matmul.c on the host cores
over a bounded sample), SM clocks sampled during the timed region.

``--impl reference``: the reference's CPU implementation of the same path
(oracle/_ref, built unmodified from its compressed_matmul.c) on all host
threads; each step is a bounded sample (layer 0's seven matrices and 1/64 of
lm_head) scaled to tok/s of the full model.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
PKG = "codebook-quantization_b200"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="cbq", choices=["cbq", "reference"])
    ap.add_argument("--huffman", action="store_true", help="Huffman-coded streams instead of fixed width")
    ap.add_argument("--model", default="qwen3-8b", choices=["qwen3-8b", "qwen3-1.7b"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--no-graph", action="store_true", help="eager steps instead of a CUDA graph")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="decode", choices=["decode", "gemv", "prefill"],
                    help="decode: Qwen3 greedy decode (headline); gemv: one matrix shape, GB/s")
    ap.add_argument("--shape", default="12288,4096", help="gemv workload: M,K")
    ap.add_argument("--tokens", type=int, default=1, help="gemv workload: T (activation rows)")
    ap.add_argument("--x-dtype", default="bf16", choices=["bf16", "f32"], help="gemv workload: activation dtype")
    ap.add_argument("--fuse-norm", action="store_true",
                    help="decode: RMSNorm in the last CTA of the GEMV before it instead of its own launch")
    ap.add_argument("--split-rope", action="store_true",
                    help="decode: q/k norm + rope as its own launch instead of in the attention launch")
    ap.add_argument("--allreduce", default="peer", choices=["peer", "nccl"],
                    help="tensor parallelism: fused peer-memory all-reduce or NCCL")
    return ap.parse_args()


# DRAM bytes (read + write) per launch of the dominant kernel, measured once
# with ncu on the same shape (profiles/<kernel>_gemv_12288x4096_t1.md); the
# roofline's `traffic`.  Keyed by (kernel, M, K, tokens).
NCU_TRAFFIC = {
    ("k_gemv_fixed", 12288, 4096, 1): 81.880832e6 + 2.562048e6,
    ("k_gemv_huff", 12288, 4096, 1): 72.563456e6 + 1.255424e6,
}


def gemv_kernel_name(huffman: bool, tokens: int, x_bf16: bool = True) -> str:
    """The kernel cbq_linear_fixed / cbq_linear_huff dispatch to for `tokens` rows."""
    if huffman:
        return "k_gemv_huff" if tokens == 1 else "k_linear_huff"
    if tokens <= 2:
        return "k_gemv_fixed"
    return "k_gemm_fixed" if tokens >= 64 and x_bf16 else "k_linear_fixed"


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi SM clock / throttle sampling during the timed region."""
    Q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 6:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[2 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ------------------------------------------------------------------ CPU baseline (reference code)

def cpu_reference_sample(cfg, seed: int = 0):
    """Bounded CPU sample of one token on the reference's compressed_matmul.c:
    layer 0's seven matrices plus 1/64 of lm_head's rows, scaled to the full
    model.  Returns (tok/s, seconds per token, threads, description)."""
    sys.path.insert(0, str(REPO / "oracle"))
    import importlib
    import oracle
    cbq = importlib.import_module(PKG)
    q3 = cbq.qwen3
    L = oracle.ref_lib()
    kind = "reference"
    if L is None:
        kind = "port"
    specs = {s.name: s for s in q3.linear_specs(cfg)}
    sample = [n for n in specs if n.startswith("model.layers.0.")]
    lm_rows = cfg.vocab // 64
    mats = []
    for n in sample + ["lm_head.weight"]:
        sp = specs[n]
        M, K = sp.shape
        if n == "lm_head.weight":
            M = lm_rows
        bf = cbq.synth.bf16_normal_np((M, K), seed=q3.tensor_seed(sp.source, seed))
        d = cbq.synth.compress_fixed_np(bf)
        x = np.random.default_rng(1).standard_normal((1, K)).astype(np.float32)
        mats.append((n, M, K, d, x))

    def run_once():
        t = {}
        for n, M, K, d, x in mats:
            t0 = time.perf_counter()
            if kind == "reference":
                oracle.ref_linear_fixed(x, d["indices"], d["codebook"], M, K, d["bits"])
            else:
                oracle.linear_fixed(x, d["indices"], d["codebook"], M, K, d["bits"])
            t[n] = time.perf_counter() - t0
        layer = sum(v for k, v in t.items() if k != "lm_head.weight")
        return cfg.layers * layer + 64 * t["lm_head.weight"]
    run_once()
    return run_once, kind, ("one token = 36 x layer-0 (q,k,v,o,gate,up,down) + 64 x 1/64 of lm_head rows, "
                            "13-bit fixed width, T=1, fp32, one call over all rows")


def reference_arm(args):
    """--impl reference: the reference's CPU path, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import importlib
    cbq = importlib.import_module(PKG)
    cfg = cbq.qwen3.QWEN3_8B if args.model == "qwen3-8b" else cbq.qwen3.QWEN3_1_7B
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    run_once, kind, desc = cpu_reference_sample(cfg)
    for _ in range(args.warmup):
        run_once()
    secs = [run_once() for _ in range(args.steps)]
    sec = float(np.mean(secs))
    v = 1.0 / sec
    line = {"metric": "compressed decode tok/s (Qwen3-8B shape, bs1)", "value": v, "unit": "tok/s",
            "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded bf16 N(0,0.02), lossless 13-bit)",
            "config": {"workload": f"{cfg.name} decode linear stack, bs1, fixed width", "global_batch": 1},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": oracle.threads(), "kind": kind,
                             "sample": desc},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm

def graph_time_ms(torch, fn, reps, dev):
    """Average ms of fn() captured once in a CUDA graph and replayed reps times."""
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    g.replay()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize(dev)
    return a.elapsed_time(b) / reps


def gemv_workload(args):
    """One compressed matrix shape: R distinct seeded copies (> 2x L2 in total)
    decode-GEMV'd in turn from a CUDA graph; reports GB/s over algorithmic bytes."""
    import importlib
    import torch
    cbq = importlib.import_module(PKG)
    dev = torch.device("cuda", 0)
    M, K = (int(v) for v in args.shape.split(","))
    T = args.tokens
    comp = cbq.synth.GpuCompressor(dev)
    per = (M * K * 13) // 8
    R = max(2, min(64, (512 << 20) // max(per, 1) + 1))
    mats, alg = [], 0
    for r in range(R):
        bits = cbq.synth.bf16_normal_gpu((M, K), seed=1000 + r, device=dev)
        d = comp.compress(bits, huffman=args.huffman)
        if args.huffman:
            lin = cbq.HuffmanCodebookLinear("g", d["huff_stream"], d["huff_lengths"], int(d["huff_n"][0]),
                                            d["codebook"], (M, K), d["bits"],
                                            huff_row_bit_starts=d["huff_row_bit_starts"], device=dev)
            b = lin.hs.compressed_bytes
        else:
            lin = cbq.GPUAcceleratedLinear("g", d["indices"], d["codebook"], (M, K), d["bits"], device=dev)
            b = (M * K * d["bits"] + 7) // 8
        alg += b + 4 * lin.C + (2 if args.x_dtype == "bf16" else 4) * (K + M) * T
        mats.append(lin)
        del bits, d
    xdt = torch.bfloat16 if args.x_dtype == "bf16" else torch.float32
    x = torch.randn(T, K, device=dev).to(xdt)
    outs = [torch.empty(T, M, device=dev, dtype=xdt) for _ in mats]
    for _ in range(args.warmup):
        for m, o in zip(mats, outs):
            m(x, out=o)
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        ms = graph_time_ms(torch, lambda: [m(x, out=o) for m, o in zip(mats, outs)], args.steps, dev)
    us = ms * 1e3 / R
    gbs = alg / R / (us * 1e-6) / 1e9
    peak, peak_kind = measured_peaks()
    kern = gemv_kernel_name(args.huffman, T, args.x_dtype == "bf16")
    line = {"metric": "compressed GEMV GB/s vs HBM", "value": gbs, "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": args.x_dtype,
            "data": "synthetic seeded bf16 N(0,0.02), lossless per-matrix codebook",
            "config": {"workload": f"{kern} {M}x{K} T={T} {'huffman' if args.huffman else 'fixed'}",
                       "copies": R, "l2": f"{R} distinct matrices rotated (> 2x L2)",
                       "bits": mats[0].bits},
            "roofline": {"kernel": kern, "bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                         "frac": gbs / peak, "peak_kind": peak_kind,
                         "traffic": NCU_TRAFFIC.get((kern, M, K, T)),
                         "alg_bytes_per_launch": alg / R, "us_per_launch": us},
            "gpu_launches": args.steps * R, "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


def prefill_workload(args):
    """a compressed 12288 x 4096 (13-bit) matrix times a
    bf16 activation block of 4096 tokens on the tensor cores; TFLOP/s."""
    import importlib
    import torch
    cbq = importlib.import_module(PKG)
    dev = torch.device("cuda", 0)
    M, K = (int(v) for v in args.shape.split(","))
    T = args.tokens if args.tokens > 1 else 4096
    comp = cbq.synth.GpuCompressor(dev)
    mats = []
    for r in range(2):                                        # two copies, alternated
        bits = cbq.synth.bf16_normal_gpu((M, K), seed=2000 + r, device=dev)
        d = comp.compress(bits, huffman=False)
        mats.append(cbq.GPUAcceleratedLinear("w", d["indices"], d["codebook"], (M, K), d["bits"], device=dev))
        del bits, d
    x = torch.randn(T, K, device=dev).to(torch.bfloat16)
    outs = [torch.empty(T, M, device=dev, dtype=torch.bfloat16) for _ in mats]
    for _ in range(args.warmup):
        for m, o in zip(mats, outs):
            m(x, out=o)
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        ms = graph_time_ms(torch, lambda: [m(x, out=o) for m, o in zip(mats, outs)], args.steps, dev)
    us = ms * 1e3 / len(mats)
    flops = 2.0 * M * K * T
    tflops = flops / (us * 1e-6) / 1e12
    peaks = {}
    try:
        peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    peak = peaks.get("bf16_tflops") or 1590.0
    line = {"metric": "compressed prefill GEMM TFLOP/s (bf16 tensor cores)", "value": tflops, "unit": "TFLOP/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic seeded bf16 N(0,0.02) weights (13-bit lossless), bf16 N(0,1) activations",
            "config": {"workload": f"k_gemm_fixed {M}x{K} x {T} tokens", "copies": len(mats),
                       "bits": mats[0].bits},
            "roofline": {"kernel": "k_gemm_fixed", "bound": "tensor", "achieved": tflops, "peak": peak,
                         "unit": "TFLOP/s", "frac": tflops / peak,
                         "peak_kind": "measured" if peaks.get("bf16_tflops") else "fallback", "traffic": None,
                         "flops_per_launch": flops, "us_per_launch": us},
            "gpu_launches": args.steps * len(mats), "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    if args.workload == "gemv":
        return gemv_workload(args)
    if args.workload == "prefill":
        return prefill_workload(args)
    import importlib
    import torch
    import torch.distributed as dist
    cbq = importlib.import_module(PKG)
    q3 = cbq.qwen3
    from importlib import import_module
    qd = import_module(PKG + ".qwen3_decode")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=180))
        group = dist.group.WORLD
    cfg = q3.QWEN3_8B if args.model == "qwen3-8b" else q3.QWEN3_1_7B
    t0 = time.time()
    W = q3.CompressedQwen3Weights(cfg, dev, huffman=args.huffman, rank=rank, world=world)
    setup_s = time.time() - t0
    H = cfg.hidden
    prompt_len = 64
    max_len = prompt_len + args.warmup + 2 * args.steps + 8
    dec = qd.Qwen3Decoder(W, batch=args.batch, max_len=max_len, act_dtype=torch.bfloat16, group=group,
                          allreduce=args.allreduce, fuse_norm=args.fuse_norm, fuse_rope=not args.split_rope)
    g = torch.Generator().manual_seed(1234)
    prompt = torch.randint(0, cfg.vocab, (args.batch, prompt_len), generator=g)
    if not args.no_graph:
        dec.capture()
    dec.reset()
    dec.generate(prompt, 1)                      # prompt fills the cache (untimed)
    for _ in range(args.warmup):                 # greedy decode steps, untimed
        dec.ids.copy_(dec.next_ids)
        dec.run_step()
        dec.pos.add_(1)
    torch.cuda.synchronize()

    def timed(fn, n):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def decode_step():
        dec.ids.copy_(dec.next_ids)
        dec.run_step()
        dec.pos.add_(1)

    with ClockSampler(local) as clk, torch.cuda.nvtx.range("cbq_timed"):
        ms = timed(decode_step, args.steps)
    ms_step = ms / args.steps
    value = args.batch * 1000.0 / ms_step

    # end to end: the token id goes host -> device and the next one device -> host every step
    ids_host = dec.next_ids.cpu().pin_memory()
    next_host = torch.empty_like(ids_host).pin_memory()

    def e2e_step():
        dec.ids.copy_(ids_host, non_blocking=True)
        dec.run_step()
        dec.pos.add_(1)
        next_host.copy_(dec.next_ids, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        ids_host.copy_(next_host)
    ms_e2e = timed(e2e_step, args.steps) / args.steps
    dec.release()

    # dominant kernel: gate_proj decode-GEMV over all 36 layers' weights (graph-replayed)
    gates = [W.layers[f"model.layers.{i}.mlp.gate_proj.weight"] for i in range(cfg.layers)]
    xg = torch.randn(args.batch, H, device=dev).to(torch.bfloat16)
    outs = [torch.empty(args.batch, gt.M, device=dev, dtype=torch.bfloat16) for gt in gates]
    gms = graph_time_ms(torch, lambda: [gt(xg, out=o) for gt, o in zip(gates, outs)], 20, dev) / len(gates)
    g0 = gates[0]
    cbn = W.codebooks["mlp_ffn"].numel()
    alg = W.stream_bytes["model.layers.0.mlp.gate_proj.weight"] + 4 * cbn + 2 * H * args.batch \
        + 2 * g0.M * args.batch
    peak, peak_kind = measured_peaks()
    achieved = alg / (gms * 1e-3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        run_once, kind, desc = cpu_reference_sample(cfg)
        sys.path.insert(0, str(REPO / "oracle"))
        import oracle
        secs = [run_once() for _ in range(3)]
        cpu = {"value": 1.0 / float(np.mean(secs)), "unit": "tok/s", "cores": oracle.threads(),
               "kind": kind, "sample": desc}

    n_lin = len([s for s in q3.linear_specs(cfg)])          # embedding + 7 per layer + lm_head
    stack_bytes = W.total_stream_bytes()
    if rank == 0:
        line = {
            "metric": "compressed decode tok/s (Qwen3-8B shape, bs1)", "value": value, "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded bf16 N(0,0.02) weights, lossless per-category codebooks, "
                    "64 seeded prompt tokens)",
            "config": {"workload": f"{cfg.name} greedy decode, batch {args.batch}, "
                                   f"{'huffman' if args.huffman else 'fixed 13-bit'} streams, CUDA graph",
                       "global_batch": args.batch, "seq_len": max_len, "parallelism": f"tp{world}",
                       "allreduce": ("peer-memory (GEMV epilogue + RMSNorm)" if dec.peer is not None
                                     else ("nccl" if world > 1 else "none")),
                       "launches_per_layer": ("q/k/v, attention" + ("" if dec.fuse_rope else " (+ q/k norm rope)")
                                              + ", o" + (" + norm" if dec.fuse_norm else ", norm")
                                              + ", gate/up, down" + (" + norm" if dec.fuse_norm else ", norm")),
                       "l2": "weights 12.3 GB >> 126 MB L2 (no flush)",
                       "stream_bytes_per_rank": stack_bytes,
                       "hbm_gbs_whole_step": stack_bytes / (ms_step * 1e-3) / 1e9,
                       "setup_s": round(setup_s, 1)},
            "roofline": {"kernel": gemv_kernel_name(args.huffman, args.batch) + f" gate_proj {g0.M}x{g0.K}",
                         "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": NCU_TRAFFIC.get((gemv_kernel_name(args.huffman, args.batch), g0.M, g0.K,
                                                     args.batch)),
                         "alg_bytes_per_launch": alg, "us_per_launch": gms * 1e3,
                         "timing": "CUDA-graph replay of the 36 gate_proj launches, CUDA events"},
            "e2e": {"value": args.batch * 1000.0 / ms_e2e, "unit": "tok/s",
                    "h2d_bytes_per_step": 8 * args.batch, "d2h_bytes_per_step": 8 * args.batch},
            "gpu_launches": args.steps * dec.launches_per_step(),
            "clocks": clk.summary(),
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
