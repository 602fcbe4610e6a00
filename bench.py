"""Benchmark: compressed decode throughput at Qwen3-8B shape, batch 1.

One step = one decode token through every compressed matrix of a Qwen3-8B
architecture model (36 layers x q,k,v,o,gate,up,down + lm_head; 12.3 GB of
13-bit streams) at T=1 with bf16 activations, chained layer to layer, with an
NCCL all-reduce after o_proj and down_proj when tensor-parallel (N > 1).
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
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


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

def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    import importlib
    import torch
    import torch.distributed as dist
    cbq = importlib.import_module(PKG)
    q3 = cbq.qwen3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    cfg = q3.QWEN3_8B if args.model == "qwen3-8b" else q3.QWEN3_1_7B
    t0 = time.time()
    W = q3.CompressedQwen3Weights(cfg, dev, huffman=args.huffman, rank=rank, world=world)
    setup_s = time.time() - t0
    L = W.layers
    names = [s.name for s in q3.linear_specs(cfg) if s.name != "model.embed_tokens.weight"]
    H = cfg.hidden

    def allreduce(t):
        if world > 1:
            dist.all_reduce(t)
        return t

    def step(x):
        """One token through the compressed linear stack (bf16, T=1)."""
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            q = L[p + "self_attn.q_proj.weight"](x)
            L[p + "self_attn.k_proj.weight"](x)
            L[p + "self_attn.v_proj.weight"](x)
            o = allreduce(L[p + "self_attn.o_proj.weight"](q))
            x = torch.nn.functional.rms_norm(x + o, (H,))
            g = L[p + "mlp.gate_proj.weight"](x)
            u = L[p + "mlp.up_proj.weight"](x)
            dn = allreduce(L[p + "mlp.down_proj.weight"](torch.nn.functional.silu(g) * u))
            x = torch.nn.functional.rms_norm(x + dn, (H,))
        return L["lm_head.weight"](x)

    x0 = torch.randn(1, H, device=dev).to(torch.bfloat16)
    for _ in range(args.warmup):
        step(x0)
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

    with ClockSampler(local) as clk:
        ms = timed(lambda: step(x0), args.steps)
    ms_step = ms / args.steps
    value = 1000.0 / ms_step

    # end to end: pinned host input in, lm_head logits out, every step
    x_host = x0.cpu().pin_memory()
    out_host = torch.empty((1, cfg.vocab // world), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        xd = x_host.to(dev, non_blocking=True)
        y = step(xd)
        out_host.copy_(y, non_blocking=True)
    for _ in range(2):
        e2e_step()
    ms_e2e = timed(e2e_step, args.steps) / args.steps

    # dominant kernel: gate_proj decode-GEMV over all layers' weights (2.9 GB > L2)
    gates = [L[f"model.layers.{i}.mlp.gate_proj.weight"] for i in range(cfg.layers)]
    xg = torch.randn(1, H, device=dev).to(torch.bfloat16)
    reps = 5
    for g in gates:
        g(xg)
    gms = timed(lambda: [g(xg) for g in gates], reps) / (reps * len(gates))
    g0 = gates[0]
    alg = W.stream_bytes["model.layers.0.mlp.gate_proj.weight"] + 4 * W.codebooks["mlp_ffn"].numel() \
        + 2 * H + 2 * g0.M
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

    launches = args.steps * (len(names))
    stack_bytes = W.total_stream_bytes()
    if rank == 0:
        line = {
            "metric": "compressed decode tok/s (Qwen3-8B shape, bs1)", "value": value, "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded bf16 N(0,0.02) weights, lossless per-category codebooks)",
            "config": {"workload": f"{cfg.name} decode linear stack (36 layers x 7 GEMVs + lm_head), bs1, "
                                   f"{'huffman' if args.huffman else 'fixed 13-bit'}",
                       "global_batch": 1, "parallelism": f"tp{world}",
                       "l2": "inputs 12.3 GB >> 126 MB L2 (no flush)",
                       "stream_bytes_per_rank": stack_bytes,
                       "hbm_gbs_whole_step": stack_bytes / (ms_step * 1e-3) / 1e9,
                       "setup_s": round(setup_s, 1)},
            "roofline": {"kernel": "k_linear_fixed<13,1,bf16,bf16> (gate_proj 12288x4096)" if not args.huffman
                         else "k_linear_huff<1,bf16,bf16> (gate_proj)",
                         "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "traffic": None,
                         "alg_bytes_per_launch": alg, "us_per_launch": gms * 1e3},
            "e2e": {"value": 1000.0 / ms_e2e, "unit": "tok/s", "h2d_bytes_per_step": 2 * H,
                    "d2h_bytes_per_step": 2 * (cfg.vocab // world)},
            "gpu_launches": launches,
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
