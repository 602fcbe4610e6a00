"""Benchmark: compressed greedy decode throughput at Qwen3-8B shape, batch 1.

One step = one greedy decode token of a Qwen3-8B-architecture model whose
every matrix stays compressed (36 layers x q,k,v,o,gate,up,down + lm_head +
embedding; 12.3 GB of 13-bit streams), bf16 activations, KV cache, the whole
step replayed from one CUDA graph; under tensor parallelism (N > 1) the
row-parallel layers' partial products are all-reduced over NVLink peer memory
inside the GEMV epilogue (or by NCCL, ``--allreduce nccl``).
Weights are seeded synthetic bf16 N(0, 0.02) compressed losslessly on the GPU
with one codebook per category.  The 12.3 GB of inputs is
~100x the 126 MB L2, so no flush is needed between steps.  The prompt has 64
tokens and the timed steps are the last ones of a 128-token generation
(positions up to 64 + 128).

Reported (one JSON line on rank 0): ``value`` tok/s (device-timed, max over
ranks), ``e2e`` (the token id copied host -> device and the next id device ->
host every step, through the same public API), ``roofline`` of the dominant
kernel (gate_proj's decode-GEMV, timed with CUDA events over all 36 layers'
weights), ``cpu_baseline`` (the reference's own compressed_matmul.c on the
host cores over a bounded sample), SM clocks sampled during the timed region.
At N = 1 ``sub_results`` carries the other BASELINE configurations, each with
its own roofline and clocks: config 1 (2048x2048 GEMV), config 2 (Huffman
GEMVs at Qwen3-1.7B MLP shapes), config 3 (Qwen3-1.7B decode, 30 greedy
tokens), config 4 (prefill GEMM, fixed width and Huffman), config 5 variants
(128-token block, Huffman streams, batch 8) and the batch-8 GEMV.  At N > 1
``tp_tokens_match`` reports a greedy-token check of a small tensor-parallel
model (fp32 activations, fixed width over peer memory and NCCL, Huffman over
NCCL) against the same model unsharded on each rank's GPU, run before the
timed region.

``--impl reference``: the reference's CPU implementation of the same path
(oracle/_ref, built unmodified from its compressed_matmul.c) on all host
cores; each step is a bounded sample of one token (layer 0's seven matrices
with its norms and attention, and 1/64 of lm_head's rows), timed whole;
``value`` is the full token's tok/s extrapolated from the sample (36 layers,
64 lm_head slices).
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
import traceback
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
PKG = "codebook-quantization_b200"
PROMPT_LEN = 64          # config 5: 64-token prompt, 128 greedy tokens
GEN_TOKENS = 128


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
    ap.add_argument("--no-sub", action="store_true", help="headline only (no sub_results / tp check)")
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


# DRAM bytes (read + write) per launch of a kernel, from one ncu capture of
# the same kernel and shape (`ncu --metrics
# dram__bytes_read.sum,dram__bytes_write.sum -k regex:<kernel> ... python
# bench.py --workload gemv --shape M,K`); the roofline's `traffic`.  Keyed by
# (kernel, M, K, tokens); shapes not captured report null.
NCU_TRAFFIC = {
    ("k_gemv_fixed", 12288, 4096, 1): 81.880832e6 + 2.562048e6,
    ("k_gemv_fixed", 6144, 4096, 1): 40.997376e6,          # gate_proj rows of one rank at TP2
    ("k_gemv_fixed", 3072, 4096, 1): 20.549120e6,          # TP4
    ("k_gemv_fixed", 1536, 4096, 1): 10.324736e6,          # TP8
    ("k_gemv_huff", 12288, 4096, 1): 72.563456e6 + 1.255424e6,
}


def gemv_kernel_name(huffman: bool, tokens: int, x_bf16: bool = True) -> str:
    """The kernel cbq_linear_fixed / cbq_linear_huff dispatch to for `tokens` rows."""
    if huffman:
        if tokens >= 64 and x_bf16:
            return "k_huff_transcode + k_gemm_fixed"
        return "k_gemv_huff" if tokens == 1 else "k_linear_huff"
    if tokens <= 2:
        return "k_gemv_fixed"
    return "k_gemm_fixed" if tokens >= 64 and x_bf16 else "k_linear_fixed"


def peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm": float(d["hbm_gbs"]), "bf16": float(d["bf16_tflops"]),
                "bf16_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "kind": "measured"}
    return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "kind": "fallback"}


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
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)                     # the sampler is running before the timed work starts
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

def _cpu_layer_glue(cfg, pos: int, torch):
    """The non-linear work of one decoder layer at position ``pos`` on the CPU
    in fp32 torch ops (the reference runs these as HF modules around its C
    kernels): two RMSNorms, q/k norms + rotary, attention over pos + 1 keys."""
    d, hq, hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
    g = torch.Generator().manual_seed(3)
    x = torch.randn(1, cfg.hidden, generator=g)
    q = torch.randn(1, hq, 1, d, generator=g)
    kc = torch.randn(1, hkv, pos + 1, d, generator=g)
    vc = torch.randn(1, hkv, pos + 1, d, generator=g)

    def rms(v):
        return v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + cfg.rms_eps)

    def run():
        rms(x), rms(x)
        qq = rms(q)
        kk = rms(kc[:, :, -1:])
        qq = qq * 0.5 + torch.cat((-qq[..., d // 2:], qq[..., :d // 2]), -1) * 0.5
        kk = kk * 0.5 + torch.cat((-kk[..., d // 2:], kk[..., :d // 2]), -1) * 0.5
        torch.nn.functional.scaled_dot_product_attention(qq, kc, vc, scale=d ** -0.5, enable_gqa=True)
    return run


def cpu_reference_sample(cfg, seed: int = 0):
    """Bounded CPU sample of one token on the reference's compressed_matmul.c,
    all host cores: layer 0 (seven matrices, norms, attention) plus 1/64 of
    lm_head's rows.  Returns (run_once, kind, description, cores); run_once()
    times the whole sample and returns (sample seconds, extrapolated seconds
    per token = 36 x layer + 64 x lm_head slice)."""
    sys.path.insert(0, str(REPO / "oracle"))
    import importlib
    import torch
    import oracle
    cbq = importlib.import_module(PKG)
    q3 = cbq.qwen3
    cores = oracle.set_threads(oracle.host_cores())
    torch.set_num_threads(cores)
    L = oracle.ref_lib()
    kind = "reference" if L is not None else "port"
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
    glue = _cpu_layer_glue(cfg, PROMPT_LEN + GEN_TOKENS // 2, torch)

    def run_once():
        t0 = time.perf_counter()
        glue()
        for n, M, K, d, x in mats:
            if n == "lm_head.weight":
                t1 = time.perf_counter()
            if kind == "reference":
                oracle.ref_linear_fixed(x, d["indices"], d["codebook"], M, K, d["bits"])
            else:
                oracle.linear_fixed(x, d["indices"], d["codebook"], M, K, d["bits"])
        t2 = time.perf_counter()
        layer, lm = t1 - t0, t2 - t1
        return t2 - t0, cfg.layers * layer + 64 * lm
    run_once()
    desc = (f"one step = layer 0 of {cfg.name} (q,k,v,o,gate,up,down on compressed_matmul.c, one call over all "
            f"rows; RMSNorms, q/k norm + rope, attention at position {PROMPT_LEN + GEN_TOKENS // 2} in torch "
            f"fp32) + 1/64 of lm_head rows, 13-bit fixed width, T=1; tok/s extrapolated as "
            f"{cfg.layers} x layer + 64 x lm_head slice")
    return run_once, kind, desc, cores


def reference_arm(args):
    """--impl reference: the reference's CPU path, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import importlib
    cbq = importlib.import_module(PKG)
    cfg = cbq.qwen3.QWEN3_8B if args.model == "qwen3-8b" else cbq.qwen3.QWEN3_1_7B
    run_once, kind, desc, cores = cpu_reference_sample(cfg)
    for _ in range(args.warmup):
        run_once()
    t0 = time.perf_counter()
    res = [run_once() for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    sample_s = float(np.mean([r[0] for r in res]))
    token_s = float(np.mean([r[1] for r in res]))
    v = 1.0 / token_s
    line = {"metric": "compressed decode tok/s (Qwen3-8B shape, bs1)", "value": v, "unit": "tok/s",
            "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": sample_s * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded bf16 N(0,0.02), lossless 13-bit)",
            "config": {"workload": f"{cfg.name} greedy decode, batch 1, fixed 13-bit streams (bounded sample "
                                   "per step)", "global_batch": 1},
            "timed_region_s": wall, "ms_per_token_extrapolated": token_s * 1e3,
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": kind, "sample": desc},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm: single matrices

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
    del g
    return a.elapsed_time(b) / reps


def gemv_line(shape, tokens, huffman, x_dtype, steps, warmup):
    """One compressed matrix shape: R distinct seeded copies (> 2x L2 in total)
    decode-GEMV'd in turn from a CUDA graph; GB/s over algorithmic bytes."""
    import importlib
    import torch
    cbq = importlib.import_module(PKG)
    dev = torch.device("cuda", 0)
    M, K = shape
    T = tokens
    comp = cbq.synth.GpuCompressor(dev)
    per = (M * K * 13) // 8
    R = max(2, min(64, (512 << 20) // max(per, 1) + 1))
    mats, alg = [], 0
    xb = 2 if x_dtype == "bf16" else 4
    for r in range(R):
        bits = cbq.synth.bf16_normal_gpu((M, K), seed=1000 + r, device=dev)
        d = comp.compress(bits, huffman=huffman)
        if huffman:
            lin = cbq.HuffmanCodebookLinear("g", d["huff_stream"], d["huff_lengths"], int(d["huff_n"][0]),
                                            d["codebook"], (M, K), d["bits"],
                                            huff_row_bit_starts=d["huff_row_bit_starts"], device=dev)
            b = lin.hs.compressed_bytes
        else:
            lin = cbq.GPUAcceleratedLinear("g", d["indices"], d["codebook"], (M, K), d["bits"], device=dev)
            b = (M * K * d["bits"] + 7) // 8
        alg += b + 4 * lin.C + xb * (K + M) * T
        mats.append(lin)
        del bits, d
    xdt = torch.bfloat16 if x_dtype == "bf16" else torch.float32
    x = torch.randn(T, K, device=dev).to(xdt)
    outs = [torch.empty(T, M, device=dev, dtype=xdt) for _ in mats]
    for _ in range(warmup):
        for m, o in zip(mats, outs):
            m(x, out=o)
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        ms = graph_time_ms(torch, lambda: [m(x, out=o) for m, o in zip(mats, outs)], steps, dev)
    us = ms * 1e3 / R
    gbs = alg / R / (us * 1e-6) / 1e9
    pk = peaks()
    kern = gemv_kernel_name(huffman, T, x_dtype == "bf16")
    bits = mats[0].bits
    del mats, outs
    torch.cuda.empty_cache()
    return {"metric": "compressed GEMV GB/s vs HBM", "value": gbs, "unit": "GB/s", "n_gpus": 1,
            "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": x_dtype,
            "data": "synthetic seeded bf16 N(0,0.02), lossless per-matrix codebook",
            "config": {"workload": f"{kern} {M}x{K} T={T} {'huffman' if huffman else 'fixed'} x {x_dtype}",
                       "copies": R, "l2": f"{R} distinct matrices rotated (> 2x L2)", "bits": bits},
            "roofline": {"kernel": kern, "bound": "hbm", "achieved": gbs, "peak": pk["hbm"], "unit": "GB/s",
                         "frac": gbs / pk["hbm"], "peak_kind": pk["kind"],
                         "traffic": NCU_TRAFFIC.get((kern, M, K, T)),
                         "alg_bytes_per_launch": alg / R, "us_per_launch": us},
            "gpu_launches": steps * R, "clocks": clk.summary()}


def prefill_line(shape, tokens, huffman, steps, warmup):
    """a compressed 12288 x 4096 (13-bit) matrix times a
    bf16 activation block of 4096 tokens on the tensor cores; TFLOP/s."""
    import importlib
    import torch
    cbq = importlib.import_module(PKG)
    dev = torch.device("cuda", 0)
    M, K = shape
    T = tokens
    comp = cbq.synth.GpuCompressor(dev)
    mats = []
    for r in range(2):                                        # two copies, alternated
        bits = cbq.synth.bf16_normal_gpu((M, K), seed=2000 + r, device=dev)
        d = comp.compress(bits, huffman=huffman)
        if huffman:
            mats.append(cbq.HuffmanCodebookLinear("w", d["huff_stream"], d["huff_lengths"], int(d["huff_n"][0]),
                                                  d["codebook"], (M, K), d["bits"],
                                                  huff_row_bit_starts=d["huff_row_bit_starts"], device=dev))
        else:
            mats.append(cbq.GPUAcceleratedLinear("w", d["indices"], d["codebook"], (M, K), d["bits"], device=dev))
        del bits, d
    x = torch.randn(T, K, device=dev).to(torch.bfloat16)
    outs = [torch.empty(T, M, device=dev, dtype=torch.bfloat16) for _ in mats]
    for _ in range(warmup):
        for m, o in zip(mats, outs):
            m(x, out=o)
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        ms = graph_time_ms(torch, lambda: [m(x, out=o) for m, o in zip(mats, outs)], steps, dev)
    us = ms * 1e3 / len(mats)
    flops = 2.0 * M * K * T
    tflops = flops / (us * 1e-6) / 1e12
    pk = peaks()
    kern = gemv_kernel_name(huffman, T, True)
    bits = mats[0].bits
    del mats, outs
    torch.cuda.empty_cache()
    return {"metric": "compressed prefill GEMM TFLOP/s (bf16 tensor cores)", "value": tflops, "unit": "TFLOP/s",
            "n_gpus": 1, "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic seeded bf16 N(0,0.02) weights (13-bit lossless), bf16 N(0,1) activations",
            "config": {"workload": f"{kern} {M}x{K} x {T} tokens {'huffman' if huffman else 'fixed'}",
                       "copies": 2, "bits": bits},
            "roofline": {"kernel": kern, "bound": "tensor", "achieved": tflops, "peak": pk["bf16"],
                         "unit": "TFLOP/s", "frac": tflops / pk["bf16"], "peak_kind": pk["kind"] + " (burst)",
                         "traffic": None, "flops_per_launch": flops, "us_per_launch": us},
            "gpu_launches": steps * 2, "clocks": clk.summary()}


# ------------------------------------------------------------------ GPU arm: decode

def timed_ms(torch, dist, fn, n, world, dev):
    """ms of n calls of fn, CUDA events on the current stream, barrier +
    synchronize on both sides, max over ranks."""
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


def decode_run(W, batch, steps, warmup, world, group, dev, local, allreduce="peer", fuse_norm=False,
               split_rope=False, graph=True, prompt_len=PROMPT_LEN, gen=GEN_TOKENS, e2e=True, block=False):
    """Greedy decode of ``W``: prompt fills the cache, untimed steps advance to
    the end of the generation, then ``warmup`` untimed and ``steps`` timed
    steps (and ``steps`` end-to-end ones) end at position prompt + gen.
    ``block``: time all ``gen`` generated tokens as one region instead."""
    import importlib
    import torch
    import torch.distributed as dist
    qd = importlib.import_module(PKG + ".qwen3_decode")
    cfg = W.cfg
    max_len = prompt_len + gen + 8
    dec = qd.Qwen3Decoder(W, batch=batch, max_len=max_len, act_dtype=torch.bfloat16, group=group,
                          allreduce=allreduce, fuse_norm=fuse_norm, fuse_rope=not split_rope)
    g = torch.Generator().manual_seed(1234)
    prompt = torch.randint(0, cfg.vocab, (batch, prompt_len), generator=g)
    if graph:
        dec.capture()
    dec.reset()
    dec.generate(prompt, 1)                      # the prompt fills the cache (untimed)

    def step():
        dec.ids.copy_(dec.next_ids)
        dec.run_step()
        dec.pos.add_(1)
    res = {}
    if block:
        for _ in range(warmup):                  # warm-up at the start of the generation, then rewind
            step()
        dec.pos.fill_(prompt_len)
        torch.cuda.synchronize()
        with ClockSampler(local) as clk:
            ms = timed_ms(torch, dist, step, gen, world, dev)
        res.update(ms_step=ms / gen, clocks=clk.summary(), timed_steps=gen)
    else:
        n_timed = steps * (2 if e2e else 1)
        pre = max(0, gen - n_timed - warmup - 1)
        for _ in range(pre):                     # untimed decode up to the timed window
            step()
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        with ClockSampler(local) as clk, torch.cuda.nvtx.range("cbq_timed"):
            ms = timed_ms(torch, dist, step, steps, world, dev)
        res.update(ms_step=ms / steps, clocks=clk.summary(), timed_steps=steps,
                   positions=[prompt_len + 1 + pre + warmup, prompt_len + 1 + pre + warmup + steps])
        if e2e:
            ids_host = dec.next_ids.cpu().pin_memory()
            next_host = torch.empty_like(ids_host).pin_memory()

            def e2e_step():
                dec.ids.copy_(ids_host, non_blocking=True)
                dec.run_step()
                dec.pos.add_(1)
                next_host.copy_(dec.next_ids, non_blocking=True)
                torch.cuda.current_stream().synchronize()
                ids_host.copy_(next_host)
            res["ms_e2e"] = timed_ms(torch, dist, e2e_step, steps, world, dev) / steps
    res["launches_per_step"] = dec.launches_per_step()
    res["layer_launches"] = dec.layer_launches()
    res["peer"] = dec.peer is not None
    res["fuse_norm"], res["fuse_rope"] = dec.fuse_norm, dec.fuse_rope
    res["max_len"] = max_len
    dec.release()
    del dec
    return res


def decode_sub(cbq, cfg, dev, huffman, batch, steps, warmup, prompt_len, gen, block, what):
    """A decode sub-result (one GPU): tok/s with the whole step's stream
    bytes over its time as the HBM roofline."""
    import torch
    q3 = cbq.qwen3
    t0 = time.time()
    W = q3.CompressedQwen3Weights(cfg, dev, huffman=huffman)
    setup = time.time() - t0
    r = decode_run(W, batch, steps, warmup, 1, None, dev, 0, prompt_len=prompt_len, gen=gen, e2e=False,
                   block=block)
    stack = W.total_stream_bytes()
    pk = peaks()
    gbs = stack / (r["ms_step"] * 1e-3) / 1e9
    del W
    torch.cuda.empty_cache()
    return {"metric": f"compressed decode tok/s ({cfg.name}, bs{batch})", "value": batch * 1000.0 / r["ms_step"],
            "unit": "tok/s", "n_gpus": 1, "steps": r["timed_steps"], "warmup": warmup, "ms_per_step": r["ms_step"],
            "higher_is_better": True, "dtype": "bf16",
            "config": {"workload": what, "global_batch": batch, "prompt": prompt_len, "generated": gen,
                       "streams": "huffman" if huffman else "fixed 13-bit", "setup_s": round(setup, 1),
                       "stream_bytes": stack},
            "roofline": {"kernel": "whole decode step (all linears' streams)", "bound": "hbm", "achieved": gbs,
                         "peak": pk["hbm"], "unit": "GB/s", "frac": gbs / pk["hbm"], "peak_kind": pk["kind"],
                         "traffic": None},
            "gpu_launches": r["timed_steps"] * r["launches_per_step"], "clocks": r["clocks"]}


def _safe(name, fn, out):
    try:
        t0 = time.time()
        d = fn()
        d["name"] = name
        d["wall_s"] = round(time.time() - t0, 1)
        out.append(d)
    except Exception as e:                        # a failed sub-result is reported, not fatal
        out.append({"name": name, "error": f"{type(e).__name__}: {e}",
                    "trace": traceback.format_exc(limit=3)[-600:]})


def sub_results(cbq, dev, W8, args):
    """The other BASELINE configurations on one GPU (see the module docstring)."""
    import torch
    q3 = cbq.qwen3
    out = []
    pk = peaks()

    def bs8():
        r = decode_run(W8, 8, 10, 3, 1, None, dev, 0, e2e=False)
        gbs = W8.total_stream_bytes() / (r["ms_step"] * 1e-3) / 1e9
        return {"metric": "compressed decode tok/s (qwen3-8b, bs8)", "value": 8000.0 / r["ms_step"],
                "unit": "tok/s", "ms_per_step": r["ms_step"], "steps": r["timed_steps"], "warmup": 3,
                "config": {"workload": "config 5: qwen3-8b greedy decode, batch 8, fixed 13-bit streams, CUDA graph",
                           "positions": r["positions"]},
                "roofline": {"kernel": "whole decode step", "bound": "hbm", "achieved": gbs, "peak": pk["hbm"],
                             "unit": "GB/s", "frac": gbs / pk["hbm"], "peak_kind": pk["kind"], "traffic": None},
                "gpu_launches": r["timed_steps"] * r["launches_per_step"], "clocks": r["clocks"]}

    def block128():
        r = decode_run(W8, 1, 0, 3, 1, None, dev, 0, e2e=False, block=True)
        gbs = W8.total_stream_bytes() / (r["ms_step"] * 1e-3) / 1e9
        return {"metric": "compressed decode tok/s (qwen3-8b, bs1, 128 tokens)", "value": 1000.0 / r["ms_step"],
                "unit": "tok/s", "ms_per_step": r["ms_step"], "steps": r["timed_steps"], "warmup": 3,
                "config": {"workload": "config 5: 128 greedy tokens after a 64-token prompt, timed as one block"},
                "roofline": {"kernel": "whole decode step", "bound": "hbm", "achieved": gbs, "peak": pk["hbm"],
                             "unit": "GB/s", "frac": gbs / pk["hbm"], "peak_kind": pk["kind"], "traffic": None},
                "gpu_launches": r["timed_steps"] * r["launches_per_step"], "clocks": r["clocks"]}

    _safe("config5_decode_128_tokens_bs1", block128, out)
    _safe("config5_decode_fixed_bs8", bs8, out)
    _safe("gemv_12288x4096_t8_fixed", lambda: gemv_line((12288, 4096), 8, False, "bf16", 20, 3), out)
    _safe("config1_gemv_2048x2048_fixed_f32", lambda: gemv_line((2048, 2048), 1, False, "f32", 50, 3), out)
    _safe("config2_gemv_6144x2048_huffman_f32", lambda: gemv_line((6144, 2048), 1, True, "f32", 50, 3), out)
    _safe("config2_gemv_2048x6144_huffman_f32", lambda: gemv_line((2048, 6144), 1, True, "f32", 50, 3), out)
    _safe("gemv_12288x4096_huffman_bf16", lambda: gemv_line((12288, 4096), 1, True, "bf16", 20, 3), out)
    _safe("config4_prefill_fixed", lambda: prefill_line((12288, 4096), 4096, False, 10, 3), out)
    _safe("config4_prefill_huffman", lambda: prefill_line((12288, 4096), 4096, True, 10, 3), out)
    return out


def sub_results_other_models(cbq, dev):
    """Decode sub-results that need their own weights (built after the
    headline model is freed)."""
    q3 = cbq.qwen3
    out = []
    _safe("config5_decode_huffman_bs1",
          lambda: decode_sub(cbq, q3.QWEN3_8B, dev, True, 1, 10, 3, PROMPT_LEN, GEN_TOKENS, False,
                             "config 5: qwen3-8b greedy decode, batch 1, Huffman streams, CUDA graph"), out)
    _safe("config3_decode_qwen3_1.7b_bs1",
          lambda: decode_sub(cbq, q3.QWEN3_1_7B, dev, False, 1, 0, 3, 16, 30, True,
                             "config 3: qwen3-1.7b, 16-token prompt, 30 greedy tokens timed as one block, "
                             "fixed 13-bit streams, CUDA graph"), out)
    return out


def tp_token_check(cbq, dev, rank, world, group):
    """Greedy tokens of a small tensor-parallel model (fp32 activations)
    against the same model unsharded on this rank's GPU, for fixed-width
    streams over the peer-memory all-reduce and over NCCL and for Huffman
    streams over NCCL.  Every rank takes the same collective steps."""
    import importlib
    import torch
    import torch.distributed as dist
    qd = importlib.import_module(PKG + ".qwen3_decode")
    q3 = cbq.qwen3
    cfg = q3.Qwen3Config("tiny-tp", 2, 512, 1024, 16, 8, 64, 2048, 1e6, False)
    prompt = torch.randint(0, cfg.vocab, (2, 12), generator=torch.Generator().manual_seed(8))
    cases = {}
    for huffman, allreduce in ((False, "peer"), (False, "nccl"), (True, "nccl")):
        name = f"{'huffman' if huffman else 'fixed'}-{allreduce}"
        ok, why = True, ""
        try:
            full = q3.CompressedQwen3Weights(cfg, dev, huffman=huffman, seed=3)
            ref = qd.Qwen3Decoder(full, batch=2, max_len=48, act_dtype=torch.float32).generate(prompt, 30).cpu()
            del full
            Wt = q3.CompressedQwen3Weights(cfg, dev, huffman=huffman, rank=rank, world=world, seed=3)
            dec = qd.Qwen3Decoder(Wt, batch=2, max_len=48, act_dtype=torch.float32, group=group, allreduce=allreduce)
            if allreduce == "peer" and dec.peer is None:
                ok, why = False, "peer path not taken"
            eager = dec.generate(prompt, 30).cpu()
            dec.reset()
            dec.capture()
            dec.reset()
            graphed = dec.generate(prompt, 30).cpu()
            dec.release()
            if dec.peer is not None and int(dec.peer.status[0].item()) != 0:
                ok, why = False, f"peer status {dec.peer.status.tolist()}"
            if not torch.equal(eager, ref):
                ok, why = False, "eager tokens differ from the unsharded model"
            if not torch.equal(graphed, ref):
                ok, why = False, "graph-replay tokens differ from the unsharded model"
            del dec, Wt
        except Exception as e:
            ok, why = False, f"{type(e).__name__}: {e}"
        flag = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
        cases[name] = {"match": bool(flag.item()), **({"rank0_note": why} if why else {})}
    torch.cuda.empty_cache()
    return all(c["match"] for c in cases.values()), cases


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    if args.workload == "gemv":
        M, K = (int(v) for v in args.shape.split(","))
        print(json.dumps(gemv_line((M, K), args.tokens, args.huffman, args.x_dtype, args.steps, args.warmup)),
              flush=True)
        return
    if args.workload == "prefill":
        M, K = (int(v) for v in args.shape.split(","))
        T = args.tokens if args.tokens > 1 else 4096
        print(json.dumps(prefill_line((M, K), T, args.huffman, args.steps, args.warmup)), flush=True)
        return
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
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=180))
        group = dist.group.WORLD
    tp_ok, tp_cases = None, None
    if world > 1 and not args.no_sub:
        tp_ok, tp_cases = tp_token_check(cbq, dev, rank, world, group)
    cfg = q3.QWEN3_8B if args.model == "qwen3-8b" else q3.QWEN3_1_7B
    t0 = time.time()
    W = q3.CompressedQwen3Weights(cfg, dev, huffman=args.huffman, rank=rank, world=world)
    setup_s = time.time() - t0
    H = cfg.hidden
    r = decode_run(W, args.batch, args.steps, args.warmup, world, group, dev, local, allreduce=args.allreduce,
                   fuse_norm=args.fuse_norm, split_rope=args.split_rope, graph=not args.no_graph)
    ms_step, ms_e2e = r["ms_step"], r["ms_e2e"]
    value = args.batch * 1000.0 / ms_step

    # dominant kernel: gate_proj decode-GEMV over all 36 layers' weights (graph-replayed)
    gates = [W.layers[f"model.layers.{i}.mlp.gate_proj.weight"] for i in range(cfg.layers)]
    xg = torch.randn(args.batch, H, device=dev).to(torch.bfloat16)
    outs = [torch.empty(args.batch, gt.M, device=dev, dtype=torch.bfloat16) for gt in gates]
    gms = graph_time_ms(torch, lambda: [gt(xg, out=o) for gt, o in zip(gates, outs)], 20, dev) / len(gates)
    g0 = gates[0]
    cbn = W.codebooks["mlp_ffn"].numel()
    alg = W.stream_bytes["model.layers.0.mlp.gate_proj.weight"] + 4 * cbn + 2 * H * args.batch \
        + 2 * g0.M * args.batch
    pk = peaks()
    achieved = alg / (gms * 1e-3) / 1e9
    kern = gemv_kernel_name(args.huffman, args.batch)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        run_once, kind, desc, cores = cpu_reference_sample(cfg)
        res = [run_once() for _ in range(3)]
        cpu = {"value": 1.0 / float(np.mean([x[1] for x in res])), "unit": "tok/s", "cores": cores,
               "kind": kind, "sample": desc, "ms_per_sample": 1e3 * float(np.mean([x[0] for x in res]))}

    subs = None
    if world == 1 and not args.no_sub and args.model == "qwen3-8b" and not args.huffman and args.batch == 1:
        subs = sub_results(cbq, dev, W, args)
    stack_bytes = W.total_stream_bytes()
    del gates, outs, W
    torch.cuda.empty_cache()
    if subs is not None:
        subs += sub_results_other_models(cbq, dev)

    if rank == 0:
        line = {
            "metric": "compressed decode tok/s (Qwen3-8B shape, bs1)", "value": value, "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded bf16 N(0,0.02) weights, lossless per-category codebooks, "
                    "64 seeded prompt tokens)",
            "config": {"workload": f"{cfg.name} greedy decode, batch {args.batch}, "
                                   f"{'huffman' if args.huffman else 'fixed 13-bit'} streams, CUDA graph",
                       "global_batch": args.batch, "seq_len": r["max_len"], "parallelism": f"tp{world}",
                       "timed_positions": r["positions"],
                       "allreduce": ("peer-memory (GEMV epilogue + RMSNorm)" if r["peer"]
                                     else ("nccl" if world > 1 else "none")),
                       "launches_per_layer": r["layer_launches"],
                       "l2": "weights 12.3 GB >> 126 MB L2 (no flush)",
                       "stream_bytes_per_rank": stack_bytes,
                       "hbm_gbs_whole_step": stack_bytes / (ms_step * 1e-3) / 1e9,
                       "setup_s": round(setup_s, 1)},
            "roofline": {"kernel": kern + f" gate_proj {g0.M}x{g0.K}",
                         "bound": "hbm", "achieved": achieved, "peak": pk["hbm"], "unit": "GB/s",
                         "frac": achieved / pk["hbm"], "peak_kind": pk["kind"],
                         "traffic": NCU_TRAFFIC.get((kern, g0.M, g0.K, args.batch)),
                         "alg_bytes_per_launch": alg, "us_per_launch": gms * 1e3,
                         "timing": "CUDA-graph replay of the 36 gate_proj launches, CUDA events"},
            "e2e": {"value": args.batch * 1000.0 / ms_e2e, "unit": "tok/s",
                    "h2d_bytes_per_step": 8 * args.batch, "d2h_bytes_per_step": 8 * args.batch},
            "gpu_launches": args.steps * r["launches_per_step"],
            "clocks": r["clocks"],
        }
        if cpu:
            line["cpu_baseline"] = cpu
        if tp_ok is not None:
            line["tp_tokens_match"] = tp_ok
            line["tp_token_cases"] = tp_cases
        if subs is not None:
            line["sub_results"] = subs
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
