"""Decode-step kernels: the multi-matrix decode-GEMV with its fused epilogues,
RMSNorm, q/k RMSNorm + rotary + cache write, and decode attention.

The multi-matrix launch is checked bit for bit against one cbq_linear_fixed
call per matrix followed by the torch operations its epilogue replaces (the
per-row sums are computed identically and the epilogue rounds where torch
does).  The other kernels are checked against the torch formulation of HF
Qwen3 within fp32 / bf16 tolerances (their reductions run in a different
order from torch's).
"""
import importlib

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helpers import cbq, need_cuda, rel_l2

pytestmark = pytest.mark.gpu
L = cbq._lib
G = cbq.gpu_accelerated_functions


def _mats(dev, Ms, K, bits=13, seed=0):
    rng = np.random.default_rng(seed)
    C = (1 << bits) - 5
    cb = torch.from_numpy((rng.standard_normal(C) * 0.02).astype(np.float32)).to(dev)
    mats = []
    for i, M in enumerate(Ms):
        idx = rng.integers(0, 1 << bits, size=M * K).astype(np.uint16)   # some >= C: clamped
        mats.append(G.GPUAcceleratedLinear(f"m{i}", cbq.bitpack.pack_any_bits(idx, bits), cb, (M, K), bits,
                                           device=dev))
    return mats


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("T", [1, 2])
@pytest.mark.parametrize("epi,Ms,K", [(0, [4096, 1024, 1024], 4096), (2, [3072, 3072], 2048), (0, [151936], 256)],
                         ids=["qkv", "gate-up", "lm-head"])
@pytest.mark.parametrize("weighted", [False, True], ids=["unit", "weight"])
def test_multi_norm_matches_rmsnorm_then_gemv(dt, T, epi, Ms, K, weighted):
    """cbq_linear_fixed_multi_norm (RMSNorm applied while the GEMV loads the
    residual stream) against cbq_rmsnorm followed by cbq_linear_fixed_multi:
    the same roundings, only the sum-of-squares order differs (fp32: rel-L2
    1e-5; bf16: a rare last-bit flip of a normalised activation, 1e-2)."""
    dev = need_cuda()
    mats = _mats(dev, Ms, K, seed=len(Ms) + K)
    x = (torch.randn(T, K, device=dev) * 3).to(dt)
    w = (torch.rand(K, device=dev) + 0.5) if weighted else None
    code = L.CBQ_BF16 if dt == torch.bfloat16 else L.CBQ_F32
    h = torch.empty_like(x)
    L.call("cbq_rmsnorm", x.data_ptr(), None, code, T, K, None if w is None else w.data_ptr(), 1e-6, h.data_ptr(),
           torch.cuda.current_stream(dev).cuda_stream)
    n_out = 1 if epi == L.CBQ_EPI_SILU_MUL else len(Ms)
    ref = [torch.empty(T, Ms[i], device=dev, dtype=dt) for i in range(n_out)]
    got = [torch.empty_like(r) for r in ref]
    assert G.linear_fixed_multi(mats, h, ref, epi)
    x0 = x.clone()
    assert G.linear_fixed_multi(mats, x, got, epi, norm=(w, 1e-6))
    torch.cuda.synchronize()
    assert torch.equal(x, x0)                              # the residual stream is only read
    tol = 1e-5 if dt == torch.float32 else 1e-2
    for r, g in zip(ref, got):
        assert rel_l2(g.float().cpu().numpy(), r.float().cpu().numpy()) < tol


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("T", [1, 2])
def test_multi_store_matches_single_calls(dt, T):
    dev = need_cuda()
    mats = _mats(dev, [512, 128, 128], 1024)
    x = torch.randn(T, 1024, device=dev).to(dt)
    outs = [torch.empty(T, m.M, device=dev, dtype=dt) for m in mats]
    assert G.linear_fixed_multi(mats, x, outs)
    for m, o in zip(mats, outs):
        assert torch.equal(o, m(x)), m.name


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_multi_residual_epilogue_is_the_torch_add(dt):
    dev = need_cuda()
    (m,) = _mats(dev, [2048], 4096, seed=1)
    h = torch.randn(2, 4096, device=dev).to(dt)
    x = torch.randn(2, 2048, device=dev).to(dt)
    want = x + m(h)
    got = x.clone()
    assert G.linear_fixed_multi([m], h, [got], L.CBQ_EPI_RESIDUAL, [got])
    assert torch.equal(got, want)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("M", [1536, 770])
def test_multi_silu_mul_epilogue_is_the_torch_mlp(dt, M):
    dev = need_cuda()
    g, u = _mats(dev, [M, M], 2048, seed=2)
    h = torch.randn(1, 2048, device=dev).to(dt)
    want = F.silu(g(h)) * u(h)
    got = torch.empty(1, M, device=dev, dtype=dt)
    assert G.linear_fixed_multi([g, u], h, [got], L.CBQ_EPI_SILU_MUL)
    assert torch.equal(got, want)


def test_multi_declines_three_tokens():
    dev = need_cuda()
    mats = _mats(dev, [256], 1024)
    x = torch.randn(3, 1024, device=dev)
    out = torch.full((3, 256), 7.0, device=dev)
    assert not G.linear_fixed_multi(mats, x, [out])
    assert bool((out == 7.0).all())


def _rms_ref(x, eps):
    x32 = x.float()
    return (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_rmsnorm_with_and_without_residual_add(dt):
    dev = need_cuda()
    x = torch.randn(3, 4096, device=dev).to(dt)
    y = torch.randn(3, 4096, device=dev).to(dt)
    out = torch.empty_like(x)
    code = L.CBQ_BF16 if dt == torch.bfloat16 else L.CBQ_F32
    s = torch.cuda.current_stream(dev).cuda_stream
    x0 = x.clone()
    L.call("cbq_rmsnorm", x.data_ptr(), None, code, 3, 4096, None, 1e-6, out.data_ptr(), s)
    assert torch.equal(x, x0)
    tol = 1e-6 if dt == torch.float32 else 8e-3
    assert rel_l2(out.float().cpu().numpy(), _rms_ref(x0, 1e-6).float().cpu().numpy()) < tol
    L.call("cbq_rmsnorm", x.data_ptr(), y.data_ptr(), code, 3, 4096, None, 1e-6, out.data_ptr(), s)
    assert torch.equal(x, x0 + y)                                  # the residual update, rounded like torch
    assert rel_l2(out.float().cpu().numpy(), _rms_ref(x0 + y, 1e-6).float().cpu().numpy()) < tol


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("d", [64, 128])
def test_qk_norm_rope_and_cache_write(dt, d):
    dev = need_cuda()
    qd = importlib.import_module("codebook-quantization_b200.qwen3_decode")
    B, Hq, Hkv, Lc, pos = 2, 8, 2, 20, 13
    cos, sin = qd.rope_tables(d, Lc, 1e6, dev)
    q = torch.randn(B, Hq * d, device=dev).to(dt)
    k = torch.randn(B, Hkv * d, device=dev).to(dt)
    v = torch.randn(B, Hkv * d, device=dev).to(dt)
    q_out = torch.empty(B, Hq, d, device=dev, dtype=dt)
    kc = torch.zeros(B, Hkv, Lc, d, device=dev, dtype=dt)
    vc = torch.zeros_like(kc)
    p = torch.tensor([pos], device=dev)
    code = L.CBQ_BF16 if dt == torch.bfloat16 else L.CBQ_F32
    L.call("cbq_qk_norm_rope", q.data_ptr(), k.data_ptr(), v.data_ptr(), code, B, Hq, Hkv, d, 1e-6, None, None,
           cos.data_ptr(), sin.data_ptr(), p.data_ptr(), q_out.data_ptr(), kc.data_ptr(), vc.data_ptr(), Lc,
           torch.cuda.current_stream(dev).cuda_stream)
    c, s_ = cos[pos].to(dt), sin[pos].to(dt)
    qn = _rms_ref(q.view(B, Hq, d), 1e-6)
    kn = _rms_ref(k.view(B, Hkv, d), 1e-6)
    q_ref = qn * c + _rotate_half(qn) * s_
    k_ref = kn * c + _rotate_half(kn) * s_
    tol = 1e-6 if dt == torch.float32 else 8e-3
    assert rel_l2(q_out.float().cpu().numpy(), q_ref.float().cpu().numpy()) < tol
    assert rel_l2(kc[:, :, pos].float().cpu().numpy(), k_ref.float().cpu().numpy()) < tol
    assert torch.equal(vc[:, :, pos], v.view(B, Hkv, d))
    others = torch.ones(Lc, dtype=torch.bool)
    others[pos] = False
    assert not bool(kc[:, :, others].any()) and not bool(vc[:, :, others].any())
    # a position outside the cache writes nothing
    p.fill_(Lc)
    kc2 = kc.clone()
    L.call("cbq_qk_norm_rope", q.data_ptr(), k.data_ptr(), v.data_ptr(), code, B, Hq, Hkv, d, 1e-6, None, None,
           cos.data_ptr(), sin.data_ptr(), p.data_ptr(), q_out.data_ptr(), kc.data_ptr(), vc.data_ptr(), Lc,
           torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(kc, kc2)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("d,pos", [(128, 0), (128, 77), (64, 300)])
def test_attn_decode_matches_sdpa(dt, d, pos):
    dev = need_cuda()
    B, Hq, Hkv, Lc = 2, 8, 2, 512
    q = torch.randn(B, Hq, d, device=dev).to(dt)
    kc = torch.randn(B, Hkv, Lc, d, device=dev).to(dt)
    vc = torch.randn(B, Hkv, Lc, d, device=dev).to(dt)
    out = torch.empty(B, Hq * d, device=dev, dtype=dt)
    p = torch.tensor([pos], device=dev)
    code = L.CBQ_BF16 if dt == torch.bfloat16 else L.CBQ_F32
    L.call("cbq_attn_decode", q.data_ptr(), kc.data_ptr(), vc.data_ptr(), code, B, Hq, Hkv, d, Lc, p.data_ptr(),
           d ** -0.5, out.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    kr = kc[:, :, :pos + 1].float().repeat_interleave(Hq // Hkv, dim=1)
    vr = vc[:, :, :pos + 1].float().repeat_interleave(Hq // Hkv, dim=1)
    att = torch.softmax((q.float().unsqueeze(2) @ kr.transpose(-1, -2)) * d ** -0.5, dim=-1)
    ref = (att @ vr).reshape(B, Hq * d)
    tol = 1e-5 if dt == torch.float32 else 8e-3
    assert rel_l2(out.float().cpu().numpy(), ref.cpu().numpy()) < tol


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("d,G,pos", [(128, 4, 0), (128, 4, 57), (64, 3, 140), (128, 8, 9)])
def test_attn_decode_rope_equals_the_two_launches(dt, d, G, pos):
    """The fused launch (q/k norm + rope + cache write + attention) gives the
    same output and cache rows, bit for bit, as cbq_qk_norm_rope followed by
    cbq_attn_decode; a position outside the cache writes nothing and gives 0."""
    dev = need_cuda()
    qd = importlib.import_module("codebook-quantization_b200.qwen3_decode")
    B, Hkv, Lc = 2, 2, 160
    Hq = G * Hkv
    cos, sin = qd.rope_tables(d, Lc, 1e6, dev)
    q = torch.randn(B, Hq * d, device=dev).to(dt)
    k = torch.randn(B, Hkv * d, device=dev).to(dt)
    v = torch.randn(B, Hkv * d, device=dev).to(dt)
    qw = torch.rand(d, device=dev) + 0.5
    kw = torch.rand(d, device=dev) + 0.5
    kc0 = torch.randn(B, Hkv, Lc, d, device=dev).to(dt)
    vc0 = torch.randn(B, Hkv, Lc, d, device=dev).to(dt)
    p = torch.tensor([pos], device=dev)
    code = L.CBQ_BF16 if dt == torch.bfloat16 else L.CBQ_F32
    st = torch.cuda.current_stream(dev).cuda_stream
    kc1, vc1 = kc0.clone(), vc0.clone()
    qn = torch.empty(B, Hq, d, device=dev, dtype=dt)
    ref = torch.empty(B, Hq * d, device=dev, dtype=dt)
    L.call("cbq_qk_norm_rope", q.data_ptr(), k.data_ptr(), v.data_ptr(), code, B, Hq, Hkv, d, 1e-6, qw.data_ptr(),
           kw.data_ptr(), cos.data_ptr(), sin.data_ptr(), p.data_ptr(), qn.data_ptr(), kc1.data_ptr(),
           vc1.data_ptr(), Lc, st)
    L.call("cbq_attn_decode", qn.data_ptr(), kc1.data_ptr(), vc1.data_ptr(), code, B, Hq, Hkv, d, Lc, p.data_ptr(),
           d ** -0.5, ref.data_ptr(), st)
    kc2, vc2 = kc0.clone(), vc0.clone()
    out = torch.empty_like(ref)
    L.call("cbq_attn_decode_rope", q.data_ptr(), k.data_ptr(), v.data_ptr(), code, B, Hq, Hkv, d, 1e-6,
           qw.data_ptr(), kw.data_ptr(), cos.data_ptr(), sin.data_ptr(), p.data_ptr(), kc2.data_ptr(),
           vc2.data_ptr(), Lc, d ** -0.5, out.data_ptr(), st)
    assert torch.equal(kc2, kc1) and torch.equal(vc2, vc1)
    assert torch.equal(out, ref)
    p.fill_(Lc)
    kc3, vc3 = kc0.clone(), vc0.clone()
    L.call("cbq_attn_decode_rope", q.data_ptr(), k.data_ptr(), v.data_ptr(), code, B, Hq, Hkv, d, 1e-6,
           qw.data_ptr(), kw.data_ptr(), cos.data_ptr(), sin.data_ptr(), p.data_ptr(), kc3.data_ptr(),
           vc3.data_ptr(), Lc, d ** -0.5, out.data_ptr(), st)
    torch.cuda.synchronize()
    assert torch.equal(kc3, kc0) and torch.equal(vc3, vc0)
    assert not bool(out.any())


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("B,Hq,Hkv,d,Lc,pos", [(1, 32, 8, 128, 200, 171), (2, 8, 2, 128, 512, 77),
                                               (1, 4, 1, 128, 200, 0), (8, 32, 8, 128, 200, 150),
                                               (2, 12, 4, 64, 400, 399), (1, 16, 2, 256, 64, 35)])
def test_attn_decode_split_matches_sdpa(dt, B, Hq, Hkv, d, Lc, pos):
    """Split-key attention (flash-decoding: chunks of the keys on separate
    CTAs, the last CTA combines) against the fp32 softmax reference, on two
    calls in a row (the arrival counters are reused)."""
    dev = need_cuda()
    q = torch.randn(B, Hq, d, device=dev).to(dt)
    kc = torch.randn(B, Hkv, Lc, d, device=dev).to(dt)
    vc = torch.randn(B, Hkv, Lc, d, device=dev).to(dt)
    p = torch.tensor([pos], device=dev)
    code = L.CBQ_BF16 if dt == torch.bfloat16 else L.CBQ_F32
    nws = L.query("cbq_attn_workspace_bytes", B, Hq, Hkv, d, Lc)
    ws = torch.zeros(nws, dtype=torch.uint8, device=dev)
    kr = kc[:, :, :pos + 1].float().repeat_interleave(Hq // Hkv, dim=1)
    vr = vc[:, :, :pos + 1].float().repeat_interleave(Hq // Hkv, dim=1)
    att = torch.softmax((q.float().unsqueeze(2) @ kr.transpose(-1, -2)) * d ** -0.5, dim=-1)
    ref = (att @ vr).reshape(B, Hq * d)
    tol = 1e-5 if dt == torch.float32 else 8e-3
    outs = []
    for _ in range(2):
        out = torch.full((B, Hq * d), float("nan"), device=dev).to(dt)
        L.call("cbq_attn_decode_split", q.data_ptr(), kc.data_ptr(), vc.data_ptr(), code, B, Hq, Hkv, d, Lc,
               p.data_ptr(), d ** -0.5, out.data_ptr(), ws.data_ptr(), nws, torch.cuda.current_stream(dev).cuda_stream)
        torch.cuda.synchronize()
        assert rel_l2(out.float().cpu().numpy(), ref.cpu().numpy()) < tol
        outs.append(out)
    assert torch.equal(outs[0], outs[1])                    # deterministic combine order


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("d,G,pos", [(128, 4, 0), (128, 4, 157), (64, 3, 140), (128, 8, 9)])
def test_attn_decode_rope_split_matches_one_cta(dt, d, G, pos):
    """The split form of the fused rope + attention launch writes the same
    cache rows as the one-CTA form, bit for bit, and the same output within
    the fp32 summation-order tolerance; a position outside the cache writes
    nothing and gives 0."""
    dev = need_cuda()
    qd = importlib.import_module("codebook-quantization_b200.qwen3_decode")
    B, Hkv, Lc = 2, 2, 160
    Hq = G * Hkv
    cos, sin = qd.rope_tables(d, Lc, 1e6, dev)
    q = torch.randn(B, Hq * d, device=dev).to(dt)
    k = torch.randn(B, Hkv * d, device=dev).to(dt)
    v = torch.randn(B, Hkv * d, device=dev).to(dt)
    qw = torch.rand(d, device=dev) + 0.5
    kw = torch.rand(d, device=dev) + 0.5
    kc0 = torch.randn(B, Hkv, Lc, d, device=dev).to(dt)
    vc0 = torch.randn(B, Hkv, Lc, d, device=dev).to(dt)
    p = torch.tensor([pos], device=dev)
    code = L.CBQ_BF16 if dt == torch.bfloat16 else L.CBQ_F32
    st = torch.cuda.current_stream(dev).cuda_stream
    nws = L.query("cbq_attn_workspace_bytes", B, Hq, Hkv, d, Lc)
    ws = torch.zeros(nws, dtype=torch.uint8, device=dev)
    kc1, vc1 = kc0.clone(), vc0.clone()
    ref = torch.empty(B, Hq * d, device=dev, dtype=dt)
    L.call("cbq_attn_decode_rope", q.data_ptr(), k.data_ptr(), v.data_ptr(), code, B, Hq, Hkv, d, 1e-6,
           qw.data_ptr(), kw.data_ptr(), cos.data_ptr(), sin.data_ptr(), p.data_ptr(), kc1.data_ptr(),
           vc1.data_ptr(), Lc, d ** -0.5, ref.data_ptr(), st)
    kc2, vc2 = kc0.clone(), vc0.clone()
    out = torch.empty_like(ref)
    L.call("cbq_attn_decode_rope_split", q.data_ptr(), k.data_ptr(), v.data_ptr(), code, B, Hq, Hkv, d, 1e-6,
           qw.data_ptr(), kw.data_ptr(), cos.data_ptr(), sin.data_ptr(), p.data_ptr(), kc2.data_ptr(),
           vc2.data_ptr(), Lc, d ** -0.5, out.data_ptr(), ws.data_ptr(), nws, st)
    torch.cuda.synchronize()
    assert torch.equal(kc2, kc1) and torch.equal(vc2, vc1)
    tol = 1e-6 if dt == torch.float32 else 8e-3
    assert rel_l2(out.float().cpu().numpy(), ref.float().cpu().numpy()) < tol
    p.fill_(Lc)
    kc3, vc3 = kc0.clone(), vc0.clone()
    L.call("cbq_attn_decode_rope_split", q.data_ptr(), k.data_ptr(), v.data_ptr(), code, B, Hq, Hkv, d, 1e-6,
           qw.data_ptr(), kw.data_ptr(), cos.data_ptr(), sin.data_ptr(), p.data_ptr(), kc3.data_ptr(),
           vc3.data_ptr(), Lc, d ** -0.5, out.data_ptr(), ws.data_ptr(), nws, st)
    torch.cuda.synchronize()
    assert torch.equal(kc3, kc0) and torch.equal(vc3, vc0)
    assert not bool(out.any())


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("T,M,K", [(1, 4096, 4096), (2, 2048, 6144), (1, 1024, 512), (1, 6144, 1024)])
def test_residual_norm_launch_equals_gemv_then_rmsnorm(dt, T, M, K):
    """cbq_linear_fixed_residual_norm (the GEMV whose last CTA normalises)
    gives the residual stream and normalised rows of the residual GEMV
    followed by cbq_rmsnorm, bit for bit, and leaves its arrival count 0."""
    dev = need_cuda()
    (m,) = _mats(dev, [M], K, seed=3)
    xin = torch.randn(T, K, device=dev).to(dt)
    resid0 = torch.randn(T, M, device=dev).to(dt)
    w = torch.rand(M, device=dev) + 0.5
    code = L.CBQ_BF16 if dt == torch.bfloat16 else L.CBQ_F32
    st = torch.cuda.current_stream(dev).cuda_stream
    r1 = resid0.clone()
    h1 = torch.empty(T, M, device=dev, dtype=dt)
    assert G.linear_fixed_multi([m], xin, [r1], L.CBQ_EPI_RESIDUAL, [r1])
    L.call("cbq_rmsnorm", r1.data_ptr(), None, code, T, M, w.data_ptr(), 1e-6, h1.data_ptr(), st)
    arrive = torch.zeros(1, dtype=torch.int32, device=dev)
    for _ in range(3):                                   # the count is reusable
        r2 = resid0.clone()
        h2 = torch.empty_like(h1)
        L.call("cbq_linear_fixed_residual_norm", xin.data_ptr(), code, T, K, m.packed.data_ptr(), m.nbytes,
               m.codebook.data_ptr(), m.C, m.bits, M, K, None, r2.data_ptr(), M, code, w.data_ptr(), 1e-6,
               h2.data_ptr(), M, arrive.data_ptr(), st)
        torch.cuda.synchronize()
        assert torch.equal(r2, r1)
        assert torch.equal(h2, h1)
        assert int(arrive.item()) == 0


@pytest.mark.parametrize("world", [2, 5, 8])
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_flagged_peer_slots_feed_the_consuming_gemv(dt, world):
    """Row-parallel partial products written as epoch-flagged slot words
    (cbq_linear_fixed_peer_flagged, one 'rank' each, every slot on this GPU,
    each producer finished before the consumer starts) and consumed by
    cbq_linear_fixed_multi_allreduce_norm: the residual it writes is
    round(resid + round(p0 + p1 + ...)) in rank order, and its GEMV equals
    RMSNorm of that residual through cbq_linear_fixed_multi_norm; a second
    step (next epoch) over the same slots gives the same."""
    import ctypes as ct
    dev = need_cuda()
    H, Kp, T = 1024, 512, 1
    os_ = _mats(dev, [H] * world, Kp, seed=21)
    (g,) = _mats(dev, [768], H, seed=22)
    code = L.CBQ_BF16 if dt == torch.bfloat16 else L.CBQ_F32
    st = torch.cuda.current_stream(dev).cuda_stream
    per = T * H * (4 if dt == torch.bfloat16 else 8)
    slots = torch.zeros(world * per, dtype=torch.uint8, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    status = torch.tensor([0, -1, 0, 0], dtype=torch.int32, device=dev)
    resid = (torch.randn(T, H, device=dev) * 2).to(dt)
    for step in range(2):
        epoch.add_(1)
        acts = [torch.randn(T, Kp, device=dev).to(dt) for _ in range(world)]
        for r, (m, a) in enumerate(zip(os_, acts)):
            ptrs = (ct.c_void_p * 1)(slots.data_ptr() + r * per)
            rc = L.lib().cbq_linear_fixed_peer_flagged(a.data_ptr(), code, T, Kp, m.packed.data_ptr(), m.nbytes,
                                                       m.codebook.data_ptr(), m.C, m.bits, H, Kp, None, 1, ptrs,
                                                       epoch.data_ptr(), H, code, st)
            assert rc == L.CBQ_OK, rc
        x = torch.zeros(T, H, device=dev, dtype=dt)
        out = torch.empty(T, 768, device=dev, dtype=dt)
        ar = (world, resid, slots.data_ptr(), None, epoch.data_ptr(), H, status.data_ptr())
        assert G.linear_fixed_multi([g], x, [out], norm=(None, 1e-6), allreduce=ar)
        tot = torch.zeros(T, H, device=dev)
        for m, a in zip(os_, acts):                    # rank order
            tot = tot + m(a).float()
        want = (resid.float() + tot.to(dt).float()).to(dt)
        ref = torch.empty_like(out)
        assert G.linear_fixed_multi([g], want, [ref], norm=(None, 1e-6))
        torch.cuda.synchronize()
        assert int(status[0].item()) == 0
        assert torch.equal(x, want), step
        assert torch.equal(out, ref), step
        resid = x.clone()


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_greedy_pick_equals_torch_argmax(dt):
    """cbq_greedy_pick on one GPU: the first index of the row maximum, like
    torch's max, including ties; and the two-'rank' exchange (both ranks'
    pick buffers on this GPU) gives the global argmax over both halves."""
    import ctypes as ct
    dev = need_cuda()
    B, V = 3, 151936
    lg = torch.randn(B, V, device=dev).to(dt)
    lg[1, 777] = lg[1, 99999] = 1e4                        # a tie: the first index wins
    ids = torch.full((B,), -1, dtype=torch.int64, device=dev)
    code = L.CBQ_BF16 if dt == torch.bfloat16 else L.CBQ_F32
    st = torch.cuda.current_stream(dev).cuda_stream
    L.call("cbq_greedy_pick", lg.data_ptr(), code, B, V, V, 0, 1, None, None, None, ids.data_ptr(), None, st)
    torch.cuda.synchronize()
    assert torch.equal(ids, lg.float().max(dim=-1).indices)
    # two ranks: rank 1's pair is already in rank 0's pick buffer (written
    # here as rank 1's launch would), so rank 0's launch finds every pair it
    # waits for; it publishes its own pair into both buffers
    W, Vh = 2, V // 2
    bufs = torch.zeros(W, W * B * 2, dtype=torch.int64, device=dev)
    epoch = torch.full((1,), 5, dtype=torch.int32, device=dev)
    status = torch.tensor([0, -1, 0, 0], dtype=torch.int32, device=dev)
    v1, i1 = lg[:, Vh:].float().max(dim=-1)
    words = torch.stack([(v1.view(torch.int32).to(torch.int64) & 0xFFFFFFFF) | (5 << 32),
                         (i1 + Vh) | (5 << 32)], dim=1).reshape(-1)
    bufs[0, B * 2:].copy_(words)
    out = torch.full((B,), -1, dtype=torch.int64, device=dev)
    part = lg[:, :Vh].contiguous()
    P = ct.c_void_p
    ptrs = (P * W)(*[bufs[p].data_ptr() for p in range(W)])           # slot 0 of each buffer
    L.call("cbq_greedy_pick", part.data_ptr(), code, B, Vh, Vh, 0, W, ptrs, bufs[0].data_ptr(),
           epoch.data_ptr(), out.data_ptr(), status.data_ptr(), st)
    torch.cuda.synchronize()
    assert int(status[0].item()) == 0
    assert torch.equal(out, lg.float().max(dim=-1).indices)
    v0, i0 = lg[:, :Vh].float().max(dim=-1)                           # what rank 0 published
    got = bufs[1, :B * 2].view(B, 2)
    assert torch.equal(got[:, 1] & 0xFFFFFFFF, i0) and bool(((got >> 32) == 5).all())


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_silu_mul_equals_torch(dt):
    """cbq_silu_mul (SiLU * up of separately computed gate and up rows) is
    bit-identical to torch's F.silu(g) * u in the same dtype, out of place
    and in place."""
    import torch.nn.functional as F
    dev = need_cuda()
    n = 3 * 12288 + 5
    g = (torch.randn(n, device=dev) * 3).to(dt)
    u = torch.randn(n, device=dev).to(dt)
    code = L.CBQ_BF16 if dt == torch.bfloat16 else L.CBQ_F32
    st = torch.cuda.current_stream(dev).cuda_stream
    out = torch.empty_like(g)
    L.call("cbq_silu_mul", g.data_ptr(), u.data_ptr(), code, n, out.data_ptr(), st)
    want = F.silu(g) * u
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    L.call("cbq_silu_mul", g.data_ptr(), u.data_ptr(), code, n, g.data_ptr(), st)     # out aliases g
    torch.cuda.synchronize()
    assert torch.equal(g, want)


_ATTN_SCRIPT = r"""
import sys, numpy as np, torch
from pathlib import Path
sys.path.insert(0, str(Path(sys.argv[1]).parent))
sys.path.insert(0, sys.argv[1])
from helpers import cbq
L = cbq._lib
B, Hq, Hkv, d, Lc, pos = 1, 32, 8, 128, 200, 171
g = torch.Generator().manual_seed(17)
dev = torch.device("cuda", 0)
q = torch.randn(B, Hq, d, generator=g).to(dev).to(torch.bfloat16)
kc = torch.randn(B, Hkv, Lc, d, generator=g).to(dev).to(torch.bfloat16)
vc = torch.randn(B, Hkv, Lc, d, generator=g).to(dev).to(torch.bfloat16)
p = torch.tensor([pos], device=dev)
nws = L.query("cbq_attn_workspace_bytes", B, Hq, Hkv, d, Lc)
ws = torch.zeros(nws, dtype=torch.uint8, device=dev)
out = torch.empty(B, Hq * d, device=dev, dtype=torch.bfloat16)
L.call("cbq_attn_decode_split", q.data_ptr(), kc.data_ptr(), vc.data_ptr(), L.CBQ_BF16, B, Hq, Hkv, d, Lc,
       p.data_ptr(), d ** -0.5, out.data_ptr(), ws.data_ptr(), nws, torch.cuda.current_stream(dev).cuda_stream)
torch.cuda.synchronize()
np.save(sys.argv[2], out.view(torch.int16).cpu().numpy())
"""


def test_attn_cluster_combine_equals_workspace_combine(tmp_path):
    """The cluster combine (distributed shared memory) and the workspace
    combine (global partial states, last CTA) do the same arithmetic in the
    same chunk order: bit-identical outputs.  Each form runs in its own
    process (CBQ_ATTN_CLUSTER is read once per process)."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    need_cuda()
    here = str(Path(__file__).resolve().parent)
    outs = []
    for flag in ("1", "0"):
        f = tmp_path / f"attn_{flag}.npy"
        env = dict(os.environ, CBQ_ATTN_CLUSTER=flag)
        subprocess.run([sys.executable, "-c", _ATTN_SCRIPT, here, str(f)], env=env, check=True, timeout=300)
        outs.append(np.load(f))
    assert np.array_equal(outs[0], outs[1])
