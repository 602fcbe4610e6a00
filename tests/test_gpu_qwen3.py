"""Whole-model greedy decode against HF transformers' Qwen3ForCausalLM.

The compressed model's decoded weights (codebook[index], exact bf16 values)
are loaded into HF's Qwen3 implementation, which is then the model-level
oracle: with fp32 activations on both sides the greedy token sequences must be
identical (BASELINE: identical greedy tokens over 30 steps).  The smallest
top-2 logit gap seen along the way is reported so a near-tie is visible.
"""
import importlib

import numpy as np
import pytest
import torch

from helpers import cbq, need_cuda

pytestmark = pytest.mark.gpu
q3 = cbq.qwen3
qd = importlib.import_module("codebook-quantization_b200.qwen3_decode")

TINY = q3.Qwen3Config("tiny", 2, 256, 512, 4, 2, 64, 1000, 1e6, False)
TINY_TIED = q3.Qwen3Config("tiny-tied", 3, 384, 768, 6, 2, 64, 1280, 1e6, True)


def hf_from(W):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    c = W.cfg
    hc = Qwen3Config(vocab_size=c.vocab, hidden_size=c.hidden, intermediate_size=c.inter,
                     num_hidden_layers=c.layers, num_attention_heads=c.heads,
                     num_key_value_heads=c.kv_heads, head_dim=c.head_dim, max_position_embeddings=512,
                     rms_norm_eps=c.rms_eps, tie_word_embeddings=c.tie_embeddings,
                     rope_parameters={"rope_theta": c.rope_theta, "rope_type": "default"})
    m = Qwen3ForCausalLM(hc).eval()
    sd = m.state_dict()
    cat = {s.name: s.category for s in q3.linear_specs(c)}
    with torch.no_grad():
        for name, idx in W.indices.items():
            w = W.codebooks[cat[name]][idx.long() & 0xFFFF].cpu()
            if name in sd:
                sd[name].copy_(w)
        for k, v in sd.items():
            if k.endswith("norm.weight"):
                v.fill_(1.0)
    return m


def hf_greedy(m, prompt, n):
    ids = prompt.clone()
    gaps = []
    past = None
    cur = ids
    out = []
    with torch.no_grad():
        for _ in range(n):
            r = m(input_ids=cur, past_key_values=past, use_cache=True)
            past = r.past_key_values
            logits = r.logits[:, -1, :].float()
            top2 = logits.topk(2, dim=-1).values
            gaps.append(float((top2[:, 0] - top2[:, 1]).min()))
            nxt = logits.argmax(-1)
            out.append(nxt)
            cur = nxt[:, None]
    return torch.stack(out, 1), min(gaps)


@pytest.mark.parametrize("cfg", [TINY, TINY_TIED], ids=lambda c: c.name)
@pytest.mark.parametrize("huffman", [False, True])
@pytest.mark.parametrize("fused", [True, False], ids=["fused", "torch-ops"])
def test_greedy_tokens_match_hf(cfg, huffman, fused):
    dev = need_cuda()
    W = q3.CompressedQwen3Weights(cfg, dev, huffman=huffman, keep_indices=True, seed=5)
    m = hf_from(W)
    prompt = torch.randint(0, cfg.vocab, (2, 16), generator=torch.Generator().manual_seed(7))
    ref, gap = hf_greedy(m, prompt, 30)
    dec = qd.Qwen3Decoder(W, batch=2, max_len=64, act_dtype=torch.float32, fused=fused)
    eager = dec.generate(prompt, 30).cpu()
    dec.reset()
    dec.capture()
    dec.reset()
    graphed = dec.generate(prompt, 30).cpu()
    dec.release()
    assert torch.equal(eager, graphed)
    assert torch.equal(graphed, ref), f"greedy tokens differ (smallest top-2 gap {gap:.3e})"


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "torch-ops"])
def test_bf16_decode_runs_and_mostly_agrees(fused):
    """bf16 activations (the bench's setting) against HF in bf16 on the CPU."""
    dev = need_cuda()
    W = q3.CompressedQwen3Weights(TINY, dev, keep_indices=True, seed=9)
    m = hf_from(W).to(torch.bfloat16)
    prompt = torch.randint(0, TINY.vocab, (1, 16), generator=torch.Generator().manual_seed(3))
    ref, _ = hf_greedy(m, prompt, 30)
    dec = qd.Qwen3Decoder(W, batch=1, max_len=64, act_dtype=torch.bfloat16, fused=fused)
    dec.capture()
    dec.reset()
    got = dec.generate(prompt, 30).cpu()
    dec.release()
    agree = int((got == ref).cumprod(1).sum())
    assert agree >= 8, f"bf16 decode agrees with HF bf16 for only {agree} leading tokens"


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_fused_and_torch_op_steps_agree(dt):
    """The fused step (8 launches per layer) against the torch-op step on the
    same weights: the element-wise parts round identically, only reduction
    orders differ, so the logits agree closely and the tokens exactly."""
    dev = need_cuda()
    W = q3.CompressedQwen3Weights(TINY_TIED, dev, seed=11)
    prompt = torch.randint(0, TINY_TIED.vocab, (2, 12), generator=torch.Generator().manual_seed(4))
    outs, logits = [], []
    for fused in (True, False):
        dec = qd.Qwen3Decoder(W, batch=2, max_len=40, act_dtype=dt, fused=fused)
        outs.append(dec.generate(prompt, 10).cpu())
        logits.append(dec.logits.float().cpu())
    tol = 1e-5 if dt == torch.float32 else 2e-2
    rel = float((logits[0] - logits[1]).norm() / logits[1].norm())
    assert rel < tol, rel
    if dt == torch.float32:
        assert torch.equal(outs[0], outs[1])


def test_batch4_step_matches_hf():
    """Batch 4 (the T > 2 linears: tensor-core GEMM, the norm launch adding the
    residual, cbq_silu_mul) gives HF's greedy tokens with fp32 activations."""
    dev = need_cuda()
    W = q3.CompressedQwen3Weights(TINY, dev, keep_indices=True, seed=13)
    m = hf_from(W)
    prompt = torch.randint(0, TINY.vocab, (4, 12), generator=torch.Generator().manual_seed(8))
    ref, gap = hf_greedy(m, prompt, 20)
    dec = qd.Qwen3Decoder(W, batch=4, max_len=40, act_dtype=torch.float32)
    dec.capture()
    dec.reset()
    got = dec.generate(prompt, 20).cpu()
    dec.release()
    assert torch.equal(got, ref), f"greedy tokens differ (smallest top-2 gap {gap:.3e})"
