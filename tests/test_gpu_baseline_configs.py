"""BASELINE configurations at their full shapes on the GPU.

* Config 3: a Qwen3-1.7B-architecture model (28 layers, hidden 2048, vocab
  151936, tied embeddings) compressed losslessly with one codebook per
  category; 16 seeded prompt ids, 30 greedy tokens at batch 1.  The oracle is
  HF transformers' ``Qwen3ForCausalLM`` loaded with the decoded weights
  (codebook[index], exact bf16 values) and run in fp32 (TF32 off); with fp32
  activations on both sides the greedy tokens must be identical (north_star's
  third check), and the last logits agree to rel-L2 1e-4.  The reference's
  model-level path is its CPU ``AdaptiveCodebookLinear`` forward inside HF
  (``src/compressed_modules.py:131-154``), checked end to end in
  ``tests/test_compressed_roundtrip.py:1483-1664``.
* Config 5 (Qwen3-8B shape): the same check with the BASELINE's 64-token
  prompt.
* Config 4: 12288 x 4096 13-bit weights times 4096 bf16 tokens through the
  public entry points (tensor-core GEMM for fixed width, the Huffman form
  through ``cbq_linear_huff``), against the C oracle on two 128-row blocks
  and against an fp32 product of the oracle-decoded weights on every row;
  rel-L2 1e-5 (bf16-exact codebook, fp32 accumulation: only the summation
  order differs).

The smallest top-2 logit gap along each greedy run is printed so that a
near-tie would be visible.
"""
import importlib

import numpy as np
import pytest
import torch

import oracle
from helpers import cbq, need_cuda, rel_l2

pytestmark = pytest.mark.gpu
q3 = cbq.qwen3
qd = importlib.import_module("codebook-quantization_b200.qwen3_decode")


def hf_on_gpu(W, dev):
    """HF Qwen3ForCausalLM (fp32, on ``dev``) holding the decoded weights of W."""
    from transformers import Qwen3Config, Qwen3ForCausalLM
    c = W.cfg
    hc = Qwen3Config(vocab_size=c.vocab, hidden_size=c.hidden, intermediate_size=c.inter,
                     num_hidden_layers=c.layers, num_attention_heads=c.heads,
                     num_key_value_heads=c.kv_heads, head_dim=c.head_dim, max_position_embeddings=512,
                     rms_norm_eps=c.rms_eps, tie_word_embeddings=c.tie_embeddings,
                     rope_parameters={"rope_theta": c.rope_theta, "rope_type": "default"})
    with torch.device(dev):
        m = Qwen3ForCausalLM(hc).eval()
    sd = m.state_dict()
    cat = {s.name: s.category for s in q3.linear_specs(c)}
    with torch.no_grad():
        for name, idx in W.indices.items():
            if name in sd:
                sd[name].copy_(W.codebooks[cat[name]][idx.long() & 0xFFFF])
        for k, v in sd.items():
            if k.endswith("norm.weight"):
                v.fill_(1.0)
    return m


def hf_greedy(m, prompt, n):
    gaps, out = [], []
    past, cur = None, prompt
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
    return torch.stack(out, 1), min(gaps), logits


def _greedy_vs_hf(cfg, prompt_len, n_new, seed):
    dev = need_cuda()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        W = q3.CompressedQwen3Weights(cfg, dev, keep_indices=True, seed=seed)
        prompt = torch.randint(0, cfg.vocab, (1, prompt_len), generator=torch.Generator().manual_seed(seed))
        m = hf_on_gpu(W, dev)
        W.indices.clear()
        ref, gap, ref_logits = hf_greedy(m, prompt.to(dev), n_new)
        del m
        torch.cuda.empty_cache()
        dec = qd.Qwen3Decoder(W, batch=1, max_len=prompt_len + n_new + 4, act_dtype=torch.float32)
        dec.capture()
        dec.reset()
        got = dec.generate(prompt, n_new)
        logits = dec.logits.float()
        dec.release()
        print(f"{cfg.name}: smallest top-2 logit gap over {n_new} greedy steps {gap:.3e}")
        assert torch.equal(got.cpu(), ref.cpu()), f"greedy tokens differ (smallest top-2 gap {gap:.3e})"
        rel = float((logits - ref_logits).norm() / ref_logits.norm())
        assert rel < 1e-4, rel
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def test_config3_qwen3_1_7b_greedy_30_tokens_match_hf():
    _greedy_vs_hf(q3.QWEN3_1_7B, 16, 30, seed=0)


def test_config5_qwen3_8b_greedy_30_tokens_match_hf():
    _greedy_vs_hf(q3.QWEN3_8B, 64, 30, seed=1)


@pytest.mark.parametrize("huffman", [False, True], ids=["fixed", "huffman"])
def test_config4_prefill_12288x4096x4096(huffman):
    dev = need_cuda()
    M, K, T = 12288, 4096, 4096
    comp = cbq.synth.GpuCompressor(dev)
    bits = cbq.synth.bf16_normal_gpu((M, K), seed=44, device=dev)
    d = comp.compress(bits, huffman=huffman)
    idx = comp.indices(bits, comp.codebook(comp.histogram(bits))[1])
    del bits
    cb = d["codebook"]
    if huffman:
        lin = cbq.HuffmanCodebookLinear("w", d["huff_stream"], d["huff_lengths"], int(d["huff_n"][0]), cb, (M, K),
                                        d["bits"], huff_row_bit_starts=d["huff_row_bit_starts"], device=dev)
    else:
        lin = cbq.GPUAcceleratedLinear("w", d["indices"], cb, (M, K), d["bits"], device=dev)
    x = torch.randn(T, K, device=dev, generator=torch.Generator(device=dev).manual_seed(5)).to(torch.bfloat16)
    y = lin(x, out_dtype=torch.float32)
    if huffman:
        lin.hs.check()
        assert torch.equal(lin.hs.decode_indices().to(torch.int64), idx.to(torch.int64) & 0xFFFF)
    cb_h = cb.cpu().numpy()
    x_h = x.float().cpu().numpy()
    b = d["bits"]
    row_bytes = K * b // 8
    if not huffman:
        packed_h = d["indices"].cpu().numpy()
        # the oracle's own decode of every index equals the encoder's indices
        dec_idx = oracle.unpack_fixed(packed_h, b, M * K)
        assert np.array_equal(dec_idx, (idx.cpu().numpy().reshape(-1).astype(np.int64) & 0xFFFF).astype(np.uint16))
        for r0 in (0, 7040):                                    # C oracle on two 128-row blocks
            sub = np.concatenate([packed_h[r0 * row_bytes:(r0 + 128) * row_bytes], np.zeros(8, np.uint8)])
            ref = oracle.linear_fixed(x_h, sub, cb_h, 128, K, b)
            assert rel_l2(y[:, r0:r0 + 128].cpu().numpy(), ref) < 1e-5, r0
    else:
        for r0 in (0, 7040):                                    # C oracle (Huffman) on two 128-row blocks
            sub = cbq.tp_shard.shard_huffman_rows({k: (v.cpu().numpy() if isinstance(v, torch.Tensor) else v)
                                                   for k, v in d.items()}, M, K, r0, r0 + 128)
            ref = oracle.huff_linear(x_h, sub, cb_h, 128, K)
            assert rel_l2(y[:, r0:r0 + 128].cpu().numpy(), ref) < 1e-5, r0
    # every row: fp32 product of the decoded weights (TF32 off)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        w = cb[(idx.to(torch.int64) & 0xFFFF)]
        ref_all = x.float() @ w.T
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    rel = float((y - ref_all).norm() / ref_all.norm())
    assert rel < 1e-5, rel
