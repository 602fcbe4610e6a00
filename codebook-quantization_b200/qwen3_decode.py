"""Greedy decode of a compressed Qwen3-architecture model on the GPU.

The math is HF ``Qwen3ForCausalLM``'s (transformers ``models/qwen3``): RMSNorm
in fp32 then cast back, q/k per-head RMSNorm before rotary embedding
(rotate-half form, inv_freq = theta^(-2i/d)), grouped-query attention with
softmax scaling d^-1/2, SiLU-gated MLP, residual adds in the activation dtype,
final RMSNorm and lm_head, greedy argmax (first index on ties).  Every linear
and the embedding run on ``libcbq``'s kernels; norms have unit weights (the
synthetic models keep them exact at 1.0).

Decode is one token per sequence per step.  The step reads the token ids and
the position from static device buffers, writes the new key/value rows into a
static cache and attends over it with a position mask, so it is captured once
in a CUDA graph and replayed for every prompt and generated token with no host
synchronisation.  Under tensor parallelism (``group`` given) heads and MLP
columns are split per rank, o_proj/down_proj partial sums are all-reduced over
NCCL, and the greedy argmax combines each rank's (max, index) pair.

Two step implementations compute the same function:

* ``fused=True`` (default): eight ``libcbq`` launches per layer -- one
  decode-GEMV launch for q/k/v, q/k RMSNorm + rotary + cache write, decode
  attention, o_proj with the residual add fused, RMSNorm, one launch for
  gate/up with SiLU(gate)*up fused, down_proj with the residual add fused,
  RMSNorm (under tensor parallelism the residual adds move into the RMSNorm
  launch, after the all-reduce);
* ``fused=False``: the same layer written with torch operations around one
  ``libcbq`` launch per linear layer (about fifty launches per layer).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _lib
from .gpu_accelerated_functions import GPUAcceleratedLinear, device_stream, linear_fixed_multi
from .qwen3 import CompressedQwen3Weights

__all__ = ["Qwen3Decoder", "rope_tables"]


class _PeerAllReduce:
    """The row-parallel layers' all-reduce over NVLink peer memory.

    One symmetric buffer per decoder: for every all-reduce site (o_proj and
    down_proj of each layer) a slot per rank ([world][B][hidden] in the
    activation dtype) and an arrival counter per rank.  Rank s's GEMV writes
    its partial product into slot s of every rank and adds its rows to every
    rank's counter s; the last CTA of each rank's GEMV waits for epoch * hidden
    rows from every rank, adds the slots in rank order into the residual
    stream and normalises (``cbq_linear_fixed_peer_norm``, one launch; with
    ``fuse_norm=False`` the split pair ``cbq_linear_fixed_peer`` +
    ``cbq_rmsnorm_allreduce``).  Counters only grow (``epoch`` counts the
    steps), so nothing is reset between steps."""

    def __init__(self, dec, sites: int):
        import ctypes as ct
        import torch.distributed._symmetric_memory as symm
        self.dec = dec
        W, r = dec.world, dec.rank
        self.W, self.rank = W, r
        self.n = dec.B * dec.cfg.hidden
        self.elem = 2 if dec.dt == torch.bfloat16 else 4
        self.slot_bytes = self.n * self.elem           # the consumer reads the slots back to back
        if self.slot_bytes % 16:
            raise ValueError("batch * hidden must fill whole 16-byte units")
        data = sites * W * self.slot_bytes
        counters = ((sites * W * 4 + 127) // 128) * 128
        # flagged slots (cbq_linear_fixed_peer_flagged): 64-bit words of 32
        # data bits + the epoch, two bf16 or one fp32 value per word
        self.flag_bytes = dec.B * dec.cfg.hidden * (4 if self.elem == 2 else 8)
        self.flag_off = data + counters
        # greedy pick: per rank, [W][B][2] 64-bit words (value, id) flagged with the epoch
        self.pick_off = self.flag_off + sites * W * self.flag_bytes
        total = self.pick_off + W * dec.B * 16
        self.buf = symm.empty(total, dtype=torch.uint8, device=dec.dev)
        self.buf.zero_()
        self.hdl = symm.rendezvous(self.buf, dec.group)
        ptrs = list(self.hdl.buffer_ptrs)
        self.local = self.buf.data_ptr()
        self.data = data
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dec.dev)
        self.status = torch.zeros(4, dtype=torch.int32, device=dec.dev)
        self.slots, self.counts, self.flagged = [], [], []
        P = ct.c_void_p
        for i in range(sites):
            self.slots.append((P * W)(*[ptrs[p] + (i * W + r) * self.slot_bytes for p in range(W)]))
            self.counts.append((P * W)(*[ptrs[p] + data + (i * W + r) * 4 for p in range(W)]))
            self.flagged.append((P * W)(*[ptrs[p] + self.flag_off + (i * W + r) * self.flag_bytes
                                          for p in range(W)]))
        self.pick = (P * W)(*[ptrs[p] + self.pick_off + r * dec.B * 16 for p in range(W)])
        self.local_pick = self.local + self.pick_off
        torch.cuda.synchronize(dec.dev)
        dist.barrier(group=dec.group)

    def produce(self, site: int, lin, x):
        """The row-parallel GEMV whose epilogue stores its partial rows, as
        epoch-flagged words, into slot ``rank`` of every rank's buffer for
        ``site`` (cbq_linear_fixed_peer_flagged)."""
        dec = self.dec
        rc = _lib.lib().cbq_linear_fixed_peer_flagged(
            x.data_ptr(), dec.code, dec.B, x.shape[1], lin.packed.data_ptr(), lin.nbytes, lin.codebook.data_ptr(),
            lin.C, lin.bits, lin.M, lin.K, None, self.W, self.flagged[site], self.epoch.data_ptr(), lin.M, dec.code,
            device_stream(dec.dev))
        if rc != _lib.CBQ_OK:
            raise _lib.CbqError("cbq_linear_fixed_peer_flagged", rc)

    def local_flagged(self, site: int) -> int:
        """This rank's flagged slots of ``site`` (rank s's slot at + s * flag_bytes)."""
        return self.local + self.flag_off + site * self.W * self.flag_bytes

    def run(self, site: int, lin, x):
        dec = self.dec
        W = self.W
        stream = device_stream(dec.dev)
        if dec.fuse_norm:
            rc = _lib.lib().cbq_linear_fixed_peer_norm(
                x.data_ptr(), dec.code, dec.B, x.shape[1], lin.packed.data_ptr(), lin.nbytes,
                lin.codebook.data_ptr(), lin.C, lin.bits, lin.M, lin.K, None, W, self.slots[site], self.counts[site],
                lin.M, dec.code, self.local + site * W * self.slot_bytes, self.local + self.data + site * W * 4,
                self.epoch.data_ptr(), lin.M, dec.x.data_ptr(), dec.cfg.hidden, None, float(dec.cfg.rms_eps),
                dec.h.data_ptr(), dec.cfg.hidden, dec.arrive.data_ptr(), self.status.data_ptr(), stream)
            if rc != _lib.CBQ_OK:
                raise _lib.CbqError("cbq_linear_fixed_peer_norm", rc)
            return
        rc = _lib.lib().cbq_linear_fixed_peer(
            x.data_ptr(), dec.code, dec.B, x.shape[1], lin.packed.data_ptr(), lin.nbytes, lin.codebook.data_ptr(),
            lin.C, lin.bits, lin.M, lin.K, None, W, self.slots[site], self.counts[site], lin.M, dec.code, stream)
        if rc != _lib.CBQ_OK:
            raise _lib.CbqError("cbq_linear_fixed_peer", rc)
        _lib.call("cbq_rmsnorm_allreduce", dec.x.data_ptr(), self.local + site * W * self.slot_bytes,
                  self.local + self.data + site * W * 4, self.epoch.data_ptr(), lin.M, W, dec.code, dec.B,
                  dec.cfg.hidden, None, float(dec.cfg.rms_eps), dec.h.data_ptr(), self.status.data_ptr(), stream)


def rope_tables(head_dim: int, max_len: int, theta: float, device):
    """cos/sin [max_len, head_dim] in fp32, HF's default rotary layout,
    computed on the host (as HF does on a CPU model) and copied to ``device``."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    t = torch.arange(max_len, dtype=torch.float32)
    f = (inv[:, None] @ t[None, :]).T
    emb = torch.cat((f, f), dim=-1)
    return emb.cos().to(device), emb.sin().to(device)


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def _rms(x, eps):
    dt = x.dtype
    x32 = x.float()
    x32 = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)
    return x32.to(dt)


class Qwen3Decoder:
    def __init__(self, weights: CompressedQwen3Weights, batch: int, max_len: int,
                 act_dtype=torch.bfloat16, group: Optional[dist.ProcessGroup] = None, fused: bool = True,
                 allreduce: str = "peer", fuse_norm: bool = False, fuse_rope: bool = True, prenorm: bool = True):
        self.w, self.cfg = weights, weights.cfg
        cfg = self.cfg
        self.dev = weights.device
        self.B, self.max_len, self.dt = batch, max_len, act_dtype
        self.group = group
        self.world = weights.world
        self.rank = weights.rank
        self.hl = cfg.heads // self.world
        self.kvl = cfg.kv_heads // self.world
        if self.hl * self.world != cfg.heads or self.kvl * self.world != cfg.kv_heads:
            raise ValueError(f"heads {cfg.heads}/{cfg.kv_heads} do not split over {self.world} ranks")
        d = cfg.head_dim
        self.cos, self.sin = rope_tables(d, max_len, cfg.rope_theta, self.dev)
        self.k_cache = [torch.zeros(batch, self.kvl, max_len, d, dtype=act_dtype, device=self.dev)
                        for _ in range(cfg.layers)]
        self.v_cache = [torch.zeros_like(self.k_cache[0]) for _ in range(cfg.layers)]
        self.ids = torch.zeros(batch, dtype=torch.int64, device=self.dev)
        self.pos = torch.zeros(1, dtype=torch.int64, device=self.dev)
        self.next_ids = torch.zeros(batch, dtype=torch.int64, device=self.dev)
        self.logits = None
        self.graph = None
        self.vocab_local = cfg.vocab // self.world
        self.ar = torch.arange(max_len, device=self.dev)
        self.fused = fused
        # fused step: q/k norm + rope done by the attention launch, and
        # optionally the RMSNorm done by the last CTA of the row-parallel GEMV
        # before it (measured slower on a B200 than its own one-CTA launch,
        # which waits on the SM the GEMV grid leaves free; off by default)
        self.fuse_norm, self.fuse_rope = fuse_norm, fuse_rope
        # one GPU, fixed-width streams, batch <= 2: each RMSNorm runs inside the
        # GEMV that consumes it (the norm applied as the residual stream is
        # loaded; cbq_linear_fixed_multi_norm), so a layer is five launches
        self.prenorm = (fused and prenorm and not fuse_norm and weights.world == 1 and not weights.huffman
                        and batch <= 2)
        if fused:
            hq, hkv = self.hl * d, self.kvl * d
            z = lambda n: torch.zeros(batch, n, dtype=act_dtype, device=self.dev)
            self.x, self.h, self.y = z(cfg.hidden), z(cfg.hidden), z(cfg.hidden)
            self.q, self.k, self.v = z(hq), z(hkv), z(hkv)
            self.a, self.qn = z(hq), (None if fuse_rope else z(hq))
            self.m = z(cfg.inter // self.world)
            # gate and up computed by separate launches (Huffman, batch > 2)
            self.gm, self.um = z(cfg.inter // self.world), z(cfg.inter // self.world)
            self.logits_buf = z(cfg.vocab // self.world)
            self.code = _lib.CBQ_BF16 if act_dtype == torch.bfloat16 else _lib.CBQ_F32
            # arrival count of the GEMVs whose last CTA normalises (0 between launches)
            self.arrive = torch.zeros(1, dtype=torch.int32, device=self.dev)
            # split-key attention: partial softmax states + arrival counters (0 between launches)
            n = _lib.query("cbq_attn_workspace_bytes", batch, self.hl, self.kvl, d, max_len)
            self.attn_ws = torch.zeros(n, dtype=torch.uint8, device=self.dev)
        self.peer = None
        if fused and self.world > 1 and allreduce == "peer" and not weights.huffman and batch <= 2:
            self.peer = _PeerAllReduce(self, 2 * cfg.layers)
        # tensor parallel over peer memory: each all-reduce is consumed inside
        # the next GEMV launch (cbq_linear_fixed_multi_allreduce_norm), which
        # writes the updated residual stream into the other of two buffers
        self.peer_prenorm = self.peer is not None and prenorm and not fuse_norm
        if self.peer_prenorm:
            self.xr = (self.x, torch.zeros_like(self.x))
        L = weights.layers
        self.emb = L["model.embed_tokens.weight"]
        self.lm_head = L["lm_head.weight"]
        self.layer_mods = []
        for i in range(cfg.layers):
            p = f"model.layers.{i}."
            self.layer_mods.append(tuple(L[p + n + ".weight"] for n in (
                "self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")))

    # --------------------------------------------------------------- one step
    def _allreduce(self, t):
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def _step(self):
        if self.fused:
            return self._step_fused()
        cfg, B, d, eps, dt = self.cfg, self.B, self.cfg.head_dim, self.cfg.rms_eps, self.dt
        x = self.emb(self.ids, out_dtype=dt)                         # [B, H]
        cos = self.cos.index_select(0, self.pos).to(dt)              # [1, d]
        sin = self.sin.index_select(0, self.pos).to(dt)
        mask = (self.ar <= self.pos).view(1, 1, 1, self.max_len)
        for li, (q_p, k_p, v_p, o_p, g_p, u_p, d_p) in enumerate(self.layer_mods):
            h = _rms(x, eps)
            q = _rms(q_p(h).view(B, self.hl, d), eps)
            k = _rms(k_p(h).view(B, self.kvl, d), eps)
            v = v_p(h).view(B, self.kvl, d)
            q = q * cos + _rotate_half(q) * sin
            k = k * cos + _rotate_half(k) * sin
            self.k_cache[li].index_copy_(2, self.pos, k.unsqueeze(2))
            self.v_cache[li].index_copy_(2, self.pos, v.unsqueeze(2))
            a = F.scaled_dot_product_attention(q.unsqueeze(2), self.k_cache[li], self.v_cache[li],
                                               attn_mask=mask, scale=d ** -0.5, enable_gqa=True)
            x = x + self._allreduce(o_p(a.reshape(B, self.hl * d)))
            h = _rms(x, eps)
            x = x + self._allreduce(d_p(F.silu(g_p(h)) * u_p(h)))
        self._finish(self.lm_head(_rms(x, eps)))                    # logits [B, V / world]

    # ------------------------------------------------------------ fused step
    def _rmsnorm(self, x, out, add=None):
        _lib.call("cbq_rmsnorm", x.data_ptr(), None if add is None else add.data_ptr(), self.code,
                  x.shape[0], x.shape[1], None, float(self.cfg.rms_eps), out.data_ptr(),
                  device_stream(self.dev))

    def _residual_norm(self, lin, x):
        """self.x += x @ W^T, then self.h = RMSNorm(self.x): one launch
        (``cbq_linear_fixed_residual_norm``, whose last CTA normalises) when the
        fused kernel takes the layer, else the GEMV and ``cbq_rmsnorm``."""
        if self.fuse_norm and isinstance(lin, GPUAcceleratedLinear):
            rc = _lib.lib().cbq_linear_fixed_residual_norm(
                x.data_ptr(), self.code, self.B, x.shape[1], lin.packed.data_ptr(), lin.nbytes,
                lin.codebook.data_ptr(), lin.C, lin.bits, lin.M, lin.K, None, self.x.data_ptr(), self.x.shape[1],
                self.code, None, float(self.cfg.rms_eps), self.h.data_ptr(), self.h.shape[1],
                self.arrive.data_ptr(), device_stream(self.dev))
            if rc == _lib.CBQ_OK:
                return
            if rc != _lib.CBQ_ERR_UNSUPPORTED:
                raise _lib.CbqError("cbq_linear_fixed_residual_norm", rc)
        fixed = isinstance(lin, GPUAcceleratedLinear)
        if fixed and linear_fixed_multi((lin,), x, (self.x,), _lib.CBQ_EPI_RESIDUAL, (self.x,)):
            self._rmsnorm(self.x, self.h)
            return
        lin(x, out=self.y)                   # separate launch: the norm launch adds the residual
        self._rmsnorm(self.x, self.h, add=self.y)

    def _linear(self, mats, outs, epilogue=_lib.CBQ_EPI_STORE, resids=None, x=None):
        x = self.h if x is None else x
        fixed = all(isinstance(m, GPUAcceleratedLinear) for m in mats)
        if fixed and linear_fixed_multi(mats, x, outs, epilogue, resids):
            return
        # matrices one by one (Huffman streams, or shapes outside the fused kernel)
        if epilogue == _lib.CBQ_EPI_SILU_MUL:
            if outs[0] is self.m and x.dtype == self.dt:
                mats[0](x, out=self.gm)
                mats[1](x, out=self.um)
                _lib.call("cbq_silu_mul", self.gm.data_ptr(), self.um.data_ptr(), self.code, self.m.numel(),
                          self.m.data_ptr(), device_stream(self.dev))
            else:
                g, u = mats[0](x), mats[1](x)
                outs[0].copy_(F.silu(g) * u)
        elif epilogue == _lib.CBQ_EPI_RESIDUAL:
            for m, o, r in zip(mats, outs, resids):
                o.copy_(r + m(x))
        else:
            for m, o in zip(mats, outs):
                m(x, out=o)

    def _linear_normed(self, mats, outs, epilogue=_lib.CBQ_EPI_STORE):
        """RMSNorm(self.x) @ W^T for ``mats``: the norm inside the GEMV launch
        when ``prenorm`` is on and the shape is supported, else cbq_rmsnorm
        into self.h followed by the GEMV."""
        if self.prenorm and linear_fixed_multi(mats, self.x, outs, epilogue, norm=(None, self.cfg.rms_eps)):
            return
        self._rmsnorm(self.x, self.h)
        self._linear(mats, outs, epilogue)

    def _step_fused(self):
        cfg, B, d, dt = self.cfg, self.B, self.cfg.head_dim, self.dt
        stream = device_stream(self.dev)
        if self.peer is not None:
            self.peer.epoch.add_(1)
        self.emb(self.ids, out=self.x)
        if self.prenorm:
            return self._step_prenorm()
        if self.peer_prenorm:
            return self._step_peer_prenorm()
        self._rmsnorm(self.x, self.h)
        for li, (q_p, k_p, v_p, o_p, g_p, u_p, d_p) in enumerate(self.layer_mods):
            self._linear((q_p, k_p, v_p), (self.q, self.k, self.v))
            ws, nws = self.attn_ws.data_ptr(), self.attn_ws.numel()
            if self.fuse_rope:
                _lib.call("cbq_attn_decode_rope_split", self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(),
                          self.code, B, self.hl, self.kvl, d, float(cfg.rms_eps), None, None, self.cos.data_ptr(),
                          self.sin.data_ptr(), self.pos.data_ptr(), self.k_cache[li].data_ptr(),
                          self.v_cache[li].data_ptr(), self.max_len, float(d ** -0.5), self.a.data_ptr(), ws, nws,
                          stream)
            else:
                _lib.call("cbq_qk_norm_rope", self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), self.code,
                          B, self.hl, self.kvl, d, float(cfg.rms_eps), None, None, self.cos.data_ptr(),
                          self.sin.data_ptr(), self.pos.data_ptr(), self.qn.data_ptr(),
                          self.k_cache[li].data_ptr(), self.v_cache[li].data_ptr(), self.max_len, stream)
                _lib.call("cbq_attn_decode_split", self.qn.data_ptr(), self.k_cache[li].data_ptr(),
                          self.v_cache[li].data_ptr(), self.code, B, self.hl, self.kvl, d, self.max_len,
                          self.pos.data_ptr(), float(d ** -0.5), self.a.data_ptr(), ws, nws, stream)
            if self.world == 1:
                self._residual_norm(o_p, self.a)
            elif self.peer is not None:
                self.peer.run(2 * li, o_p, self.a)
            else:
                self._linear((o_p,), (self.y,), x=self.a)
                self._allreduce(self.y)
                self._rmsnorm(self.x, self.h, add=self.y)
            self._linear((g_p, u_p), (self.m,), _lib.CBQ_EPI_SILU_MUL)
            if self.world == 1:
                self._residual_norm(d_p, self.m)
            elif self.peer is not None:
                self.peer.run(2 * li + 1, d_p, self.m)
            else:
                self._linear((d_p,), (self.y,), x=self.m)
                self._allreduce(self.y)
                self._rmsnorm(self.x, self.h, add=self.y)
        self._finish(self.lm_head(self.h))

    def _step_prenorm(self):
        """One GPU: five launches per layer (q/k/v with the input norm,
        attention, o with the residual add, gate/up with the post-attention
        norm, down with the residual add); the final norm runs in lm_head."""
        cfg, B, d = self.cfg, self.B, self.cfg.head_dim
        stream = device_stream(self.dev)
        ws, nws = self.attn_ws.data_ptr(), self.attn_ws.numel()
        for li, (q_p, k_p, v_p, o_p, g_p, u_p, d_p) in enumerate(self.layer_mods):
            self._linear_normed((q_p, k_p, v_p), (self.q, self.k, self.v))
            _lib.call("cbq_attn_decode_rope_split", self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(),
                      self.code, B, self.hl, self.kvl, d, float(cfg.rms_eps), None, None, self.cos.data_ptr(),
                      self.sin.data_ptr(), self.pos.data_ptr(), self.k_cache[li].data_ptr(),
                      self.v_cache[li].data_ptr(), self.max_len, float(d ** -0.5), self.a.data_ptr(), ws, nws,
                      stream)
            self._linear((o_p,), (self.x,), _lib.CBQ_EPI_RESIDUAL, (self.x,), x=self.a)
            self._linear_normed((g_p, u_p), (self.m,), _lib.CBQ_EPI_SILU_MUL)
            self._linear((d_p,), (self.x,), _lib.CBQ_EPI_RESIDUAL, (self.x,), x=self.m)
        if isinstance(self.lm_head, GPUAcceleratedLinear):
            self._linear_normed((self.lm_head,), (self.logits_buf,))
            self._finish(self.logits_buf)
        else:
            self._rmsnorm(self.x, self.h)
            self._finish(self.lm_head(self.h))

    def _consume(self, site: int, j: int, mats, outs, epilogue=_lib.CBQ_EPI_STORE) -> int:
        """The GEMV that consumes all-reduce ``site``: reads residual buffer
        j % 2 plus every rank's partial rows, writes buffer (j + 1) % 2,
        normalises and multiplies; returns the next consumer index."""
        pr = self.peer
        W = pr.W
        src, dst = self.xr[j % 2], self.xr[(j + 1) % 2]
        ar = (W, src, pr.local_flagged(site), None, pr.epoch.data_ptr(), self.cfg.hidden, pr.status.data_ptr())
        if not linear_fixed_multi(mats, dst, outs, epilogue, norm=(None, self.cfg.rms_eps), allreduce=ar):
            raise RuntimeError("tensor-parallel all-reduce GEMV: shape not supported by the fused kernel")
        return j + 1

    def _step_peer_prenorm(self):
        """Tensor parallel over peer memory, five launches per layer: q/k/v
        (consuming the previous layer's down_proj all-reduce, norm inside),
        attention, o_proj writing its partial rows to every rank, gate/up
        (consuming o_proj's all-reduce, norm inside), down_proj writing its
        partial rows to every rank; lm_head consumes the last all-reduce."""
        cfg, B, d = self.cfg, self.B, self.cfg.head_dim
        stream = device_stream(self.dev)
        ws, nws = self.attn_ws.data_ptr(), self.attn_ws.numel()
        j = 0
        for li, (q_p, k_p, v_p, o_p, g_p, u_p, d_p) in enumerate(self.layer_mods):
            if li == 0:
                if not linear_fixed_multi((q_p, k_p, v_p), self.xr[0], (self.q, self.k, self.v),
                                          norm=(None, cfg.rms_eps)):
                    raise RuntimeError("q/k/v GEMV: shape not supported by the fused kernel")
            else:
                j = self._consume(2 * li - 1, j, (q_p, k_p, v_p), (self.q, self.k, self.v))
            _lib.call("cbq_attn_decode_rope_split", self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(),
                      self.code, B, self.hl, self.kvl, d, float(cfg.rms_eps), None, None, self.cos.data_ptr(),
                      self.sin.data_ptr(), self.pos.data_ptr(), self.k_cache[li].data_ptr(),
                      self.v_cache[li].data_ptr(), self.max_len, float(d ** -0.5), self.a.data_ptr(), ws, nws,
                      stream)
            self.peer.produce(2 * li, o_p, self.a)
            j = self._consume(2 * li, j, (g_p, u_p), (self.m,), _lib.CBQ_EPI_SILU_MUL)
            self.peer.produce(2 * li + 1, d_p, self.m)
        if not isinstance(self.lm_head, GPUAcceleratedLinear):
            raise RuntimeError("lm_head must be fixed width on the peer-memory path")
        self._consume(2 * cfg.layers - 1, j, (self.lm_head,), (self.logits_buf,))
        self._finish(self.logits_buf)

    def _finish(self, logits):
        self.logits = logits
        if self.fused and (self.world == 1 or self.peer is not None) and logits.is_contiguous():
            # one launch: the row argmax, exchanged between ranks through
            # epoch-flagged words in peer memory (cbq_greedy_pick)
            pr = self.peer
            code = _lib.CBQ_BF16 if logits.dtype == torch.bfloat16 else _lib.CBQ_F32
            lg = logits if logits.dtype in (torch.bfloat16, torch.float32) else logits.float()
            _lib.call("cbq_greedy_pick", lg.data_ptr(), code, self.B, lg.shape[-1], lg.shape[-1], self.rank,
                      self.world, None if pr is None else pr.pick, None if pr is None else pr.local_pick,
                      None if pr is None else pr.epoch.data_ptr(), self.next_ids.data_ptr(),
                      None if pr is None else pr.status.data_ptr(), device_stream(self.dev))
            return
        val, idx = logits.float().max(dim=-1)
        idx = idx + self.rank * self.vocab_local
        if self.world > 1:
            vals = [torch.empty_like(val) for _ in range(self.world)]
            idxs = [torch.empty_like(idx) for _ in range(self.world)]
            dist.all_gather(vals, val, group=self.group)
            dist.all_gather(idxs, idx, group=self.group)
            best = torch.stack(vals).max(dim=0).indices              # first rank on ties
            idx = torch.stack(idxs).gather(0, best.unsqueeze(0)).squeeze(0)
        self.next_ids.copy_(idx)

    def launches_per_step(self) -> int:
        """libcbq kernel launches in one step (embedding, linears, fused block kernels)."""
        n = self.cfg.layers
        if not self.fused:
            return 1 + 7 * n + 1          # embedding, 7 linears per layer, lm_head
        attn = 1 if self.fuse_rope else 2
        if self.prenorm or self.peer_prenorm:   # embedding, 5 per layer (norms inside the GEMVs), lm_head, pick
            return 1 + 5 * n + 2
        pick = 1 if (self.world == 1 or self.peer is not None) else 0   # cbq_greedy_pick
        if self.w.huffman or self.B > 2:  # one launch per linear, separate RMSNorms (+ residual), SiLU * up
            per = 3 + attn + 1 + 1 + 2 + 1 + 1 + 1
        elif (self.world == 1 or self.peer is not None) and self.fuse_norm:
            per = 4 + attn                # q/k/v, attention, o (+norm), gate/up, down (+norm)
        else:
            per = 6 + attn                # the same with two RMSNorm launches (after NCCL at TP > 1)
        return 2 + per * n + 1 + pick     # embedding + first RMSNorm, the layers, lm_head

    def layer_launches(self) -> str:
        """The launches of one decoder layer of the step, in order."""
        if not self.fused:
            return "one per linear layer, torch operations around them"
        attn = "attention (q/k norm + rope, split keys)" if self.fuse_rope else "q/k norm + rope, attention"
        if self.prenorm:
            return f"q/k/v (+ input norm), {attn}, o (+ residual), gate/up (+ norm, SiLU*up), down (+ residual)"
        if self.peer_prenorm:
            return (f"q/k/v (+ all-reduce of down, norm), {attn}, o (partial rows to every rank), "
                    f"gate/up (+ all-reduce of o, norm, SiLU*up), down (partial rows to every rank)")
        if self.w.huffman or self.B > 2:
            return f"q, k, v, {attn}, o, residual + norm, gate, up, SiLU*up, down, residual + norm"
        norm = " + norm" if self.fuse_norm else ", norm"
        ar = " (peer all-reduce)" if self.peer is not None else (" + NCCL all-reduce" if self.world > 1 else "")
        return f"q/k/v, {attn}, o{ar}{norm}, gate/up, down{ar}{norm}"

    def step(self, ids: torch.Tensor, pos: int) -> torch.Tensor:
        """Eager step (no graph): returns the greedy next ids [B]."""
        self.ids.copy_(ids)
        self.pos.fill_(pos)
        self._step()
        return self.next_ids

    def capture(self, warmup: int = 2) -> None:
        """Warm up then capture one step in a CUDA graph."""
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        torch.cuda.synchronize(self.dev)

    def release(self) -> None:
        """Drop the graph (before destroying an NCCL process group)."""
        self.graph = None
        torch.cuda.synchronize(self.dev)

    def reset(self) -> None:
        for k, v in zip(self.k_cache, self.v_cache):
            k.zero_()
            v.zero_()

    def run_step(self) -> None:
        if self.graph is not None:
            self.graph.replay()
        else:
            self._step()

    def generate(self, prompt: torch.Tensor, n_new: int) -> torch.Tensor:
        """Greedy tokens [B, n_new] after the prompt [B, S] (fed one token per step)."""
        B, S = prompt.shape
        if S + n_new > self.max_len:
            raise ValueError("sequence longer than the cache")
        prompt = prompt.to(self.dev)
        out = torch.empty(B, n_new, dtype=torch.int64, device=self.dev)
        self.pos.zero_()
        for t in range(S):
            self.ids.copy_(prompt[:, t])
            self.run_step()
            self.pos.add_(1)
        for t in range(n_new):
            out[:, t].copy_(self.next_ids)
            self.ids.copy_(self.next_ids)
            if t + 1 < n_new:
                self.run_step()
                self.pos.add_(1)
        return out
