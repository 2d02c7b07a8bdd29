"""A Qwen2 decode step around the B200 paged-decode path (benchmark workload C5).

infrared runs its model as ``Qwen2ForCausalLM.forward`` (infrared/model/qwen2.py:
89-118): per layer RMSNorm -> q/k/v projections (with bias) -> RoPE
(infrared/model/layers.py:79-89, 121-136) -> paged attention (the path this
package replaces) -> o projection -> residual -> RMSNorm -> SwiGLU MLP
(:185-196) -> residual; final norm and lm_head; greedy sampling. This module
restates that decode step for a whole batch in plain PyTorch (GEMMs and
elementwise ops are library calls; RoPE, the K/V cache write and the GQA
decode are one kernel, ``paged_decode_rope_write``, fed with row views of
the QKV projection output) with random weights, so the attention kernels can
be measured inside a real 28-layer decode step under CUDA-graph replay. It is a measurement harness for the path, not a model
implementation to serve with: no prefill (the KV history is synthetic, as in
the kernel benchmarks) and no tokenizer.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

from . import ops


@dataclass(frozen=True)
class Qwen2Geometry:
    vocab: int
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    inter: int
    eps: float = 1e-6
    theta: float = 1e6


QWEN25_7B = Qwen2Geometry(152064, 3584, 28, 28, 4, 128, 18944)


class Qwen2DecodeStep:
    """Random-init Qwen2 weights, a paged K/V pool holding a synthetic history
    for ``batch`` sequences, and ``step()``: one greedy decode token for all.

    ``fuse_rope`` (class attribute): True runs RoPE inside the attention
    kernel; False rotates q/k with PyTorch ops first (infrared's
    apply_rotary_pos_emb) and calls :meth:`attention` on the rotated rows.
    """

    fuse_rope = True

    def __init__(self, geo: Qwen2Geometry, context_lens, max_new: int, block_size: int = 16,
                 device="cuda", dtype=torch.bfloat16, seed: int = 0, std: float = 0.02):
        self.geo, self.bs, self.dtype = geo, block_size, dtype
        dev = torch.device(device)
        self.device = dev
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        ctx = np.asarray(context_lens, dtype=np.int64)
        self.batch = b = len(ctx)
        h, d, hq, hkv = geo.hidden, geo.head_dim, geo.heads, geo.kv_heads

        def rnd(*shape, s=std):
            return (torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * s).to(dtype)

        self.embed = rnd(geo.vocab, h)
        self.lm_head = rnd(h, geo.vocab)
        self.final_norm = torch.ones(h, device=dev, dtype=dtype)
        self.layers = []
        for _ in range(geo.layers):
            self.layers.append({
                "ln1": torch.ones(h, device=dev, dtype=dtype),
                "ln2": torch.ones(h, device=dev, dtype=dtype),
                "wqkv": rnd(h, (hq + 2 * hkv) * d),
                "bqkv": rnd((hq + 2 * hkv) * d),
                "wo": rnd(hq * d, h),
                "wgu": rnd(h, 2 * geo.inter),
                "wd": rnd(geo.inter, h),
            })
        # pool: every sequence owns consecutive random blocks for ctx + max_new tokens
        self.max_blocks = int(-(-(ctx.max() + max_new) // block_size))
        nblk = b * self.max_blocks
        perm = np.random.default_rng(seed).permutation(nblk).astype(np.int32)
        self.block_tables = torch.from_numpy(perm.reshape(b, self.max_blocks)).to(dev)
        self.num_slots = nblk * block_size
        shape = (geo.layers, self.num_slots, hkv, d)
        self.k_pool = torch.empty(shape, device=dev, dtype=dtype)
        self.v_pool = torch.empty(shape, device=dev, dtype=dtype)
        for l in range(geo.layers):   # synthetic history, N(0, 0.5)
            self.k_pool[l].normal_(0.0, 0.5, generator=g)
            self.v_pool[l].normal_(0.0, 0.5, generator=g)
        # decode state: the next token sits at position ctx (history [0, ctx))
        self.positions = torch.from_numpy(ctx).to(dev)
        self.ids = torch.randint(0, geo.vocab, (b,), generator=g, device=dev)
        inv = 1.0 / (geo.theta ** (torch.arange(0, d, 2, device=dev, dtype=torch.float32) / d))
        self.inv_freq = inv
        self.scale = d ** -0.5
        self.ws = torch.empty(0, dtype=torch.uint8, device=dev)

    # -- building blocks (infrared/model/layers.py) ------------------------

    def _rms(self, x, w):
        """RMSNorm of infrared (layers.py:56-69): fp32 normalisation, cast, then
        the weight. One fused library kernel (normalise in fp32, scale by the
        weight, round once) — the same values for the unit weights used here."""
        return F.rms_norm(x, (x.shape[-1],), w, self.geo.eps)

    def _rope(self, x, cos, sin):
        half = x.shape[-1] // 2
        rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
        return x * cos + rot * sin

    def attention(self, layer: int, q, k, v, slots, ctx):
        """Write this step's (rotated) K/V and attend: the fused kernel."""
        return ops.paged_decode_write(q, k, v, self.k_pool[layer], self.v_pool[layer], slots,
                                      self.block_tables, ctx, self.scale, self.bs)

    def attend(self, layer: int, q, k, v, slots, ctx, cos, sin):
        """RoPE + cache write + decode of one layer on un-rotated q/k/v views."""
        if self.fuse_rope:
            return ops.paged_decode_rope_write(q, k, v, self.k_pool[layer], self.v_pool[layer],
                                               slots, self.block_tables, ctx, cos, sin,
                                               self.scale, self.bs)
        c = cos.to(self.dtype).unsqueeze(1)
        s = sin.to(self.dtype).unsqueeze(1)
        return self.attention(layer, self._rope(q, c, s), self._rope(k, c, s), v.contiguous(),
                              slots, ctx)

    def step(self) -> torch.Tensor:
        """One decode token for every sequence; advances ids / positions in place
        (so a captured graph of step() can be replayed token after token)."""
        geo, b = self.geo, self.batch
        hq, hkv, d = geo.heads, geo.kv_heads, geo.head_dim
        pos = self.positions
        ctx = (pos + 1).to(torch.int32)
        slots = (self.block_tables.gather(1, (pos // self.bs).unsqueeze(1)).squeeze(1).long()
                 * self.bs + pos % self.bs)
        freqs = pos.float().unsqueeze(1) * self.inv_freq
        emb = torch.cat((freqs, freqs), dim=-1)
        cos, sin = emb.cos(), emb.sin()          # fp32 [B, D], as RotaryEmbedding returns
        x = self.embed[self.ids]
        for l, w in enumerate(self.layers):
            hdn = self._rms(x, w["ln1"])
            qkv = torch.addmm(w["bqkv"], hdn, w["wqkv"])
            q = qkv[:, : hq * d].view(b, hq, d)
            k = qkv[:, hq * d:(hq + hkv) * d].view(b, hkv, d)
            v = qkv[:, (hq + hkv) * d:].view(b, hkv, d)
            attn = self.attend(l, q, k, v, slots, ctx, cos, sin)
            # residual adds folded into the GEMMs (C = x + A.B, one rounding)
            x = torch.addmm(x, attn.view(b, hq * d), w["wo"])
            hdn = self._rms(x, w["ln2"])
            gate, up = (hdn @ w["wgu"]).chunk(2, dim=-1)
            x = torch.addmm(x, F.silu(gate) * up, w["wd"])
        logits = self._rms(x, self.final_norm) @ self.lm_head
        nxt = torch.argmax(logits, dim=-1)
        self.ids.copy_(nxt)
        self.positions.add_(1)
        return logits

    def reference_attention(self, layer, q, k, v, slots, ctx):
        """Plain-PyTorch attention of the same step (write, gather, softmax in
        fp32), the naive path of infrared (triton_attention.py:81-129)."""
        self.k_pool[layer][slots] = k
        self.v_pool[layer][slots] = v
        out = torch.empty_like(q)
        rep = self.geo.heads // self.geo.kv_heads
        for i in range(self.batch):
            c = int(ctx[i])
            p = torch.arange(c, device=q.device)
            sl = self.block_tables[i, p // self.bs].long() * self.bs + p % self.bs
            kk = self.k_pool[layer][sl].float().repeat_interleave(rep, dim=1)   # [c, H, D]
            vv = self.v_pool[layer][sl].float().repeat_interleave(rep, dim=1)
            s = torch.einsum("hd,chd->hc", q[i].float(), kk) * self.scale
            out[i] = torch.einsum("hc,chd->hd", torch.softmax(s, -1), vv).to(q.dtype)
        return out

    def weight_bytes(self) -> int:
        n = self.embed.numel() * 0 + self.lm_head.numel()   # one embedding row per token only
        for w in self.layers:
            n += sum(t.numel() for t in w.values())
        return n * self.embed.element_size()

    def kv_bytes_per_step(self) -> int:
        ctx = self.positions.double() + 1
        return int(ctx.sum().item()) * 2 * self.geo.kv_heads * self.geo.head_dim * \
            self.k_pool.element_size() * self.geo.layers


def random_context_lens(batch: int, lo: int, hi: int, seed: int = 0) -> np.ndarray:
    return np.random.default_rng(seed).integers(lo, hi + 1, size=batch)


def tiny_geometry() -> Qwen2Geometry:
    """A small geometry of the same structure for parity tests."""
    return Qwen2Geometry(vocab=512, hidden=256, layers=2, heads=8, kv_heads=2, head_dim=64,
                         inter=512)


__all__ = ["QWEN25_7B", "Qwen2DecodeStep", "Qwen2Geometry", "random_context_lens",
           "tiny_geometry", "math"]
