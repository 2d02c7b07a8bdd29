"""Install the B200 kernels behind infrared's own paged-attention seam.

infrared's ``Attention.forward`` calls ``paged_attention(q, k, v, paged,
mask, layer_idx, scale, n_rep)`` (infrared/model/triton_attention.py:81-107),
which first scatters this step's K/V with ``paged.pool.write`` and then, when
``_should_use_triton(q, paged.use_triton)`` says so, reads the history with
``_paged_attention_triton``; otherwise it runs the naive gather path. Both
names are module globals looked up at call time, and ``PagedKVPool.write``
is a class attribute (infrared/cache/paged_kv_cache.py:48), so replacing
those three routes the engine's decode steps — eager
(infrared/engine/paged_engine.py:290-332) and CUDA-graph
(infrared/engine/cuda_graph.py:231-287) — to this package without editing
infrared:

* ``PagedKVPool.write`` on CUDA tensors -> ``ir_cache_write``;
* ``_should_use_triton`` -> True for CUDA decode calls (``Sq == 1``) with
  ``head_dim`` 64 or 128 in fp32 / bf16 / fp16 and ``use_triton`` set;
  with ``prefill=True`` also for packed prefill / mixed frames (``B == 1``,
  ``Sq > 1``), which otherwise keep infrared's own path;
* ``_paged_attention_triton`` -> ``ir_derive_block_metadata`` (once per
  forward) + ``ir_paged_decode`` for decode calls, and
  ``ir_derive_varlen_metadata`` (once per forward) + ``ir_paged_prefill``
  (tcgen05 tensor cores) for packed frames;
* (optional, ``graph_inputs=True``) ``cuda_graph.build_decode_static_inputs``
  (infrared/engine/cuda_graph.py:105-155, a module global read by
  ``CudaGraphDecoder.decode`` at :211) -> ``ir_build_decode_inputs`` for CUDA
  devices, which removes the per-element Python loop of every graph step;
* (optional, ``eager_inputs=True``) ``PagedBatchEngine._decode_logits_eager``
  (infrared/engine/paged_engine.py:290-332, a method) -> the same forward
  with its decode inputs (write slots, per-row slot lists, mask, positions,
  ids) built by ``ir_build_decode_inputs`` in one launch instead of one
  small tensor build per sequence; other devices keep infrared's method;
* (optional, ``fuse_rope=True``) ``layers.Attention.forward``
  (infrared/model/layers.py:156-182, a class attribute) -> the same
  projections, then ONE ``ir_paged_decode_rope_write`` that applies RoPE to
  q and the new K, writes K/V and attends, for paged CUDA decode calls the
  gate accepts; every other call runs infrared's own forward;
* (optional, ``fuse_kv_proj=True``, implies the above) for bf16 / fp16
  decode calls with ``hidden % 64 == 0`` the K and V projections themselves
  run in ``ir_kv_proj_rope_write`` (tensor cores; bias, RoPE and the pool
  write in its epilogue: the new K/V rows go from the accumulator to their
  slots), then ``ir_paged_decode_rope`` attends with RoPE applied to q.

The replacement read path trusts the engine's decode metadata: the mask is a
prefix of zeros and ``gather_slots`` lists whole blocks; a call that breaks
either is reported by the device error flag (``check_device_errors``).
"""

from __future__ import annotations

import importlib
from dataclasses import dataclass

import torch

from . import ops
from .attention import block_metadata, prefill_frame

_SUPPORTED = (torch.float32, torch.bfloat16, torch.float16)


def should_use_b200(q: torch.Tensor, want: bool) -> bool:
    """Gate with the reference's signature (triton_attention.py:68-76)."""
    return (bool(want) and q.is_cuda and q.dim() == 4 and q.shape[1] == 1
            and q.shape[-1] in (64, 128) and q.dtype in _SUPPORTED)


def should_use_b200_with_prefill(q: torch.Tensor, want: bool) -> bool:
    """The gate plus packed Sq > 1 frames (B == 1)."""
    return (bool(want) and q.is_cuda and q.dim() == 4 and
            (q.shape[1] == 1 or q.shape[0] == 1)
            and q.shape[-1] in (64, 128) and q.dtype in _SUPPORTED)


def paged_attention_b200(q: torch.Tensor, paged, mask: torch.Tensor, layer_idx: int,
                         scale: float, n_rep: int) -> torch.Tensor:
    """Read path with the signature of ``_paged_attention_triton``
    (triton_attention.py:310-318): the pool already holds this step's K/V."""
    b, sq, h, d = q.shape
    if sq != 1:
        return prefill_frame(q, paged, mask, layer_idx, scale)
    pool = paged.pool
    bt, ctx = block_metadata(paged, mask)
    out = torch.empty((b, sq, h, d), dtype=q.dtype, device=q.device)
    ops.paged_decode(q.reshape(b, h, d), pool.k[layer_idx], pool.v[layer_idx], bt, ctx,
                     scale, pool.block_size, out=out.view(b, h, d))
    return out


def _make_write(original):
    def write(self, layer_idx, k, v, slots):
        if k.is_cuda and k.dtype in _SUPPORTED and self.k.dtype == k.dtype:
            ops.cache_write(k, v, self.k[layer_idx], self.v[layer_idx], slots)
        else:
            original(self, layer_idx, k, v, slots)
    write.__doc__ = "PagedKVPool.write on the B200 cache-write kernel (CUDA tensors)."
    return write


def _make_attention_forward(original, fuse_kv_proj: bool = False):
    def forward(self, x, ctx, layer_idx):
        paged = ctx.paged
        b = x.shape[0]
        # the gate of should_use_b200, applied to the layer's input
        if (paged is None or not paged.use_triton or x.dim() != 3 or x.shape[1] != 1
                or not x.is_cuda or x.dtype not in _SUPPORTED
                or self.head_dim not in (64, 128) or paged.pool.k.dtype != x.dtype
                or ctx.cos.dtype != torch.float32 or ctx.cos.numel() != b * self.head_dim):
            return original(self, x, ctx, layer_idx)
        q = self.q_proj(x).view(b, self.num_heads, self.head_dim)
        pool = paged.pool
        bt, cl = block_metadata(paged, ctx.mask)
        cos = ctx.cos.reshape(b, self.head_dim)
        sin = ctx.sin.reshape(b, self.head_dim)
        if fuse_kv_proj and x.dtype != torch.float32 and x.shape[-1] % 64 == 0:
            # K/V projected, rotated and written to the pool in one kernel
            ops.kv_proj_rope_write(x.reshape(b, x.shape[-1]), self.k_proj.weight,
                                   self.v_proj.weight, self.k_proj.bias, self.v_proj.bias,
                                   cos, sin, paged.write_slots.reshape(-1),
                                   pool.k[layer_idx], pool.v[layer_idx])
            out = ops.paged_decode_rope(q, pool.k[layer_idx], pool.v[layer_idx], bt, cl, cos,
                                        sin, self.scale, pool.block_size)
            return self.o_proj(out.view(b, 1, self.num_heads * self.head_dim))
        k = self.k_proj(x).view(b, self.num_kv_heads, self.head_dim)
        v = self.v_proj(x).view(b, self.num_kv_heads, self.head_dim)
        out = ops.paged_decode_rope_write(q, k, v, pool.k[layer_idx], pool.v[layer_idx],
                                          paged.write_slots.reshape(-1), bt, cl,
                                          ctx.cos.reshape(b, self.head_dim),
                                          ctx.sin.reshape(b, self.head_dim), self.scale,
                                          pool.block_size)
        return self.o_proj(out.view(b, 1, self.num_heads * self.head_dim))
    forward.__doc__ = ("Attention.forward with RoPE + cache write + decode in one kernel "
                       "for paged CUDA decode calls.")
    return forward


def _make_decode_logits_eager(original, paged_context_cls):
    from .graph_inputs import build_decode_static_inputs as on_device

    def _decode_logits_eager(self, running):
        device, dtype = self.model.device, self.model.dtype
        if torch.device(device).type != "cuda" or not running:
            return original(self, running)
        num_cached = [s.num_cached_tokens for s in running]
        inp = on_device([s.block_table for s in running], num_cached,
                        [s.last_token for s in running], len(running), max(num_cached) + 1,
                        self.block_size, device, dtype)
        logits = self.model.forward(
            inp.ids, inp.positions, inp.mask,
            paged=paged_context_cls(self.pool, inp.write_slots, inp.gather_slots,
                                    use_triton=self.enable_triton_attention))
        return logits[:, -1]
    _decode_logits_eager.__doc__ = ("PagedBatchEngine._decode_logits_eager with its inputs "
                                    "built on the device (ir_build_decode_inputs).")
    return _decode_logits_eager


def _make_graph_inputs(original, decode_inputs_cls):
    from .graph_inputs import build_decode_static_inputs as on_device

    def build(block_tables, num_cached, last_tokens, bucket_b, t_max, block_size, device,
              dtype):
        if torch.device(device).type == "cuda":
            return on_device(block_tables, num_cached, last_tokens, bucket_b, t_max,
                             block_size, device, dtype, decode_inputs_cls)
        return original(block_tables, num_cached, last_tokens, bucket_b, t_max, block_size,
                        device, dtype)
    build.__doc__ = "build_decode_static_inputs on the device (ir_build_decode_inputs)."
    return build


@dataclass
class Installed:
    """Handle of an installation; ``uninstall()`` restores infrared's functions."""

    triton_attention: object
    pool_cls: object
    saved: dict
    cuda_graph: object = None
    attention_cls: object = None
    engine_cls: object = None

    def uninstall(self) -> None:
        self.triton_attention._should_use_triton = self.saved["gate"]
        self.triton_attention._paged_attention_triton = self.saved["read"]
        self.pool_cls.write = self.saved["write"]
        if self.cuda_graph is not None:
            self.cuda_graph.build_decode_static_inputs = self.saved["graph_inputs"]
        if self.attention_cls is not None:
            self.attention_cls.forward = self.saved["forward"]
        if self.engine_cls is not None:
            self.engine_cls._decode_logits_eager = self.saved["eager"]


def install(triton_attention=None, paged_kv_cache=None, cuda_graph=None,
            graph_inputs: bool = True, layers=None, fuse_rope: bool = False,
            prefill: bool = False, paged_engine=None,
            eager_inputs: bool = False, fuse_kv_proj: bool = False) -> Installed:
    """Route infrared's paged decode attention to the B200 kernels.

    ``triton_attention`` / ``paged_kv_cache`` / ``cuda_graph`` / ``layers``
    default to the installed ``infrared.model.triton_attention``,
    ``infrared.cache.paged_kv_cache``, ``infrared.engine.cuda_graph`` and
    ``infrared.model.layers`` modules (any modules with the same names and call
    contract work); ``graph_inputs=False`` leaves infrared's graph-input
    builder alone; ``fuse_rope=True`` also replaces ``Attention.forward`` so
    that RoPE runs inside the decode kernel; ``prefill=True`` also routes
    packed prefill / mixed frames (``Sq > 1``) to the tensor-core kernel;
    ``eager_inputs=True`` builds the eager decode step's inputs on the device
    (``paged_engine`` defaults to ``infrared.engine.paged_engine``);
    ``fuse_kv_proj=True`` (implies ``fuse_rope``) also runs the K/V projections
    of 16-bit decode calls in the tensor-core kernel that writes the pool.
    """
    ta = triton_attention or importlib.import_module("infrared.model.triton_attention")
    pk = paged_kv_cache or importlib.import_module("infrared.cache.paged_kv_cache")
    cg = None
    if graph_inputs:
        cg = cuda_graph or importlib.import_module("infrared.engine.cuda_graph")
    pool_cls = pk.PagedKVPool
    saved = {"gate": ta._should_use_triton, "read": ta._paged_attention_triton,
             "write": pool_cls.write}
    ta._should_use_triton = should_use_b200_with_prefill if prefill else should_use_b200
    ta._paged_attention_triton = paged_attention_b200
    pool_cls.write = _make_write(saved["write"])
    if cg is not None:
        saved["graph_inputs"] = cg.build_decode_static_inputs
        cg.build_decode_static_inputs = _make_graph_inputs(saved["graph_inputs"],
                                                           cg.DecodeInputs)
    attn_cls = None
    if fuse_rope or fuse_kv_proj:
        ly = layers or importlib.import_module("infrared.model.layers")
        attn_cls = ly.Attention
        saved["forward"] = attn_cls.forward
        attn_cls.forward = _make_attention_forward(saved["forward"], fuse_kv_proj)
    eng_cls = None
    if eager_inputs:
        pe = paged_engine or importlib.import_module("infrared.engine.paged_engine")
        eng_cls = pe.PagedBatchEngine
        saved["eager"] = eng_cls._decode_logits_eager
        eng_cls._decode_logits_eager = _make_decode_logits_eager(saved["eager"], pk.PagedContext)
    return Installed(ta, pool_cls, saved, cg, attn_cls, eng_cls)
