"""infrared_b200 — B200-native paged-decode attention for the infrared engine.

Three hand-written sm_100a CUDA paths behind a C ABI
(``include/infrared_b200.h``, ``libinfrared_b200.so``):

* ``cache_write`` — scatter of a step's K/V into the paged pool;
* ``paged_decode`` / ``paged_decode_write`` / ``paged_decode_rope_write`` —
  GQA decode attention over block tables (optionally fused with the cache
  write, and with the rotary embedding of q and the new K), split across all
  SMs in equal token shares with a log-sum-exp merge;
* ``kv_proj_rope_write`` — the K/V projections of a step's new tokens with
  bias, RoPE and the pool write in the epilogue (tcgen05 tensor cores), and
  ``paged_decode_rope`` — decode with RoPE on q, for such a step;
* ``paged_decode_lse`` + ``lse_merge`` — partials of a KV range and their
  combination, used to spread one long context over several GPUs;
* ``paged_prefill`` — causal attention of packed query rows (prefill with a
  cached prefix, mixed prefill + decode frames) on the tcgen05 tensor cores.

``PagedKVPool``, ``PagedContext`` and ``paged_attention`` keep the
reference engine's interface; ``shim.install()`` routes infrared's own
decode calls here; ``dist`` shards the work over the GPUs of one node.
"""

from ._lib import InfraredB200Error, UnsupportedShape
from .attention import paged_attention
from .ops import (DeviceError, cache_gather, cache_write, check_device_errors,
                  derive_block_metadata, kv_proj_rope_write, lse_merge, paged_decode,
                  paged_decode_lse, paged_decode_rope, paged_decode_rope_write,
                  paged_decode_write, paged_prefill)
from .paged_kv_cache import PagedContext, PagedKVPool

__all__ = [
    "DeviceError", "InfraredB200Error", "PagedContext", "PagedKVPool", "UnsupportedShape",
    "cache_gather", "cache_write", "check_device_errors", "derive_block_metadata",
    "kv_proj_rope_write", "lse_merge", "paged_attention", "paged_decode", "paged_decode_lse",
    "paged_decode_rope", "paged_decode_rope_write", "paged_decode_write", "paged_prefill",
]
