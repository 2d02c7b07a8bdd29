"""Generate the golden fixtures by running the REFERENCE engine's own code.

Run where the infrared reference is importable (``tests/infrared_ref.py``:
``INFRARED_REF`` names a checkout; by default the repository's own
``baseline/_ref`` install from ``oracle/reference_install.py``):

    python tests/golden/make_golden.py

For every case in ``cases.py`` it rebuilds the seeded inputs, calls
infrared's naive path ``paged_attention(..., PagedContext(use_triton=False))``
(infrared/model/triton_attention.py:81-129) in fp32 on the CPU, its
``build_decode_static_inputs`` (infrared/engine/cuda_graph.py:105-155) and
``paged_attention_blockwise_reference`` (:135-177), and stores outputs plus
input digests in ``tests/golden/golden.npz``. The tests and the GPU runs only
read that file; they never import the reference.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parent))
import infrared_ref  # noqa: E402

if not infrared_ref.importable():
    sys.exit("infrared not found: set INFRARED_REF to a checkout or run "
             "python -m oracle.reference_install")

import torch  # noqa: E402

import cases  # noqa: E402
from infrared.cache.paged_kv_cache import PagedContext, PagedKVPool  # noqa: E402
from infrared.engine.cuda_graph import build_decode_static_inputs  # noqa: E402
from infrared.model.inputs import build_attention_mask, build_varlen_mask  # noqa: E402
from infrared.model.layers import (RotaryEmbedding, apply_rotary_pos_emb,  # noqa: E402
                                   repeat_kv)
from infrared.model.triton_attention import (  # noqa: E402
    paged_attention, paged_attention_blockwise_reference)


def run_attention_case(name: str, out: dict) -> None:
    w, q, kp, vp, kn, vn = cases.attention_inputs(name)
    s = cases.seam_tensors(w, q, kp, vp, kn, vn)
    pool = PagedKVPool(1, w.num_blocks, w.block_size, w.num_kv_heads, w.head_dim,
                       torch.float32)
    pool.k.copy_(torch.from_numpy(s["pool_k"]))
    pool.v.copy_(torch.from_numpy(s["pool_v"]))
    ctx = PagedContext(pool, torch.from_numpy(s["write_slots"]),
                       torch.from_numpy(s["gather_slots"]), use_triton=False)
    res = paged_attention(torch.from_numpy(s["q"]), torch.from_numpy(s["k"]),
                          torch.from_numpy(s["v"]), ctx, torch.from_numpy(s["mask"]), 0,
                          w.scale, w.n_rep)
    out[f"{name}/out"] = res.numpy()[:, 0]          # [B, H, D]
    out[f"{name}/input_digest"] = np.array(cases.input_digest(name))
    out[f"{name}/pool_digest"] = np.array(cases.digest(pool.k.numpy(), pool.v.numpy()))


def run_graph_case(name: str, out: dict) -> None:
    tables, num_cached, last, bucket, t_max, bs = cases.graph_case_args(name)
    inp = build_decode_static_inputs(tables, num_cached, last, bucket, t_max, bs, "cpu",
                                     torch.float32)
    for key in ("ids", "positions", "write_slots", "gather_slots", "mask"):
        out[f"{name}/{key}"] = getattr(inp, key).numpy()


def run_blockwise(out: dict) -> None:
    w, q, kp, vp, kn, vn = cases.attention_inputs("g7_d64_bs16_shared")
    s = cases.seam_tensors(w, q, kp, vp, kn, vn)
    # history incl. the written new token, gathered like the naive path
    kpool, vpool = s["pool_k"][0].copy(), s["pool_v"][0].copy()
    kpool[s["write_slots"]] = kn
    vpool[s["write_slots"]] = vn
    k_all = repeat_kv(torch.from_numpy(kpool[s["gather_slots"]]), w.n_rep)
    v_all = repeat_kv(torch.from_numpy(vpool[s["gather_slots"]]), w.n_rep)
    for bn in cases.BLOCKWISE_BLOCKS:
        res = paged_attention_blockwise_reference(torch.from_numpy(s["q"]), k_all, v_all,
                                                  torch.from_numpy(s["mask"]), w.scale, bn)
        out[f"blockwise/{bn}"] = res.numpy()[:, 0]


def run_rope_case(name: str, theta: float, out: dict) -> None:
    """RoPE at the new token's position, then the naive path on the rotated
    q and k (what Attention.forward does, infrared/model/layers.py:160-181)."""
    w, q, kp, vp, kn, vn = cases.attention_inputs(name)
    s = cases.seam_tensors(w, q, kp, vp, kn, vn)
    pos = torch.from_numpy(w.context_lens.astype(np.int64) - 1)[:, None]   # [B, 1]
    cos, sin = RotaryEmbedding(w.head_dim, theta)(pos)                     # [B, 1, D]
    q_rot, k_rot = apply_rotary_pos_emb(torch.from_numpy(s["q"]), torch.from_numpy(s["k"]),
                                        cos, sin)
    pool = PagedKVPool(1, w.num_blocks, w.block_size, w.num_kv_heads, w.head_dim,
                       torch.float32)
    pool.k.copy_(torch.from_numpy(s["pool_k"]))
    pool.v.copy_(torch.from_numpy(s["pool_v"]))
    ctx = PagedContext(pool, torch.from_numpy(s["write_slots"]),
                       torch.from_numpy(s["gather_slots"]), use_triton=False)
    res = paged_attention(q_rot, k_rot, torch.from_numpy(s["v"]), ctx,
                          torch.from_numpy(s["mask"]), 0, w.scale, w.n_rep)
    out[f"rope/{name}/cos"] = cos.numpy()[:, 0]
    out[f"rope/{name}/sin"] = sin.numpy()[:, 0]
    out[f"rope/{name}/q_rot"] = q_rot.numpy()[:, 0]
    out[f"rope/{name}/k_rot"] = k_rot.numpy()[:, 0]
    out[f"rope/{name}/out"] = res.numpy()[:, 0]


def run_prefill_case(name: str, out: dict) -> None:
    """infrared's prefill (one prompt, cached prefix: build_attention_mask) or
    packed mixed step (build_varlen_mask) through its naive paged path."""
    c = cases.prefill_inputs(name)
    fr = c["frame"]
    pool = PagedKVPool(1, c["num_blocks"], c["bs"], c["hkv"], c["d"], torch.float32)
    pool.k[0].copy_(torch.from_numpy(c["pool_k"]))
    pool.v[0].copy_(torch.from_numpy(c["pool_v"]))
    if len(c["starts"]) == 1:
        mask = build_attention_mask([0], c["starts"][0], c["q_lens"][0],
                                    int(c["context_lens"][0]), torch.float32, "cpu")
    else:
        mask = build_varlen_mask(torch.from_numpy(fr["q_seq_ids"]),
                                 torch.from_numpy(fr["q_pos"]),
                                 torch.from_numpy(fr["k_seq_ids"]),
                                 torch.from_numpy(fr["k_pos"]), torch.float32, "cpu")
    ctx = PagedContext(pool, torch.from_numpy(fr["write_slots"]),
                       torch.from_numpy(fr["gather_slots"]), use_triton=False)
    res = paged_attention(torch.from_numpy(c["q"])[None], torch.from_numpy(c["k"])[None],
                          torch.from_numpy(c["v"])[None], ctx, mask, 0, c["scale"], c["n_rep"])
    out[f"prefill/{name}/out"] = res.numpy()[0]
    out[f"prefill/{name}/mask_digest"] = np.array(cases.digest(mask.numpy()))
    out[f"prefill/{name}/pool_digest"] = np.array(cases.digest(pool.k.numpy(), pool.v.numpy()))


def main() -> None:
    torch.manual_seed(0)
    out: dict = {}
    for name in cases.ATTENTION_CASES:
        run_attention_case(name, out)
    for name in cases.GRAPH_CASES:
        run_graph_case(name, out)
    run_blockwise(out)
    for name, theta in cases.ROPE_CASES.items():
        run_rope_case(name, theta, out)
    for name in cases.PREFILL_CASES:
        run_prefill_case(name, out)
    dst = HERE / "golden.npz"
    np.savez_compressed(dst, **out)
    print(f"wrote {dst} ({dst.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
