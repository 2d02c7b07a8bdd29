"""RoPE fused into the write + decode kernel (ir_paged_decode_rope_write).

Bars: fp32 against the reference's own rotated q/k and outputs (golden
fixtures: pool rows bit-exact, output max-abs <= 1e-5); bf16 / fp16
bit-exact against infrared's apply_rotary_pos_emb evaluated by PyTorch on
the device followed by the un-fused kernel (same rounded q and K, same
accumulation order), on every kernel path.
"""

import numpy as np
import pytest
import torch

import cases
from gpu_helpers import DEV, dev_meta, dev_values, host_f32
import infrared_b200 as irb
from infrared_b200 import ops
from infrared_b200 import workloads as wl
from oracle import paged_attention_np as orc

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


@pytest.fixture(autouse=True)
def _clean_errors():
    ops.set_decode_path(0)
    ops.error_flag().zero_()
    yield
    ops.set_decode_path(0)
    ops.check_device_errors()


def torch_rope(x, cos, sin):
    """infrared/model/layers.py:79-89 on [B, heads, D] with [B, D] fp32 tables."""
    c = cos[:, None, :].to(x.dtype)
    s = sin[:, None, :].to(x.dtype)
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * c + rot * s


@pytest.mark.parametrize("name", sorted(cases.ROPE_CASES))
def test_rope_golden_fp32(golden, name):
    w, *vals = cases.attention_inputs(name)
    q, kp, vp, kn, vn = dev_values(vals, torch.float32)
    bt, ctx, sm = dev_meta(w)
    cos = torch.from_numpy(golden[f"rope/{name}/cos"]).to(DEV)
    sin = torch.from_numpy(golden[f"rope/{name}/sin"]).to(DEV)
    out = irb.paged_decode_rope_write(q, kn, vn, kp, vp, sm, bt, ctx, cos, sin, w.scale,
                                      w.block_size)
    assert np.abs(host_f32(out) - golden[f"rope/{name}/out"]).max() <= 1e-5
    # the pool rows of the new tokens hold the reference's rotated K, bit for bit
    np.testing.assert_array_equal(host_f32(kp[sm]), golden[f"rope/{name}/k_rot"])
    np.testing.assert_array_equal(host_f32(vp[sm]), vals[4])
    # q itself is not modified
    np.testing.assert_array_equal(host_f32(q), vals[0])


ROPE_SHAPES = [
    # (B, H, Hkv, D, bs, ctx_lo, ctx_hi): group 7 (tables ride with q), group 8
    # (no room: tables read from global), D 64, bs 8, group 12 (CUDA cores)
    (9, 28, 4, 128, 16, 1, 700),
    (5, 32, 4, 128, 16, 1, 300),
    (7, 14, 2, 64, 16, 1, 400),
    (6, 16, 8, 128, 8, 1, 200),
    (3, 48, 4, 64, 16, 1, 250),
]


@pytest.mark.parametrize("path", [0, 1, 3])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("cfg", ROPE_SHAPES)
def test_rope_matches_torch_then_unfused_bit_exact(cfg, dtype, path):
    b, h, hkv, d, bs, lo, hi = cfg
    if path == 3 and h // hkv > 8:
        pytest.skip("groups above 8 take the CUDA-core kernel only")
    w = wl.custom(300 + b * h + d, b, h, hkv, d, bs, lo, hi, "bfloat16", shared_frac=0.3)
    vals = wl.numpy_values(w, 9)
    q, kp, vp, kn, vn = dev_values(vals, dtype)
    bt, ctx, sm = dev_meta(w)
    cos_np, sin_np = orc.rope_tables(w.context_lens - 1, d, 1e6)
    cos, sin = torch.from_numpy(cos_np).to(DEV), torch.from_numpy(sin_np).to(DEV)
    kp2, vp2 = kp.clone(), vp.clone()
    ops.set_decode_path(path)
    got = irb.paged_decode_rope_write(q, kn, vn, kp, vp, sm, bt, ctx, cos, sin, w.scale, bs)
    want = irb.paged_decode_write(torch_rope(q, cos, sin), torch_rope(kn, cos, sin), vn,
                                  kp2, vp2, sm, bt, ctx, w.scale, bs)
    assert torch.equal(kp, kp2) and torch.equal(vp, vp2)
    assert torch.equal(got, want)


def test_rope_on_fused_qkv_views():
    """q, k and v as row views of one projection output (the C5 layout)."""
    w = wl.custom(77, 12, 28, 4, 128, 16, 1, 900, "bfloat16")
    vals = wl.numpy_values(w, 3)
    q, kp, vp, kn, vn = dev_values(vals, torch.bfloat16)
    bt, ctx, sm = dev_meta(w)
    qkv = torch.cat([q.reshape(w.batch, -1), kn.reshape(w.batch, -1),
                     vn.reshape(w.batch, -1)], dim=1)
    hd = w.num_heads * w.head_dim
    kvd = w.num_kv_heads * w.head_dim
    qv = qkv[:, :hd].view(w.batch, w.num_heads, w.head_dim)
    kv = qkv[:, hd:hd + kvd].view(w.batch, w.num_kv_heads, w.head_dim)
    vv = qkv[:, hd + kvd:].view(w.batch, w.num_kv_heads, w.head_dim)
    cos_np, sin_np = orc.rope_tables(w.context_lens - 1, w.head_dim, 1e6)
    cos, sin = torch.from_numpy(cos_np).to(DEV), torch.from_numpy(sin_np).to(DEV)
    kp2, vp2 = kp.clone(), vp.clone()
    got = irb.paged_decode_rope_write(qv, kv, vv, kp, vp, sm, bt, ctx, cos, sin, w.scale,
                                      w.block_size)
    want = irb.paged_decode_write(torch_rope(q, cos, sin), torch_rope(kn, cos, sin), vn,
                                  kp2, vp2, sm, bt, ctx, w.scale, w.block_size)
    assert torch.equal(got, want)
    assert torch.equal(kp, kp2) and torch.equal(vp, vp2)


def test_rope_argument_errors():
    w = wl.custom(5, 2, 8, 2, 64, 16, 1, 40, "bfloat16")
    q, kp, vp, kn, vn = dev_values(wl.numpy_values(w, 1), torch.bfloat16)
    bt, ctx, sm = dev_meta(w)
    cos = torch.zeros(w.batch, 64, device=DEV)
    with pytest.raises(ValueError, match="fp32"):
        irb.paged_decode_rope_write(q, kn, vn, kp, vp, sm, bt, ctx, cos.bfloat16(), cos,
                                    w.scale, 16)
    with pytest.raises(ValueError, match="fp32"):
        irb.paged_decode_rope_write(q, kn, vn, kp, vp, sm, bt, ctx, cos[:, :32], cos,
                                    w.scale, 16)
