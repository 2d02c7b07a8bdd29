"""The K/V projection kernel with bias, RoPE and the pool write in its
epilogue (``ir_kv_proj_rope_write``), and decode with RoPE on q
(``ir_paged_decode_rope``).

Reference: infrared's own computation in PyTorch on the same inputs —
``nn.Linear`` (fp32 accumulation, one rounding to the dtype),
``apply_rotary_pos_emb`` (infrared/model/layers.py:79-89: cos/sin cast to the
dtype, each elementwise op rounded) and ``PagedKVPool.write``. The kernel's
accumulation order differs from the library GEMM's, so the rows agree at the
bf16 bar (atol = rtol = 2e-2), not bit for bit; every pool row the call does
not name stays untouched (bit-exact).
"""

import pytest
import torch

import infrared_b200 as irb
from gpu_helpers import DEV, assert_close_bf16, dev_meta, host_f32, oracle_decode_device
from infrared_b200 import ops
from infrared_b200 import workloads as wl

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


@pytest.fixture(autouse=True)
def _clean_errors():
    ops.error_flag().zero_()
    yield
    ops.check_device_errors()


def _rope_tables(positions, d, theta=1e6):
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, device=DEV, dtype=torch.float32) / d))
    f = positions.to(torch.float32)[:, None] * inv
    emb = torch.cat((f, f), dim=-1)
    return emb.cos(), emb.sin()


def _rope_ref(k, cos, sin):
    """apply_rotary_pos_emb on k [N, Hkv, D] (infrared/model/layers.py:79-89)."""
    c = cos[:, None, :].to(k.dtype)
    s = sin[:, None, :].to(k.dtype)
    half = k.shape[-1] // 2
    rot = torch.cat((-k[..., half:], k[..., :half]), dim=-1)
    return k * c + rot * s


def _case(n, hidden, hkv, d, dtype, bias=True, seed=0, num_slots=4096):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    x = torch.randn(n, hidden, generator=g, device=DEV).to(dtype)
    wk = (torch.randn(hkv * d, hidden, generator=g, device=DEV) * 0.02).to(dtype)
    wv = (torch.randn(hkv * d, hidden, generator=g, device=DEV) * 0.02).to(dtype)
    bk = (torch.randn(hkv * d, generator=g, device=DEV) * 0.1).to(dtype) if bias else None
    bv = (torch.randn(hkv * d, generator=g, device=DEV) * 0.1).to(dtype) if bias else None
    pos = torch.randint(0, 4000, (n,), generator=g, device=DEV)
    cos, sin = _rope_tables(pos, d)
    slots = torch.randperm(num_slots, generator=g, device=DEV)[:n].contiguous()
    kp = torch.randn(num_slots, hkv, d, generator=g, device=DEV).to(dtype)
    vp = torch.randn(num_slots, hkv, d, generator=g, device=DEV).to(dtype)
    return x, wk, wv, bk, bv, cos, sin, slots, kp, vp


def _reference(x, wk, wv, bk, bv, cos, sin, hkv, d, rope=True):
    k = x.float() @ wk.float().T
    v = x.float() @ wv.float().T
    if bk is not None:
        k, v = k + bk.float(), v + bv.float()
    k = k.to(x.dtype).view(-1, hkv, d)
    v = v.to(x.dtype).view(-1, hkv, d)
    if rope:
        k = _rope_ref(k, cos, sin)
    return k, v


@pytest.mark.parametrize("n,hidden,hkv,d,dtype,bias", [
    (128, 3584, 4, 128, torch.bfloat16, True),    # Qwen2.5-7B, a full token tile
    (1, 3584, 4, 128, torch.bfloat16, True),      # one token
    (37, 3584, 4, 128, torch.bfloat16, False),    # ragged tile, no bias
    (200, 3584, 4, 128, torch.float16, True),     # two token tiles, fp16
    (64, 896, 2, 64, torch.bfloat16, True),       # Qwen2.5-0.5B geometry
    (9, 448, 2, 64, torch.float16, True),         # 7 hidden chunks over 8 split CTAs
])
def test_projection_rope_write_matches_infrared_math(n, hidden, hkv, d, dtype, bias):
    x, wk, wv, bk, bv, cos, sin, slots, kp, vp = _case(n, hidden, hkv, d, dtype, bias)
    before_k, before_v = kp.clone(), vp.clone()
    irb.kv_proj_rope_write(x, wk, wv, bk, bv, cos, sin, slots, kp, vp)
    torch.cuda.synchronize()
    k_ref, v_ref = _reference(x, wk, wv, bk, bv, cos, sin, hkv, d)
    assert_close_bf16(host_f32(kp[slots]), host_f32(k_ref))
    assert_close_bf16(host_f32(vp[slots]), host_f32(v_ref))
    other = torch.ones(kp.shape[0], dtype=torch.bool, device=DEV)
    other[slots] = False
    assert torch.equal(kp[other], before_k[other]) and torch.equal(vp[other], before_v[other])


def test_projection_without_rope():
    x, wk, wv, bk, bv, cos, sin, slots, kp, vp = _case(50, 3584, 4, 128, torch.bfloat16)
    irb.kv_proj_rope_write(x, wk, wv, bk, bv, None, None, slots, kp, vp)
    torch.cuda.synchronize()
    k_ref, v_ref = _reference(x, wk, wv, bk, bv, cos, sin, 4, 128, rope=False)
    assert_close_bf16(host_f32(kp[slots]), host_f32(k_ref))
    assert_close_bf16(host_f32(vp[slots]), host_f32(v_ref))


def test_projection_is_deterministic_and_graph_capturable():
    x, wk, wv, bk, bv, cos, sin, slots, kp, vp = _case(128, 3584, 4, 128, torch.bfloat16)
    irb.kv_proj_rope_write(x, wk, wv, bk, bv, cos, sin, slots, kp, vp)
    torch.cuda.synchronize()
    first_k, first_v = kp[slots].clone(), vp[slots].clone()
    s = torch.cuda.Stream(DEV)
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            irb.kv_proj_rope_write(x, wk, wv, bk, bv, cos, sin, slots, kp, vp)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        kp[slots] = 0
        vp[slots] = 0
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(kp[slots], first_k) and torch.equal(vp[slots], first_v)
    del g


def test_out_of_range_slot_is_flagged_not_written():
    x, wk, wv, bk, bv, cos, sin, slots, kp, vp = _case(8, 3584, 4, 128, torch.bfloat16)
    slots[3] = kp.shape[0] + 5
    before = kp.clone()
    irb.kv_proj_rope_write(x, wk, wv, bk, bv, cos, sin, slots, kp, vp)
    torch.cuda.synchronize()
    with pytest.raises(irb.DeviceError, match="SLOT"):
        ops.check_device_errors()
    good = torch.cat([slots[:3], slots[4:]])
    k_ref, _ = _reference(x, wk, wv, bk, bv, cos, sin, 4, 128)
    assert_close_bf16(host_f32(kp[good]), host_f32(torch.cat([k_ref[:3], k_ref[4:]])))
    untouched = torch.ones(kp.shape[0], dtype=torch.bool, device=DEV)
    untouched[good] = False
    assert torch.equal(kp[untouched], before[untouched])


def test_projection_then_decode_with_rope_on_q():
    """A decode step with the new tokens written by the projection kernel and
    q rotated inside the decode kernel, against the fp32 oracle over the pool
    the reference computation writes."""
    w = wl.custom(5, 24, 28, 4, 128, 16, 100, 2000, "bfloat16", std=0.5)
    q, kp, vp, _, _ = wl.torch_values(w, 6, DEV)
    bt, ctx, sm = dev_meta(w)
    hidden = 3584
    g = torch.Generator(device=DEV)
    g.manual_seed(9)
    x = torch.randn(w.batch, hidden, generator=g, device=DEV).to(torch.bfloat16)
    wk = (torch.randn(512, hidden, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    wv = (torch.randn(512, hidden, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    pos = (ctx - 1).long()
    cos, sin = _rope_tables(pos, 128)
    irb.kv_proj_rope_write(x, wk, wv, None, None, cos, sin, sm, kp, vp)
    out = irb.paged_decode_rope(q, kp, vp, bt, ctx, cos, sin, w.scale, w.block_size)
    torch.cuda.synchronize()
    q_rot = _rope_ref(q, cos, sin)
    assert_close_bf16(host_f32(out), oracle_decode_device(w, q_rot, kp, vp))
    # the same as rotating q with torch and calling the plain decode
    plain = irb.paged_decode(q_rot, kp, vp, bt, ctx, w.scale, w.block_size)
    torch.cuda.synchronize()
    assert torch.equal(out, plain)
