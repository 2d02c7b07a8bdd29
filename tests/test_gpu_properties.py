"""Size-independent properties of the kernels at the benchmark sizes.

The oracle is too slow for full C2 frames on every row, so these check
relations the reference's attention satisfies exactly: outputs do not depend
on where blocks sit in the pool (bit for bit: the work partition depends only
on context lengths), attention is linear in V (within bf16 rounding), and a
decode row equals the last row of a prefill of the same history.
"""

import numpy as np
import pytest
import torch

from gpu_helpers import DEV
import infrared_b200 as irb
from infrared_b200 import ops
from infrared_b200 import workloads as wl

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


@pytest.fixture(autouse=True)
def _clean_errors():
    ops.error_flag().zero_()
    yield
    ops.check_device_errors()


def _c2():
    w = wl.c2(seed=3)
    q, kp, vp, _, _ = wl.torch_values(w, 11, DEV)
    bt = torch.from_numpy(w.block_tables).to(DEV)
    ctx = torch.from_numpy(w.context_lens).to(DEV)
    return w, q, kp, vp, bt, ctx


def test_c2_block_placement_does_not_change_outputs():
    """Move every block to another physical id (data moved with it): the
    decode output is bit-identical."""
    w, q, kp, vp, bt, ctx = _c2()
    want = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size)
    nb = w.num_blocks
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(5)).to(DEV)
    bs = w.block_size
    # new block perm[i] holds old block i
    kp2 = torch.empty_like(kp).view(nb, bs, *kp.shape[1:])
    vp2 = torch.empty_like(vp).view(nb, bs, *vp.shape[1:])
    kp2[perm] = kp.view(nb, bs, *kp.shape[1:])
    vp2[perm] = vp.view(nb, bs, *vp.shape[1:])
    bt2 = perm.to(torch.int32)[bt.long()]
    got = irb.paged_decode(q, kp2.view_as(kp), vp2.view_as(vp), bt2, ctx, w.scale, bs)
    assert torch.equal(got, want)


def test_c2_linear_in_values():
    """attn(V1 + V2) == attn(V1) + attn(V2) up to bf16 rounding (fp32 pools
    would make it exact; here V1 and V2 are bf16 and so is their sum)."""
    w, q, kp, vp, bt, ctx = _c2()
    g = torch.Generator(device=DEV)
    g.manual_seed(9)
    v2 = (torch.randn(vp.shape, generator=g, device=DEV) * 0.5).to(vp.dtype)
    a = irb.paged_decode(q, kp, vp, bt, ctx, w.scale, w.block_size).float()
    b = irb.paged_decode(q, kp, v2, bt, ctx, w.scale, w.block_size).float()
    c = irb.paged_decode(q, kp, (vp.float() + v2.float()).to(vp.dtype), bt, ctx, w.scale,
                         w.block_size).float()
    torch.testing.assert_close(c, a + b, atol=3e-2, rtol=3e-2)


def test_decode_equals_last_prefill_row():
    """For every sequence of a C2-sized frame, decoding its last position
    equals the last row of a causal prefill of its whole history."""
    w, q, kp, vp, bt, ctx = _c2()
    b = 12
    qq = q[:b]
    dec = irb.paged_decode(qq, kp, vp, bt[:b], ctx[:b], w.scale, w.block_size)
    q_start = torch.arange(b + 1, dtype=torch.int32, device=DEV)   # one row per sequence
    pre = irb.paged_prefill(qq.contiguous(), kp, vp, bt[:b].contiguous(), ctx[:b], q_start,
                            w.scale, w.block_size)
    torch.testing.assert_close(pre.float(), dec.float(), atol=2e-2, rtol=2e-2)
    # and the whole-history prefill's last row, for a few sequences
    for i in (0, 5, 11):
        c = int(w.context_lens[i])
        g = torch.Generator(device=DEV)
        g.manual_seed(100 + i)
        qrows = (torch.randn(c, w.num_heads, w.head_dim, generator=g, device=DEV) * 0.5).to(q.dtype)
        qrows[-1] = q[i]
        out = irb.paged_prefill(qrows, kp, vp, bt[i:i + 1].contiguous(), ctx[i:i + 1],
                                torch.tensor([0, c], dtype=torch.int32, device=DEV), w.scale,
                                w.block_size)
        torch.testing.assert_close(out[-1].float(), dec[i].float(), atol=2e-2, rtol=2e-2)
    assert np.isfinite(dec.float().cpu().numpy()).all()
