"""The Qwen2 decode-step harness (workload C5) on the fused write + decode
kernel against the same step with plain-PyTorch attention."""

import pytest
import torch

from infrared_b200 import model_step as ms
from infrared_b200 import ops

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


class _Checked(ms.Qwen2DecodeStep):
    """Runs the kernel, then the fp32 reference on the same pool, per layer."""

    fuse_rope = False

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        self.worst = 0.0

    def attention(self, layer, q, k, v, slots, ctx):
        out = super().attention(layer, q, k, v, slots, ctx)
        ref = self.reference_attention(layer, q, k, v, slots, ctx)
        torch.testing.assert_close(out.float(), ref.float(), atol=2e-2, rtol=2e-2)
        self.worst = max(self.worst, (out.float() - ref.float()).abs().max().item())
        return out


class _Reference(ms.Qwen2DecodeStep):
    fuse_rope = False

    def attention(self, layer, q, k, v, slots, ctx):
        return self.reference_attention(layer, q, k, v, slots, ctx)


def _ctx():
    return ms.random_context_lens(6, 1, 90, seed=3).tolist() + [16, 17]


def test_step_attention_matches_reference_per_layer():
    m = _Checked(ms.tiny_geometry(), _ctx(), max_new=4, device="cuda", seed=1)
    for _ in range(3):
        m.step()
    torch.cuda.synchronize()
    ops.check_device_errors()
    assert m.worst < 2e-2


def test_step_logits_and_cache_match_reference_model():
    ours = ms.Qwen2DecodeStep(ms.tiny_geometry(), _ctx(), max_new=4, device="cuda", seed=2)
    ref = _Reference(ms.tiny_geometry(), _ctx(), max_new=4, device="cuda", seed=2)
    assert torch.equal(ours.k_pool, ref.k_pool)
    lo = ours.step()
    lr = ref.step()
    ops.check_device_errors()
    torch.testing.assert_close(lo.float(), lr.float(), atol=2e-2, rtol=2e-2)
    # the layer-0 K/V of the new token precede any attention: written bit-exactly
    assert torch.equal(ours.k_pool[0], ref.k_pool[0])
    assert torch.equal(ours.v_pool[0], ref.v_pool[0])
    assert torch.equal(ours.positions, ref.positions)


def test_step_replays_in_a_cuda_graph():
    ctx = _ctx()
    eager = ms.Qwen2DecodeStep(ms.tiny_geometry(), ctx, max_new=6, device="cuda", seed=4)
    graphed = ms.Qwen2DecodeStep(ms.tiny_geometry(), ctx, max_new=6, device="cuda", seed=4)
    eager.step()
    graphed.step()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            logits = graphed.step()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        want = eager.step()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(logits, want)
        assert torch.equal(graphed.ids, eager.ids)
    assert torch.equal(graphed.positions, eager.positions)
    assert torch.equal(graphed.k_pool, eager.k_pool)
    ops.check_device_errors()


class _Unfused(ms.Qwen2DecodeStep):
    fuse_rope = False


def test_fused_rope_step_equals_torch_rope_step():
    """RoPE inside the kernel == PyTorch RoPE + the write/decode kernel, bit for bit."""
    ctx = _ctx()
    fused = ms.Qwen2DecodeStep(ms.tiny_geometry(), ctx, max_new=4, device="cuda", seed=5)
    plain = _Unfused(ms.tiny_geometry(), ctx, max_new=4, device="cuda", seed=5)
    for _ in range(3):
        assert torch.equal(fused.step(), plain.step())
    assert torch.equal(fused.k_pool, plain.k_pool)
    assert torch.equal(fused.v_pool, plain.v_pool)
    ops.check_device_errors()
