"""The shim that installs the B200 kernels behind infrared's own seam.

CPU part: with infrared importable (``tests/infrared_ref.py``: INFRARED_REF or
the repository's ``baseline/_ref`` install; skipped elsewhere), installing the shim leaves every CPU
call on infrared's naive path, bit for bit, and uninstalling restores the
original functions. GPU part: the same shim installed into a stand-in seam
with infrared's call contract (a dispatcher that writes through
``pool.write`` and then asks ``_should_use_triton`` whether to call
``_paged_attention_triton``), checked against the oracle.
"""

import types

import numpy as np
import pytest
import torch

import infrared_ref
from infrared_b200 import shim
from infrared_b200 import workloads as wl
from oracle import paged_attention_np as orc

@pytest.fixture
def infrared():
    if not infrared_ref.importable():
        pytest.skip("infrared (the reference) is not installed")
    import infrared.cache.paged_kv_cache as pk
    import infrared.engine.cuda_graph as cg
    import infrared.model.triton_attention as ta

    return ta, pk, cg


def test_install_uninstall_restores(infrared):
    ta, pk, cg = infrared
    before = (ta._should_use_triton, ta._paged_attention_triton, pk.PagedKVPool.write,
              cg.build_decode_static_inputs)
    h = shim.install(ta, pk, cg)
    assert ta._should_use_triton is shim.should_use_b200
    assert ta._paged_attention_triton is shim.paged_attention_b200
    assert pk.PagedKVPool.write is not before[2]
    assert cg.build_decode_static_inputs is not before[3]
    h.uninstall()
    assert (ta._should_use_triton, ta._paged_attention_triton, pk.PagedKVPool.write,
            cg.build_decode_static_inputs) == before


def test_cpu_graph_inputs_stay_on_reference_path(infrared):
    ta, pk, cg = infrared
    args = ([[0, 1], [2]], [5, 2], [7, 9], 4, 16, 4, "cpu", torch.float32)
    ref = cg.build_decode_static_inputs(*args)
    h = shim.install(ta, pk, cg)
    try:
        got = cg.build_decode_static_inputs(*args)
    finally:
        h.uninstall()
    for f in ("ids", "positions", "write_slots", "gather_slots", "mask"):
        assert torch.equal(getattr(got, f), getattr(ref, f))


def test_cpu_calls_stay_on_reference_path(infrared):
    """With the shim installed, infrared's CPU decode gives its own result."""
    ta, pk, cg = infrared
    w = wl.custom(3, 4, 14, 2, 64, 16, 5, 90, "float32")
    q, kp, vp, kn, vn = wl.numpy_values(w, 2)
    t = int(w.context_lens.max())
    gs = torch.from_numpy(orc.gather_slots_from_tables(w.block_tables, w.context_lens, 16, t))
    mask = torch.from_numpy(orc.decode_mask(w.context_lens, t))

    def run():
        pool = pk.PagedKVPool(1, w.num_blocks, 16, 2, 64, torch.float32)
        pool.k[0].copy_(torch.from_numpy(kp))
        pool.v[0].copy_(torch.from_numpy(vp))
        ctx = pk.PagedContext(pool, torch.from_numpy(w.slot_mapping), gs, use_triton=True)
        out = ta.paged_attention(torch.from_numpy(q)[:, None], torch.from_numpy(kn)[:, None],
                                 torch.from_numpy(vn)[:, None], ctx, mask, 0, w.scale, w.n_rep)
        return out, pool

    ref_out, ref_pool = run()
    h = shim.install(ta, pk, cg)
    try:
        out, pool = run()
    finally:
        h.uninstall()
    assert torch.equal(out, ref_out)
    assert torch.equal(pool.k, ref_pool.k) and torch.equal(pool.v, ref_pool.v)


def test_gate_rejects_cpu_prefill_and_opt_out():
    q = torch.zeros(2, 1, 28, 128)
    assert not shim.should_use_b200(q, True)                          # CPU
    assert not shim.should_use_b200(torch.zeros(1, 3, 28, 128), True)  # Sq > 1


# ---------------------------------------------------------------- GPU, stand-in seam


def _stand_in_seam():
    """Modules with infrared's seam contract (names and call order), written here."""
    pk = types.ModuleType("stand_in_paged_kv_cache")

    class PagedKVPool:
        def __init__(self, layers, blocks, bs, hkv, d, dtype, device):
            self.block_size = bs
            self.k = torch.zeros(layers, blocks * bs, hkv, d, dtype=dtype, device=device)
            self.v = torch.zeros_like(self.k)

        def write(self, layer_idx, k, v, slots):
            self.k[layer_idx, slots] = k
            self.v[layer_idx, slots] = v

    pk.PagedKVPool = PagedKVPool
    ta = types.ModuleType("stand_in_triton_attention")
    calls = {"b200": 0, "naive": 0}

    def _should_use_triton(q, want):
        return False

    def _paged_attention_triton(q, paged, mask, layer_idx, scale, n_rep):
        raise AssertionError("not installed")

    def _naive(q, paged, mask, layer_idx, scale, n_rep):
        calls["naive"] += 1
        kk = paged.pool.k[layer_idx][paged.gather_slots].float()
        vv = paged.pool.v[layer_idx][paged.gather_slots].float()
        kk = kk.repeat_interleave(n_rep, dim=2)
        vv = vv.repeat_interleave(n_rep, dim=2)
        s = torch.einsum("bqhd,bkhd->bhqk", q.float(), kk) * scale + mask.float()
        return torch.einsum("bhqk,bkhd->bqhd", s.softmax(-1), vv).to(q.dtype)

    def paged_attention(q, k, v, paged, mask, layer_idx, scale, n_rep):
        h, d = k.shape[-2], k.shape[-1]
        paged.pool.write(layer_idx, k.reshape(-1, h, d), v.reshape(-1, h, d), paged.write_slots)
        if ta._should_use_triton(q, paged.use_triton):
            calls["b200"] += 1
            return ta._paged_attention_triton(q, paged, mask, layer_idx, scale, n_rep)
        return _naive(q, paged, mask, layer_idx, scale, n_rep)

    ta._should_use_triton = _should_use_triton
    ta._paged_attention_triton = _paged_attention_triton
    ta.paged_attention = paged_attention
    return ta, pk, calls


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_shim_routes_decode_to_b200(dtype):
    from infrared_b200 import PagedContext, check_device_errors

    ta, pk, calls = _stand_in_seam()
    h = shim.install(ta, pk, graph_inputs=False)
    try:
        w = wl.custom(9, 6, 28, 4, 128, 16, 10, 400, "float32", shared_frac=0.3)
        q, kp, vp, kn, vn = [torch.from_numpy(x).cuda().to(dtype) for x in wl.numpy_values(w, 4)]
        pool = pk.PagedKVPool(2, w.num_blocks, 16, 4, 128, dtype, "cuda")
        pool.k[1].copy_(kp)
        pool.v[1].copy_(vp)
        t = int(w.context_lens.max())
        gs = torch.from_numpy(orc.gather_slots_from_tables(w.block_tables, w.context_lens, 16,
                                                           t)).cuda()
        mask = torch.from_numpy(orc.decode_mask(w.context_lens, t)).cuda().to(dtype)
        ctx = PagedContext(pool, torch.from_numpy(w.slot_mapping).cuda(), gs, use_triton=True)
        out = ta.paged_attention(q[:, None], kn[:, None], vn[:, None], ctx, mask, 1, w.scale,
                                 w.n_rep)
        assert calls["b200"] == 1 and calls["naive"] == 0
        assert torch.equal(pool.k[1][ctx.write_slots], kn)   # written by ir_cache_write
        host = [x.float().cpu().numpy() for x in (q, kp, vp, kn, vn)]
        kp2, vp2 = host[1][None].copy(), host[2][None].copy()
        orc.pool_write(kp2, vp2, 0, host[3], host[4], w.slot_mapping)
        want = orc.decode_from_tables(host[0], kp2, vp2, 0, w.block_tables, w.context_lens, 16,
                                      w.scale, w.n_rep)
        tol = 1e-5 if dtype == torch.float32 else 2e-2
        np.testing.assert_allclose(out[:, 0].float().cpu().numpy(), want, atol=tol,
                                   rtol=0 if dtype == torch.float32 else tol)
        # a prefill call (Sq = 2) stays on the seam's own path
        q2 = q[:1, None].expand(-1, 2, -1, -1).contiguous()
        k2 = kn[:1, None].expand(-1, 2, -1, -1).contiguous()
        slots2 = torch.tensor([0, 1], device="cuda")
        mask2 = torch.zeros(1, 1, 2, 2, device="cuda", dtype=dtype)
        mask2[0, 0, 0, 1] = torch.finfo(dtype).min
        ta.paged_attention(q2, k2, k2, PagedContext(pool, slots2, slots2[None], use_triton=True),
                           mask2, 1, w.scale, w.n_rep)
        assert calls["b200"] == 1 and calls["naive"] == 1
        check_device_errors()
    finally:
        h.uninstall()


# ---------------------------------------------------------------- RoPE-fused forward


@pytest.fixture
def infrared_layers(infrared):
    import infrared.model.layers as ly

    return ly


def test_fuse_rope_install_and_cpu_fallback(infrared, infrared_layers):
    """install(fuse_rope=True) swaps Attention.forward; a CPU paged decode call
    still runs infrared's own forward bit for bit; uninstall restores it."""
    from infrared.model.config import Qwen2Config

    ta, pk, cg = infrared
    ly = infrared_layers
    cfg = Qwen2Config(vocab_size=64, hidden_size=128, intermediate_size=256,
                      num_hidden_layers=1, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=32, rms_norm_eps=1e-6, rope_theta=1e6,
                      max_position_embeddings=512, tie_word_embeddings=False,
                      bos_token_id=0)
    torch.manual_seed(0)
    attn = ly.Attention(cfg)
    w = wl.custom(4, 3, 4, 2, 32, 16, 3, 40, "float32")
    kp, vp = wl.numpy_values(w, 1)[1:3]
    t = int(w.context_lens.max())
    gs = torch.from_numpy(orc.gather_slots_from_tables(w.block_tables, w.context_lens, 16, t))
    mask = torch.from_numpy(orc.decode_mask(w.context_lens, t))
    cos, sin = ly.RotaryEmbedding(32, 1e6)(torch.from_numpy(w.context_lens - 1)[:, None])
    x = torch.randn(3, 1, 128)

    def run():
        pool = pk.PagedKVPool(1, w.num_blocks, 16, 2, 32, torch.float32)
        pool.k[0].copy_(torch.from_numpy(kp))
        pool.v[0].copy_(torch.from_numpy(vp))
        paged = pk.PagedContext(pool, torch.from_numpy(w.slot_mapping), gs, use_triton=True)
        ctx = ly.ForwardContext(cos=cos, sin=sin, mask=mask, kv_cache=None, start_col=0,
                                paged=paged)
        with torch.no_grad():
            return attn(x, ctx, 0), pool

    before = ly.Attention.forward
    ref, ref_pool = run()
    h = shim.install(ta, pk, cg, layers=ly, fuse_rope=True)
    try:
        assert ly.Attention.forward is not before
        out, pool = run()
    finally:
        h.uninstall()
    assert ly.Attention.forward is before
    assert torch.equal(out, ref)
    assert torch.equal(pool.k, ref_pool.k) and torch.equal(pool.v, ref_pool.v)


def _stand_in_layers(ta):
    """A module with infrared's Attention contract (layers.py:142-182), written here."""
    ly = types.ModuleType("stand_in_layers")

    class Attention(torch.nn.Module):
        def __init__(self, hidden, nh, nkv, d, dtype, device):
            super().__init__()
            self.num_heads, self.num_kv_heads, self.head_dim = nh, nkv, d
            self.n_rep = nh // nkv
            self.scale = d ** -0.5
            kw = dict(dtype=dtype, device=device)
            self.q_proj = torch.nn.Linear(hidden, nh * d, bias=True, **kw)
            self.k_proj = torch.nn.Linear(hidden, nkv * d, bias=True, **kw)
            self.v_proj = torch.nn.Linear(hidden, nkv * d, bias=True, **kw)
            self.o_proj = torch.nn.Linear(nh * d, hidden, bias=False, **kw)

        def forward(self, x, ctx, layer_idx):
            b, seq, _ = x.shape
            q = self.q_proj(x).view(b, seq, self.num_heads, self.head_dim)
            k = self.k_proj(x).view(b, seq, self.num_kv_heads, self.head_dim)
            v = self.v_proj(x).view(b, seq, self.num_kv_heads, self.head_dim)
            cos = ctx.cos.unsqueeze(2).to(q.dtype)
            sin = ctx.sin.unsqueeze(2).to(q.dtype)
            half = self.head_dim // 2

            def rot(t):
                return torch.cat((-t[..., half:], t[..., :half]), dim=-1)

            q, k = q * cos + rot(q) * sin, k * cos + rot(k) * sin
            out = ta.paged_attention(q, k, v, ctx.paged, ctx.mask, layer_idx, self.scale,
                                     self.n_rep)
            return self.o_proj(out.reshape(b, seq, self.num_heads * self.head_dim))

    ly.Attention = Attention
    return ly


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_rope_forward_equals_installed_seam(dtype):
    """Attention.forward with RoPE in the kernel == the same layer through the
    installed seam (PyTorch RoPE, ir_cache_write, ir_paged_decode), bit for bit."""
    from infrared_b200 import PagedContext, check_device_errors

    ta, pk, calls = _stand_in_seam()
    ly = _stand_in_layers(ta)
    torch.manual_seed(1)
    attn = ly.Attention(512, 28, 4, 128, dtype, "cuda")
    w = wl.custom(19, 9, 28, 4, 128, 16, 1, 600, "float32", shared_frac=0.3)
    kp, vp = [torch.from_numpy(a).cuda().to(dtype) for a in wl.numpy_values(w, 2)[1:3]]
    t = int(w.context_lens.max())
    gs = torch.from_numpy(orc.gather_slots_from_tables(w.block_tables, w.context_lens, 16,
                                                       t)).cuda()
    mask = torch.from_numpy(orc.decode_mask(w.context_lens, t)).cuda().to(dtype)
    cos_np, sin_np = orc.rope_tables((w.context_lens - 1)[:, None], 128, 1e6)
    cos, sin = torch.from_numpy(cos_np).cuda(), torch.from_numpy(sin_np).cuda()   # [B,1,D]
    x = torch.randn(w.batch, 1, 512, device="cuda").to(dtype)

    def run(fuse):
        pool = pk.PagedKVPool(2, w.num_blocks, 16, 4, 128, dtype, "cuda")
        pool.k[1].copy_(kp)
        pool.v[1].copy_(vp)
        paged = PagedContext(pool, torch.from_numpy(w.slot_mapping).cuda(), gs,
                             use_triton=True)
        ctx = types.SimpleNamespace(cos=cos, sin=sin, mask=mask, paged=paged)
        h = shim.install(ta, pk, graph_inputs=False, layers=ly, fuse_rope=fuse)
        try:
            with torch.no_grad():
                return attn(x, ctx, 1), pool
        finally:
            h.uninstall()

    ref, ref_pool = run(False)
    assert calls["b200"] == 1
    out, pool = run(True)
    assert calls["b200"] == 1          # the fused forward never reached the seam
    assert torch.equal(out, ref)
    assert torch.equal(pool.k, ref_pool.k) and torch.equal(pool.v, ref_pool.v)
    check_device_errors()



@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_shim_routes_prefill_frames_when_enabled():
    """install(prefill=True): a packed Sq > 1 frame goes to the tensor-core
    prefill; without it, the seam's own path runs."""
    import cases
    from infrared_b200 import PagedContext, check_device_errors
    from infrared_b200.attention import clear_metadata_cache

    c = cases.prefill_inputs("varlen_g7")
    fr = c["frame"]
    dtype = torch.bfloat16
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    mask = t(orc.varlen_mask(fr["q_seq_ids"], fr["q_pos"], fr["k_seq_ids"],
                             fr["k_pos"])).to(dtype)
    q, k, v = (t(c[n]).to(dtype)[None] for n in ("q", "k", "v"))
    outs = {}
    for prefill in (True, False):
        ta, pk, calls = _stand_in_seam()
        h = shim.install(ta, pk, graph_inputs=False, prefill=prefill)
        try:
            pool = pk.PagedKVPool(1, c["num_blocks"], c["bs"], c["hkv"], c["d"], dtype, "cuda")
            pool.k[0].copy_(t(c["pool_k"]).to(dtype))
            pool.v[0].copy_(t(c["pool_v"]).to(dtype))
            paged = PagedContext(pool, t(fr["write_slots"]), t(fr["gather_slots"]),
                                 use_triton=True)
            clear_metadata_cache()
            outs[prefill] = ta.paged_attention(q, k, v, paged, mask, 0, c["scale"], c["n_rep"])
            assert calls["b200"] == (1 if prefill else 0)
            assert calls["naive"] == (0 if prefill else 1)
        finally:
            h.uninstall()
    check_device_errors()
    diff = (outs[True].float() - outs[False].float()).abs().max().item()
    assert diff < 2e-2


# ---------------------------------------------------------------- eager decode inputs


class _Rec:
    """A stand-in engine with the attributes _decode_logits_eager reads; its
    model records the forward's inputs."""

    def __init__(self, device, dtype, bs):
        import types as _t

        self.block_size = bs
        self.enable_triton_attention = True
        self.pool = object()
        self.calls = []

        def forward(ids, positions, mask, paged):
            self.calls.append((ids, positions, mask, paged))
            return torch.zeros(ids.shape[0], 1, 7, device=ids.device)

        self.model = _t.SimpleNamespace(device=device, dtype=dtype, forward=forward)


def _running(rng, n, bs, num_blocks):
    import types as _t

    perm = list(rng.permutation(num_blocks))
    seqs = []
    for _ in range(n):
        nc = int(rng.integers(0, 90))
        seqs.append(_t.SimpleNamespace(num_cached_tokens=nc, last_token=int(rng.integers(0, 999)),
                                       block_table=[int(perm.pop()) for _ in range(nc // bs + 1)]))
    return seqs


def test_eager_inputs_cpu_falls_through(infrared):
    ta, pk, cg = infrared
    import infrared.engine.paged_engine as pe

    sentinel = object()
    h = shim.install(ta, pk, cg, paged_engine=pe, eager_inputs=True)
    try:
        eng = _Rec("cpu", torch.float32, 4)
        calls = []
        orig = h.saved["eager"]
        h.saved["eager"] = lambda self, running: calls.append(running) or sentinel
        # rebuild the replacement around the stub to see the fall-through
        fn = shim._make_decode_logits_eager(h.saved["eager"], pk.PagedContext)
        assert fn(eng, [1, 2]) is sentinel and calls == [[1, 2]]
        h.saved["eager"] = orig
    finally:
        h.uninstall()


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_eager_inputs_built_on_device(dtype):
    """The eager decode step's forward inputs, built by ir_build_decode_inputs,
    equal infrared's per-sequence construction (restated in the oracle)."""
    from infrared_b200 import PagedContext

    rng = np.random.default_rng(5)
    bs = 8
    running = _running(rng, 6, bs, 128)
    eng = _Rec(torch.device("cuda"), dtype, bs)
    fn = shim._make_decode_logits_eager(lambda *a: pytest.fail("fell through"), PagedContext)
    out = fn(eng, running)
    assert out.shape == (6, 7)
    ids, positions, mask, paged = eng.calls[0]
    ctx = [s.num_cached_tokens + 1 for s in running]
    want = orc.build_decode_inputs([s.block_table for s in running],
                                   [s.num_cached_tokens for s in running],
                                   [s.last_token for s in running], len(running), max(ctx), bs)
    np.testing.assert_array_equal(ids.cpu().numpy(), want["ids"])
    np.testing.assert_array_equal(positions.cpu().numpy(), want["positions"])
    np.testing.assert_array_equal(paged.write_slots.cpu().numpy(), want["write_slots"])
    np.testing.assert_array_equal(paged.gather_slots.cpu().numpy(), want["gather_slots"])
    m = mask.float().cpu().numpy()
    blocked = want["mask"] != 0
    assert (m[~blocked] == 0).all()
    assert (m[blocked] == float(torch.finfo(dtype).min)).all()
    assert paged.use_triton
