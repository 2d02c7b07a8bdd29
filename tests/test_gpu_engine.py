"""infrared's own engine on the GPU with the B200 kernels installed behind its
seam (``shim.install``), against infrared's own paths.

These tests drive the reference's ``PagedBatchEngine`` unchanged — its
scheduler, block manager, prefix cache, preemption, eager decode
(infrared/engine/paged_engine.py:248-332), CUDA-graph decode
(infrared/engine/cuda_graph.py:202-287) and chunked mixed prefill
(paged_engine.py:461-551) — so that every attention call of a real engine
run goes through the installed seam. infrared comes from the repository's
``baseline/_ref`` install (``tests/infrared_ref.py``); without it the tests
skip.

Checks (the reference's own end-to-end gates, with the kernels in place):

* fp32, head_dim 64: greedy tokens equal infrared's T0 oracle
  (``infrared.model.generate``) token for token — eager, with CUDA graphs,
  under recompute preemption, with chunked (mixed) prefill, and with each
  shim option (RoPE fused into the decode kernel, decode inputs built on the
  device, prefill on the B200 kernels); the mirror of
  tests/test_paged_kv.py:126-148 and tests/test_cuda_graph.py:261-288 of
  infrared.
* bf16 at the Qwen2.5-7B attention geometry (28 / 4 heads, head_dim 128):
  graphs on equal graphs off, and the run equals infrared's own bf16 naive
  path token for token up to the first near-tie (two logits closer than
  what the two attention numerics can separate), with every logit row
  before it within the bf16 bar. infrared's bf16 path computes scores in
  bf16; the kernels in fp32, so the two can part only at such a tie.
* the installed kernels actually ran (call counters on the ops they use;
  the spy is set before the shim is installed, so the shim binds it).
"""

from __future__ import annotations

import random

import pytest
import torch

import infrared_ref
from infrared_b200 import attention, ops, shim

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU"),
    pytest.mark.skipif(not infrared_ref.importable(), reason="infrared is not installed"),
]

DEV = "cuda"
# infrared's own prompts (tests/test_paged_kv.py:101-102) and longer ones that
# span many blocks, so that sequences are split across CTAs
_PROMPTS = [[3, 9, 1, 27, 5], [8, 2], [10, 11, 12], [7], [4, 4, 4, 4]]
_MAX_NEW = [12, 8, 6, 10, 9]


def _long_prompts(n, lo, hi, vocab, seed):
    rng = random.Random(seed)
    return [[rng.randrange(1, vocab) for _ in range(rng.randint(lo, hi))] for _ in range(n)]


def _model(dtype, *, head_dim, heads, kv_heads, hidden, inter, vocab, layers=2, seed=0,
           max_pos=1024):
    from infrared.model.config import Qwen2Config
    from infrared.model.qwen2 import Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter,
                      num_hidden_layers=layers, num_attention_heads=heads,
                      num_key_value_heads=kv_heads, head_dim=head_dim, rms_norm_eps=1e-6,
                      rope_theta=1_000_000.0, max_position_embeddings=max_pos,
                      tie_word_embeddings=True, bos_token_id=0, eos_token_ids=())
    torch.manual_seed(seed)
    model = Qwen2ForCausalLM(cfg)
    model.lm_head.weight = model.model.embed_tokens.weight
    model = model.to(device=DEV, dtype=dtype).eval()
    model.lm_head.weight = model.model.embed_tokens.weight
    return model


def _small_fp32():
    return _model(torch.float32, head_dim=64, heads=4, kv_heads=2, hidden=256, inter=512,
                  vocab=256)


def _qwen7b_attention_bf16():
    return _model(torch.bfloat16, head_dim=128, heads=28, kv_heads=4, hidden=3584, inter=1024,
                  vocab=512)


class _Recorder:
    """infrared's Sampler, recording every logits row it is given."""

    def __init__(self, inner):
        self.inner = inner
        self.rows = []

    def sample(self, logits, temperature=0.0, generator=None):
        tok = self.inner.sample(logits, temperature, generator)
        self.rows.append((logits.detach().float().cpu(), tok))
        return tok


def _run_engine(model, prompts, max_new, *, record=False, **kw):
    """Submit every request, then start the engine (a fixed schedule), and
    return the outputs (and the engine)."""
    from infrared.engine.paged_engine import PagedBatchEngine
    from infrared.engine.static_batch import BatchRequest

    engine = PagedBatchEngine(model, **kw)
    if record:
        engine.sampler = _Recorder(engine.sampler)
    pends = [engine.submit(BatchRequest(p, max_new_tokens=m, eos_token_ids=()))
             for p, m in zip(prompts, max_new, strict=True)]
    engine.start()
    try:
        outs = [p.result(timeout=300) for p in pends]
    finally:
        engine.stop()
    torch.cuda.synchronize()
    ops.check_device_errors()
    return outs, engine


def _oracle(model, prompt, max_new):
    from infrared.model.generate import generate

    return generate(model, prompt, max_new_tokens=max_new, temperature=0.0,
                    eos_token_ids=()).generated_ids


@pytest.fixture
def spy(monkeypatch):
    """Counts the calls of the kernels' Python entry points the shim uses."""
    from infrared_b200 import graph_inputs

    counts = {}
    targets = [(ops, n) for n in ("cache_write", "paged_decode", "paged_decode_rope_write",
                                  "paged_prefill", "derive_block_metadata",
                                  "derive_varlen_metadata", "kv_proj_rope_write",
                                  "paged_decode_rope")]
    targets.append((graph_inputs, "build_decode_static_inputs"))
    for mod, name in targets:
        fn = getattr(mod, name)

        def wrapped(*a, _fn=fn, _name=name, **k):
            counts[_name] = counts.get(_name, 0) + 1
            return _fn(*a, **k)

        monkeypatch.setattr(mod, name, wrapped)
    return counts


@pytest.fixture
def installed():
    """Install the shim with the given options; uninstall afterwards."""
    handles = []

    def _install(**kw):
        h = shim.install(**kw)
        handles.append(h)
        return h

    yield _install
    for h in reversed(handles):
        h.uninstall()
    attention.clear_metadata_cache()


def _assert_tokens_match_up_to_near_tie(rec_ref, rec_new, what):
    """Tokens of two recorded runs agree call by call until the first place
    where the reference's top two logits are closer than the two runs' logits
    differ (a near-tie); rows before it agree within the bf16 bar."""
    assert rec_ref and rec_new
    worst = 0.0
    for i, ((a, ta), (b, tb)) in enumerate(zip(rec_ref, rec_new)):
        scale = float(a.abs().max())
        diff = float((a - b).abs().max())
        worst = max(worst, diff / max(scale, 1e-6))
        assert diff <= 0.05 * scale + 1e-3, f"{what}: logits row {i} differs by {diff}"
        if ta != tb:
            top2 = torch.topk(a, 2).values
            gap = float(top2[0] - top2[1])
            assert gap <= 2 * diff + 1e-3, (
                f"{what}: call {i} picks {tb} instead of {ta} with a top-2 gap of {gap} "
                f"(logits differ by {diff})")
            return i
    assert len(rec_ref) == len(rec_new), what
    return None


# ------------------------------------------------------------------ fp32: exact


def test_eager_engine_matches_t0_oracle(installed, spy):
    model = _small_fp32()
    prompts = _PROMPTS + _long_prompts(3, 40, 150, 256, seed=1)
    max_new = _MAX_NEW + [20, 20, 20]
    installed()
    outs, _ = _run_engine(model, prompts, max_new, max_num_seqs=8, block_size=16,
                          num_blocks=128)
    for i, (p, m) in enumerate(zip(prompts, max_new)):
        assert outs[i] == _oracle(model, p, m), f"seq {i} diverged from T0"
    assert spy.get("paged_decode", 0) > 0 and spy.get("cache_write", 0) > 0, spy


def test_engine_matches_t0_under_preemption(installed, spy):
    """infrared's own preemption gate (tests/test_paged_kv.py:138-148) with the
    kernels in place: a pool too small forces evict / recompute."""
    model = _small_fp32()
    installed()
    outs, engine = _run_engine(model, _PROMPTS, _MAX_NEW, max_num_seqs=4, block_size=4,
                               num_blocks=6)
    for i, (p, m) in enumerate(zip(_PROMPTS, _MAX_NEW)):
        assert outs[i] == _oracle(model, p, m), f"seq {i} diverged under preemption"
    assert engine.preemptions > 0
    assert engine.block_manager.num_used_blocks == 0
    assert spy.get("paged_decode", 0) > 0, spy


def test_cuda_graph_engine_matches_eager_and_t0(installed, spy):
    """infrared's graphs-on == graphs-off gate (tests/test_cuda_graph.py:261-288)
    with the kernels captured inside infrared's decode graphs."""
    model = _small_fp32()
    prompts = _PROMPTS[:3] + _long_prompts(2, 60, 120, 256, seed=2)
    max_new = [10, 8, 6, 16, 16]
    installed()
    kw = dict(max_num_seqs=8, block_size=16, num_blocks=96, graph_max_seq_len=256)
    graph_outs, engine = _run_engine(model, prompts, max_new, enable_cuda_graph=True, **kw)
    assert engine._graph_decoder is not None and engine._graph_decoder._graphs
    eager_outs, _ = _run_engine(model, prompts, max_new, enable_cuda_graph=False, **kw)
    assert graph_outs == eager_outs
    for i, (p, m) in enumerate(zip(prompts, max_new)):
        assert graph_outs[i] == _oracle(model, p, m), f"seq {i} diverged from T0"
    assert spy.get("build_decode_static_inputs", 0) > 0, spy


@pytest.mark.parametrize("options", [
    dict(fuse_rope=True),
    dict(eager_inputs=True),
    dict(prefill=True),
    dict(fuse_rope=True, eager_inputs=True, prefill=True),
])
def test_shim_options_match_t0_oracle(installed, spy, options):
    model = _small_fp32()
    prompts = _PROMPTS + _long_prompts(2, 50, 130, 256, seed=3)
    max_new = _MAX_NEW + [15, 15]
    installed(**options)
    outs, _ = _run_engine(model, prompts, max_new, max_num_seqs=8, block_size=16,
                          num_blocks=96)
    for i, (p, m) in enumerate(zip(prompts, max_new)):
        assert outs[i] == _oracle(model, p, m), f"seq {i} diverged ({options})"
    if options.get("fuse_rope"):
        assert spy.get("paged_decode_rope_write", 0) > 0, spy
    if options.get("prefill"):
        assert spy.get("derive_varlen_metadata", 0) > 0, spy


def test_chunked_prefill_engine_matches_t0_oracle(installed, spy):
    """infrared's mixed prefill + decode steps (packed varlen frames) on the
    prefill kernel path, chunks small enough that prompts span several steps."""
    model = _small_fp32()
    prompts = _long_prompts(4, 30, 90, 256, seed=4) + _PROMPTS[:2]
    max_new = [12, 12, 12, 12, 8, 8]
    installed(prefill=True)
    outs, engine = _run_engine(model, prompts, max_new, max_num_seqs=6, block_size=16,
                               num_blocks=96, enable_chunked_prefill=True, chunk_size=32)
    assert engine.mixed_steps > 0
    for i, (p, m) in enumerate(zip(prompts, max_new)):
        assert outs[i] == _oracle(model, p, m), f"seq {i} diverged (chunked prefill)"
    assert spy.get("derive_varlen_metadata", 0) > 0, spy


# ------------------------------------------------------------------ bf16, 7B geometry


def test_bf16_graphs_on_equal_graphs_off(installed):
    model = _qwen7b_attention_bf16()
    prompts = _long_prompts(6, 20, 300, 512, seed=5)
    max_new = [16] * 6
    installed(fuse_rope=True, prefill=True)
    kw = dict(max_num_seqs=8, block_size=16, num_blocks=256, graph_max_seq_len=512,
              record=True)
    g_outs, g_eng = _run_engine(model, prompts, max_new, enable_cuda_graph=True, **kw)
    e_outs, e_eng = _run_engine(model, prompts, max_new, enable_cuda_graph=False, **kw)
    assert g_eng._graph_decoder is not None and g_eng._graph_decoder._graphs
    cut = _assert_tokens_match_up_to_near_tie(e_eng.sampler.rows, g_eng.sampler.rows,
                                              "graphs on vs off")
    if cut is None:
        assert g_outs == e_outs


@pytest.mark.parametrize("graphs", [False, True])
def test_bf16_engine_matches_infrared_own_path(installed, spy, graphs):
    """The same engine run on infrared's own bf16 naive path (no shim,
    enable_triton_attention=False) and on the installed kernels."""
    model = _qwen7b_attention_bf16()
    prompts = _long_prompts(6, 20, 300, 512, seed=6)
    max_new = [16] * 6
    kw = dict(max_num_seqs=8, block_size=16, num_blocks=256, graph_max_seq_len=512,
              enable_cuda_graph=graphs, record=True)
    _, ref_eng = _run_engine(model, prompts, max_new, enable_triton_attention=False, **kw)
    installed(fuse_rope=True, prefill=True)
    _, new_eng = _run_engine(model, prompts, max_new, enable_triton_attention=True, **kw)
    _assert_tokens_match_up_to_near_tie(ref_eng.sampler.rows, new_eng.sampler.rows,
                                        f"infrared bf16 vs kernels (graphs={graphs})")
    assert spy.get("paged_prefill", 0) + spy.get("derive_varlen_metadata", 0) > 0, spy
    if not graphs:
        assert spy.get("paged_decode_rope_write", 0) > 0, spy


@pytest.mark.parametrize("graphs", [False, True])
def test_bf16_engine_with_the_projection_kernel(installed, spy, graphs):
    """``shim.install(fuse_kv_proj=True)``: each decode step's K/V projections,
    RoPE and cache write run in ir_kv_proj_rope_write and the decode applies
    RoPE to q (ir_paged_decode_rope); against infrared's own bf16 path."""
    model = _qwen7b_attention_bf16()
    prompts = _long_prompts(6, 20, 300, 512, seed=7)
    max_new = [16] * 6
    kw = dict(max_num_seqs=8, block_size=16, num_blocks=256, graph_max_seq_len=512,
              enable_cuda_graph=graphs, record=True)
    _, ref_eng = _run_engine(model, prompts, max_new, enable_triton_attention=False, **kw)
    installed(fuse_kv_proj=True, prefill=True)
    _, new_eng = _run_engine(model, prompts, max_new, enable_triton_attention=True, **kw)
    _assert_tokens_match_up_to_near_tie(ref_eng.sampler.rows, new_eng.sampler.rows,
                                        f"infrared bf16 vs projection kernel (graphs={graphs})")
    assert spy.get("kv_proj_rope_write", 0) > 0 and spy.get("paged_decode_rope", 0) > 0, spy
