"""Host logic of the model-level drop-in (``DeepSeekQwenKVAdapter``,
backend="packed") on a tiny random Qwen2, on the CPU.

The adapter's packed store is replaced by :class:`OracleManager` (the
reference's manager and dense packed attention on the numpy oracle), so these
tests check the adapter's wiring -- rotary positions, the cache handle under
the installed transformers, the dense first prefill, page-delayed commits,
output layout, the 4.x/5.x cache keyword -- without a GPU.  The GPU tests run
the same comparisons through the CUDA kernels.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import packed_ref as orc

from logitfill_b200.adapter import DeepSeekQwenKVAdapter
from logitfill_b200.packed.cache import LogitFillCache
from logitfill_b200.policy import (KeyPolicy, TierTables, check_model_fit, key_budget_report, read_policy,
                                   write_policy)
from logitfill_b200.synthetic import synthetic_levels
from tests.qwen_cases import OracleManager, adapter_logits, fake_quant_logits, stock_logits, tiny_qwen2


def _inject(adapter, page=None):
    levels = [layer.self_attn.k_levels for layer in adapter.model.model.layers]
    adapter._packed = OracleManager(levels, adapter.n_q, adapter.n_kv, adapter.head_dim,
                                    page or adapter.page_size, adapter.group_size, adapter.v_group_size)
    return adapter._packed


def _max_abs(a, b):
    return max(float((x - y).abs().max()) for x, y in zip(a, b))


def test_constructor_checks():
    model = tiny_qwen2(layers=1, n_q=2, n_kv=1, head_dim=32, vocab=64)
    with pytest.raises(TypeError):
        DeepSeekQwenKVAdapter(torch.nn.Linear(2, 2))
    with pytest.raises(ValueError):
        DeepSeekQwenKVAdapter(model, backend="dense")
    with pytest.raises(NotImplementedError):
        DeepSeekQwenKVAdapter(model, backend="fake")
    with pytest.raises(ValueError):
        DeepSeekQwenKVAdapter(model, group_size=0)
    with pytest.raises(ValueError):
        DeepSeekQwenKVAdapter(model, group_size=16, page_size=24)
    with pytest.raises(ValueError):
        DeepSeekQwenKVAdapter(model, group_size=16, v_group_size=12)
    with pytest.raises(NotImplementedError):
        DeepSeekQwenKVAdapter(model, group_size=16, bit_v=4)
    a = DeepSeekQwenKVAdapter(model, group_size=16, v_group_size=32)
    assert (a.page_size, a.v_group_size, a.backend) == (16, 32, "packed")


def test_attach_detach_and_levels():
    model = tiny_qwen2(layers=2, n_q=2, n_kv=1, head_dim=32, vocab=64)
    originals = [layer.self_attn.forward for layer in model.model.layers]
    a = DeepSeekQwenKVAdapter(model, group_size=16, v_group_size=32)
    with pytest.raises(RuntimeError):
        a.set_k_levels(None)
    a.attach()
    assert model._kv_adapter is a
    assert all(layer.self_attn.forward is not o for layer, o in zip(model.model.layers, originals))
    with pytest.raises(ValueError):
        a.set_k_levels([np.zeros((1, 32))])           # wrong layer count
    with pytest.raises(ValueError):
        a.set_k_levels([np.zeros((1, 16))] * 2)       # wrong map shape
    a._packed = object()
    a.set_k_levels([np.full((1, 32), 1)] * 2)
    assert a._packed is None                          # history dropped with the old map
    assert int(model.model.layers[1].self_attn.k_levels[0, 0]) == 1
    a.detach()
    assert model._kv_adapter is None
    assert [layer.self_attn.forward for layer in model.model.layers] == originals


def test_policy_round_trip_and_checks(tmp_path):
    model = tiny_qwen2(layers=2, n_q=4, n_kv=2, head_dim=128, vocab=64)
    levels = synthetic_levels(2, 2, 128, 2.5, seed=3)
    meta = {"n_layers": 2, "n_kv": 2, "head_dim": 128, "target_bit": 2.5, "bit_v": 2}
    write_policy(tmp_path / "p", KeyPolicy(levels, meta, {"d2": np.ones(levels.shape)}))
    pol = read_policy(tmp_path / "p")
    assert np.array_equal(pol.levels, levels) and pol.metadata == meta and set(pol.curves) == {"d2"}
    a = DeepSeekQwenKVAdapter(model).attach()
    a.load_policy(tmp_path / "p")
    assert np.array_equal(np.asarray(model.model.layers[1].self_attn.k_levels), levels[1])
    with pytest.raises(ValueError):                   # over the per-head Key budget
        KeyPolicy(np.full((2, 2, 128), 2), meta)
    KeyPolicy(np.full((2, 2, 128), 2), dict(meta, enforce_budget=False))  # budget check switched off
    with pytest.raises(ValueError):                   # metadata disagrees with the map
        KeyPolicy(levels, dict(meta, n_kv=3))
    with pytest.raises(ValueError):
        KeyPolicy(np.full((2, 2, 128), 4), {})
    with pytest.raises(ValueError):
        KeyPolicy(levels, meta, {"d4": np.ones((2, 2))})  # extra array of another shape
    other = tiny_qwen2(layers=1, n_q=4, n_kv=2, head_dim=128, vocab=64)
    with pytest.raises(ValueError):
        check_model_fit(pol, other.config)
    write_policy(tmp_path / "q", KeyPolicy(levels, dict(meta, bit_v=3, enforce_budget=False)))
    with pytest.raises(ValueError):
        a.load_policy(tmp_path / "q")


def test_reference_written_policy_loads_and_tables_match_oracle():
    """tests/golden/policy_ref was written by the reference's own
    build_policy(...).save(...); it loads, its budget check passes, and the
    vectorised tier tables (built once per map and device) equal the
    reference-restated tables of layout.py:49-68."""
    pol = read_policy(Path(__file__).resolve().parent / "golden" / "policy_ref")
    assert pol.levels.shape == (2, 2, 128) and pol.metadata["model_id"] == "tiny-qwen2-test"
    assert set(pol.curves) == {"d2"}
    report = key_budget_report(pol.levels, pol.metadata["target_bit"], pol.metadata["bit_v"])
    assert report["max_extra_bits"] <= report["allowed_extra_bits"] == pol.metadata["extra_budget_per_head"]
    for i in range(2):
        tt = TierTables.get(pol.levels[i], "cpu")
        assert TierTables.get(torch.as_tensor(pol.levels[i]), "cpu") is tt
        ref = orc.tier_tables(pol.levels[i])
        for t in range(4):
            assert tt.table[t]["width"] == ref[t]["width"]
            for key in ("index", "count", "local"):
                assert np.array_equal(tt.table[t][key].numpy(), ref[t][key]), (i, t, key)
        assert np.array_equal(tt.counts, np.stack([ref[t]["count"] for t in range(4)]))
        chan = tt.chan_code.numpy()
        for c in range(128):
            tier = int(pol.levels[i][0, c])
            assert chan[0, c] == (tier << 16) | int(ref[tier]["local"][0, c])


def test_cache_handle_under_installed_transformers():
    mgr = OracleManager([None], 2, 1, 32, 16, 16, 32)
    cache = LogitFillCache(mgr)
    mgr.seq_len = 37
    assert cache.get_seq_length() == 37
    assert cache.get_mask_sizes(5, 0) == (42, 0)
    assert cache.get_mask_sizes(torch.arange(37, 40), 0) == (40, 0)
    with pytest.raises(RuntimeError):
        cache.update(None, None, 0)
    with pytest.raises(NotImplementedError):
        cache.reorder_cache(torch.zeros(1))


@pytest.mark.parametrize("attn", ["eager", "sdpa"])
def test_no_flush_matches_stock_model(attn):
    """With a page longer than the whole run nothing is quantized: every
    step must equal the unmodified model (wiring, positions, GQA, layout)."""
    model = tiny_qwen2(layers=2, n_q=8, n_kv=2, head_dim=64, vocab=128, attn=attn)
    ids = torch.randint(0, 128, (1, 40), generator=torch.Generator().manual_seed(1))
    ref = stock_logits(model, ids, 24)
    a = DeepSeekQwenKVAdapter(model, group_size=512, v_group_size=64).attach()
    _inject(a)
    got = adapter_logits(model, a, ids, 24)
    assert _max_abs(got, ref) < 1e-4


def test_page_flushes_match_fake_quantization():
    """Pages complete during prefill and during decode; the adapter over the
    oracle store equals the stock model over the round-tripped dense cache."""
    model = tiny_qwen2(layers=2, n_q=8, n_kv=2, head_dim=128, vocab=128)
    levels = list(synthetic_levels(2, 2, 128, 2.5, seed=5))
    ids = torch.randint(0, 128, (1, 60), generator=torch.Generator().manual_seed(2))
    page = 16
    ref = fake_quant_logits(model, ids, 37, levels, page, page, 128)
    a = DeepSeekQwenKVAdapter(model, group_size=page, v_group_size=128).attach()
    a.set_k_levels(levels)
    mgr = _inject(a)
    got = adapter_logits(model, a, ids, 37)
    assert mgr.seq_len == 60 and mgr.layers[1].layer.hist_len == 48
    assert _max_abs(got, ref) < 1e-4
    # Quantization is visible: the no-quantization model differs.
    a.detach()
    assert _max_abs(got, stock_logits(model, ids, 37)) > 1e-3


def test_legacy_cache_keyword_and_position_guard():
    """A 4.x-style call (``past_key_value=``) reaches the packed branch, and a
    decode step whose cache disagrees with the packed length raises."""
    from transformers import DynamicCache

    model = tiny_qwen2(layers=1, n_q=2, n_kv=1, head_dim=32, vocab=64)
    a = DeepSeekQwenKVAdapter(model, group_size=16, v_group_size=32).attach()
    mgr = _inject(a)
    attn = model.model.layers[0].self_attn
    h = torch.randn(1, 5, model.config.hidden_size)
    pos = torch.arange(5)[None]
    emb = model.model.rotary_emb(h, pos)
    cache = a.make_cache()
    out, _ = attn(hidden_states=h, position_embeddings=emb, attention_mask=None, past_key_value=cache,
                  cache_position=torch.arange(5))
    assert out.shape == h.shape and mgr.seq_len == 5
    h1 = torch.randn(1, 1, model.config.hidden_size)
    emb1 = model.model.rotary_emb(h1, torch.tensor([[5]]))
    try:
        stale = DynamicCache(config=model.config)
    except TypeError:
        stale = DynamicCache()
    with pytest.raises(ValueError):
        attn(hidden_states=h1, position_embeddings=emb1, attention_mask=None, past_key_values=stale)
    out1, _ = attn(hidden_states=h1, position_embeddings=emb1, attention_mask=None, past_key_values=cache)
    assert out1.shape == h1.shape and mgr.seq_len == 6


def test_skip_quant_runs_the_stock_path():
    model = tiny_qwen2(layers=2, n_q=4, n_kv=2, head_dim=32, vocab=64)
    ids = torch.randint(0, 64, (1, 12), generator=torch.Generator().manual_seed(4))
    ref = stock_logits(model, ids, 8)
    a = DeepSeekQwenKVAdapter(model, group_size=4, v_group_size=32).attach()
    a.skip_quant = True
    assert _max_abs(stock_logits(model, ids, 8), ref) < 1e-5


def test_chunked_continuation_matches_fake_quantization():
    """A multi-token call with history (a second prefill chunk) goes to the
    packed attention with the causal mask; its output is laid out
    [B, q_len, heads, D] before the output projection.  Pages complete inside
    the chunk."""
    model = tiny_qwen2(layers=2, n_q=8, n_kv=2, head_dim=128, vocab=128)
    levels = list(synthetic_levels(2, 2, 128, 2.5, seed=6))
    ids = torch.randint(0, 128, (1, 80), generator=torch.Generator().manual_seed(3))
    page, chunks = 16, [23, 5]
    ref = fake_quant_logits(model, ids, 21, levels, page, page, 128, chunks=chunks)
    a = DeepSeekQwenKVAdapter(model, group_size=page, v_group_size=128).attach()
    a.set_k_levels(levels)
    mgr = _inject(a)
    got = adapter_logits(model, a, ids, 21, chunks=chunks)
    assert mgr.seq_len == 80
    assert _max_abs(got, ref) < 1e-4
