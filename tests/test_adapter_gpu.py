"""Model-level drop-in on the GPU: ``DeepSeekQwenKVAdapter(backend="packed")``
driving the CUDA kernels (K1 page pack, K2 + K3 decode) inside a tiny random
``Qwen2ForCausalLM``.

A prompt and teacher-forced decode steps cross several page boundaries.  The
adapter's CUDA store is wrapped so that every commit is mirrored into the
oracle store and every decode attention call is checked against the
reference's dense packed attention on the same inputs (max-abs 2e-3, cosine
0.9999, on the kernels' fp32 output); at the end the packed history of every
layer must equal the oracle's bit for bit.

(Comparing final logits with an independently computed model instead would
not be a parity check: a last-bit difference upstream can move a Key value
across a quantization boundary of a later page and change its code.)
"""
from __future__ import annotations

import pytest
import torch

from logitfill_b200.adapter import DeepSeekQwenKVAdapter
from logitfill_b200.synthetic import synthetic_levels
from tests.gpu_cases import ATOL, MIN_COS, bit_equal, store_arrays
from tests.oracle_runner import layer_arrays
from tests.qwen_cases import CheckedManager, OracleManager, adapter_logits, tiny_qwen2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,page,attn", [
    (torch.float32, 64, "eager"),      # CUDA-core decode kernel
    (torch.float32, 128, "sdpa"),      # tensor-core decode kernel (the DeepSeek geometry)
    (torch.bfloat16, 128, "sdpa"),
])
def test_model_decode_matches_reference_on_same_inputs(dtype, page, attn):
    layers, n_q, n_kv, D = 3, 8, 2, 128
    model = tiny_qwen2(n_q=n_q, n_kv=n_kv, head_dim=D, layers=layers, vocab=512, seed=11, device="cuda",
                       dtype=dtype, attn=attn)
    levels = list(synthetic_levels(layers, n_kv, D, 2.5, seed=11))
    ids = torch.randint(0, 512, (1, 330), generator=torch.Generator().manual_seed(11)).cuda()
    prompt = 150
    a = DeepSeekQwenKVAdapter(model, group_size=page, v_group_size=D).attach()
    a.set_k_levels(levels)
    real = a.packed_manager()
    checked = CheckedManager(real, OracleManager(levels, n_q, n_kv, D, page, page, D))
    a._packed = checked
    logits = adapter_logits(model, a, ids, prompt)
    real.cache.check_status()
    assert checked.calls == (330 - prompt) * layers
    err, cos = checked.worst
    print(f"{dtype} page {page}: worst attention max-abs {err:.2e}, min cos {cos:.8f}")
    assert err <= ATOL and cos >= MIN_COS
    assert all(torch.isfinite(x).all() for x in logits)
    for i in range(layers):
        got, want = store_arrays(real.layers[i]), layer_arrays(checked.oracle.layers[i].layer)
        assert set(got) == set(want)
        for key in want:
            assert bit_equal(got[key], want[key]), (i, key)
        assert real.layers[i].hist_len == 330 // page * page and real.layers[i].tail_len == 330 % page


def test_greedy_decode_loop_runs_on_the_packed_path():
    """The reference's sampling loop shape (benchmarks/generate.py:28-57):
    prefill, then one token at a time through the cache handle; the packed
    store holds every token and a reset starts a new sequence."""
    model = tiny_qwen2(n_q=8, n_kv=2, head_dim=128, layers=2, vocab=512, seed=13, device="cuda",
                       dtype=torch.bfloat16, attn="sdpa")
    a = DeepSeekQwenKVAdapter(model).attach()
    a.set_k_levels(list(synthetic_levels(2, 2, 128, 3.0, seed=13)))
    mgr = a.packed_manager()
    for prompt_len in (140, 60):
        prompt = torch.randint(0, 512, (1, prompt_len), generator=torch.Generator().manual_seed(prompt_len)).cuda()
        cache = a.make_cache()
        cache.reset()
        with torch.inference_mode():
            out = model(input_ids=prompt, use_cache=True, past_key_values=cache)
            for _ in range(100):
                token = out.logits[:, -1].argmax(-1, keepdim=True)
                out = model(input_ids=token, use_cache=True, past_key_values=out.past_key_values)
        assert mgr.seq_len == prompt_len + 100
        assert mgr.layers[0].hist_len == (prompt_len + 100) // 128 * 128
        assert torch.isfinite(out.logits).all()
    mgr.cache.check_status()


@pytest.mark.parametrize("page", [64, 128])
def test_chunked_prefill_continuation(page):
    """Prompt, then prefill chunks of 37 and 64 tokens over the packed
    history (q_len > 1, causal among the chunk's tokens), then decode steps:
    every call checked against the oracle on the same inputs."""
    layers, n_q, n_kv, D = 2, 8, 2, 128
    model = tiny_qwen2(n_q=n_q, n_kv=n_kv, head_dim=D, layers=layers, vocab=512, seed=21, device="cuda",
                       dtype=torch.bfloat16, attn="sdpa")
    levels = list(synthetic_levels(layers, n_kv, D, 3.0, seed=21))
    ids = torch.randint(0, 512, (1, 300), generator=torch.Generator().manual_seed(21)).cuda()
    a = DeepSeekQwenKVAdapter(model, group_size=page, v_group_size=D).attach()
    a.set_k_levels(levels)
    real = a.packed_manager()
    checked = CheckedManager(real, OracleManager(levels, n_q, n_kv, D, page, page, D))
    a._packed = checked
    adapter_logits(model, a, ids, 150, chunks=[37, 64])
    real.cache.check_status()
    assert checked.tokens == (300 - 150) * layers and checked.calls == (2 + 300 - 251) * layers
    err, cos = checked.worst
    print(f"chunked page {page}: worst attention max-abs {err:.2e}, min cos {cos:.8f}")
    assert err <= ATOL and cos >= MIN_COS
    for i in range(layers):
        got, want = store_arrays(real.layers[i]), layer_arrays(checked.oracle.layers[i].layer)
        for key in want:
            assert bit_equal(got[key], want[key]), (i, key)
