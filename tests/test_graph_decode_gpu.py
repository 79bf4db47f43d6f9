"""Device-side token commit (``lf_commit_token``) and the CUDA-graph decode
loop (``GraphDecoder``) on the GPU.

* The device commit of one token per sequence, step after step across page
  flushes at different steps for every sequence, leaves exactly the bytes of
  the host-driven commit (residual pages, packed history, meta rows, lengths).
* A tiny random Qwen2 decoded greedily through the replayed graph produces the
  same tokens as the eager adapter loop, logits within the decode tolerance's
  propagation, and (layer 0, whose Key/Value depend only on the tokens) the
  same packed history bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from logitfill_b200.adapter import DeepSeekQwenKVAdapter
from logitfill_b200.graph_decode import GraphDecoder
from logitfill_b200.packed import PackedKVCache
from logitfill_b200.synthetic import synthetic_kv, synthetic_levels
from tests.gpu_cases import bit_equal
from tests.qwen_cases import tiny_qwen2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_device_commit_equals_host_commit(dtype):
    B, H, NQ, D, P = 3, 4, 28, 128, 128
    levels = synthetic_levels(1, H, D, 2.5, seed=21)[0]
    k, v = synthetic_kv(B, H, 700, D, seed=21, layer=0, device="cuda", dtype=dtype)
    starts = [130, 250, 383]                          # tails 2, 122, 127: flushes at different steps
    dev = PackedKVCache([levels], B, NQ, H, D, device="cuda", capacity=1024)
    host = PackedKVCache([levels], B, NQ, H, D, device="cuda", capacity=1024)
    for c in (dev, host):
        c.prefill(0, k, v, starts)
    for step in range(200):
        kt = torch.stack([k[b, :, s + step] for b, s in enumerate(starts)])
        vt = torch.stack([v[b, :, s + step] for b, s in enumerate(starts)])
        dev.layers[0].commit_token_device(kt, vt)
        dev.layers[0].advance_host()
        host.commit(0, kt[:, :, None], vt[:, :, None])
    dev.check_status()
    a, b = dev.layers[0], host.layers[0]
    assert np.array_equal(a.hist_len, b.hist_len) and np.array_equal(a.tail_len, b.tail_len)
    assert torch.equal(a.dev_hist, b.dev_hist) and torch.equal(a.dev_tail, b.dev_tail)
    assert torch.equal(a.rows, b.rows) and torch.equal(a.kmeta, b.kmeta)
    for s in range(B):
        n = int(a.tail_len[s])
        assert torch.equal(a.tail_k[s, :, :n], b.tail_k[s, :, :n]) and torch.equal(a.tail_v[s, :, :n], b.tail_v[s, :, :n])


def _eager_greedy(model, adapter, prompt, n):
    cache = adapter.make_cache()
    cache.reset()
    toks, logits = [], []
    with torch.inference_mode():
        out = model(input_ids=prompt, use_cache=True, past_key_values=cache)
        for _ in range(n):
            lg = out.logits[:, -1].float()
            tok = lg.argmax(-1, keepdim=True)
            toks.append(int(tok))
            logits.append(lg)
            out = model(input_ids=tok, use_cache=True, past_key_values=out.past_key_values)
    return toks, logits


def test_graph_decode_matches_eager_loop():
    torch.manual_seed(0)
    model = tiny_qwen2(n_q=8, n_kv=2, head_dim=128, layers=2, vocab=512, seed=23, device="cuda", attn="sdpa")
    levels = list(synthetic_levels(2, 2, 128, 2.5, seed=23))
    prompt = torch.randint(0, 512, (1, 100), generator=torch.Generator().manual_seed(23)).cuda()
    n = 60                                            # crosses the page boundary at token 128

    a = DeepSeekQwenKVAdapter(model).attach()
    a.set_k_levels(levels)
    toks_e, logits_e = _eager_greedy(model, a, prompt, n)
    store_e = {k: t.clone() for k, t in (("rows", a.packed_manager().cache.layers[0].rows),
                                          ("kmeta", a.packed_manager().cache.layers[0].kmeta))}
    a.set_k_levels(levels)                            # a fresh packed store for the graph run
    g = GraphDecoder(model, a, max_tokens=256)
    lg = g.prefill(prompt).float()
    toks_g, logits_g = [], []
    for _ in range(n):
        tok = lg.argmax(-1, keepdim=True)
        toks_g.append(int(tok))
        logits_g.append(lg.clone())
        lg = g.step(tok).float()
    mgr = a.packed_manager()
    mgr.cache.check_status()
    assert toks_g == toks_e
    diff = max(float((x - y).abs().max()) for x, y in zip(logits_g, logits_e))
    scale = max(float(y.abs().max()) for y in logits_e)
    assert diff <= 1e-3 * scale, (diff, scale)
    assert mgr.seq_len == 100 + n and int(mgr.cache.layers[0].dev_hist[0]) == 128
    layer = mgr.cache.layers[0]
    hist = int(layer.hist_len[0])
    assert bit_equal(layer.rows[:, :, :hist].cpu().numpy(), store_e["rows"][:, :, :hist].cpu().numpy())
    assert bit_equal(layer.kmeta[:, :, :hist // 128].cpu().numpy(), store_e["kmeta"][:, :, :hist // 128].cpu().numpy())
    g.release()
