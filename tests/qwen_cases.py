"""Tiny random Qwen2 models and the two reference computations the
model-level adapter tests compare against.

* :class:`OracleManager` -- the reference's ``PackedKVManager`` +
  ``reference_attention`` (``src/logitfill/packed/cache.py:93-140``,
  ``packed/reference.py:30-56``) on the numpy oracle, with the ``attend``
  method the adapter calls.  Injected into an adapter it checks the adapter's
  host logic on the CPU.
* :func:`fake_quant_logits` -- the stock model with a dense cache whose
  completed pages are replaced, after each forward, by their packed-codec
  round trip (the page-delayed quantization of
  ``models/qwen2_attention.py:47-71,188-220`` with the packed codec of
  ``packed/layout.py``).  This is what the packed backend computes, without
  any packed store.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import packed_ref as orc


def tiny_qwen2(*, n_q=8, n_kv=2, head_dim=128, layers=2, vocab=512, seed=0, dtype=torch.float32,
               device="cpu", attn="eager"):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(seed)
    cfg = Qwen2Config(vocab_size=vocab, hidden_size=n_q * head_dim, intermediate_size=2 * n_q * head_dim,
                      num_hidden_layers=layers, num_attention_heads=n_q, num_key_value_heads=n_kv,
                      max_position_embeddings=4096, attention_dropout=0.0, rope_theta=10000.0)
    cfg._attn_implementation = attn
    model = Qwen2ForCausalLM(cfg).eval()
    # Larger projections than the 0.02 default so attention is far from uniform.
    with torch.no_grad():
        for layer in model.model.layers:
            for proj in (layer.self_attn.q_proj, layer.self_attn.k_proj):
                proj.weight.mul_(4.0)
    return model.to(device=device, dtype=dtype)


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


class _OracleStore:
    def __init__(self, levels, page, k_group, v_group):
        self.layer = orc.OracleLayer(np.asarray(levels), page, k_group, v_group, 2)

    @property
    def length(self) -> int:
        return self.layer.length


class OracleManager:
    """``PackedKVManager`` semantics on the CPU oracle (cache.py:93-140)."""

    def __init__(self, levels, n_q, n_kv, head_dim, page_size, k_group_size, v_group_size):
        self.n_q, self.n_kv, self.head_dim, self.bit_v = n_q, n_kv, head_dim, 2
        self.page_size = page_size
        self._args = (page_size, k_group_size, v_group_size)
        self._levels = [np.zeros((n_kv, head_dim), np.int64) if lv is None else np.asarray(lv) for lv in levels]
        self.reset()

    def reset(self) -> None:
        self.seq_len = 0
        self.layers = [_OracleStore(lv, *self._args) for lv in self._levels]

    def layer_length(self, layer_idx: int) -> int:
        return self.layers[layer_idx].length

    def commit(self, layer_idx, key, value) -> None:
        if key.shape[0] != 1:
            raise NotImplementedError("packed KV supports one sequence at a time")
        self.layers[layer_idx].layer.append(_np(key[0]), _np(value[0]))
        if layer_idx == len(self.layers) - 1:
            self.seq_len = self.layers[layer_idx].length

    def attend(self, layer_idx, query, key_new, value_new, scaling):
        out = orc.reference_attention(self.layers[layer_idx].layer, _np(query[0]), _np(key_new[0]),
                                      _np(value_new[0]), scaling)
        return torch.from_numpy(out.astype(np.float32))[None].to(device=query.device, dtype=query.dtype)


def _steps(ids, prompt_len, chunks=None):
    """The prompt, then ``chunks`` (token counts; default one token per step)
    up to the end of ``ids``."""
    out, t = [ids[:, :prompt_len]], prompt_len
    for n in (chunks or []):
        out.append(ids[:, t:t + n])
        t += n
    out.extend(ids[:, u:u + 1] for u in range(t, ids.shape[1]))
    return out


def _layer_kv(cache, i):
    if hasattr(cache, "layers") and len(getattr(cache, "layers")) > i and hasattr(cache.layers[i], "keys"):
        return cache.layers[i].keys, cache.layers[i].values
    return cache.key_cache[i], cache.value_cache[i]


def _round_trip_pages(cache, n_layers, levels, page, k_group, v_group, start, stop) -> None:
    """Replace tokens ``[start, stop)`` (whole pages) of every layer's dense
    cache with their packed-codec round trip."""
    for i in range(n_layers):
        keys, values = _layer_kv(cache, i)
        lv = levels[i]
        table = orc.tier_tables(np.zeros(keys.shape[1:2] + keys.shape[3:], np.int64) if lv is None
                                else np.asarray(lv))
        D = keys.shape[-1]
        for a in range(start, stop, page):
            pk = keys[0, :, a:a + page].float().cpu().numpy()
            pv = values[0, :, a:a + page].float().cpu().numpy()
            rk = orc.dequantize_key(page, table, orc.quantize_key_page(pk, table, k_group), k_group)
            rv = orc.dequantize_value(orc.quantize_value_page(pv, 2, v_group), page, D, 2, v_group)
            keys[0, :, a:a + page] = torch.from_numpy(rk).to(keys.dtype)
            values[0, :, a:a + page] = torch.from_numpy(rv).to(values.dtype)


@torch.no_grad()
def fake_quant_logits(model, ids, prompt_len, levels, page, k_group, v_group, chunks=None):
    """Last-position logits of the prefill and of every teacher-forced decode
    step, with page-delayed packed-codec quantization of the dense cache."""
    from transformers import DynamicCache

    n_layers = model.config.num_hidden_layers
    try:
        cache = DynamicCache(config=model.config)
    except TypeError:
        cache = DynamicCache()
    outs = []
    done = 0
    steps = _steps(ids, prompt_len, chunks)
    for chunk in steps:
        out = model(input_ids=chunk, past_key_values=cache, use_cache=True)
        outs.append(out.logits[:, -1].float())
        total = cache.get_seq_length()
        flushed = total // page * page
        if flushed > done:
            _round_trip_pages(cache, n_layers, levels, page, k_group, v_group, done, flushed)
            done = flushed
    return outs


@torch.no_grad()
def adapter_logits(model, adapter, ids, prompt_len, chunks=None):
    """Same steps through ``adapter`` (packed backend) with its cache handle."""
    cache = adapter.make_cache()
    outs = []
    steps = _steps(ids, prompt_len, chunks)
    for chunk in steps:
        out = model(input_ids=chunk, past_key_values=cache, use_cache=True)
        outs.append(out.logits[:, -1].float())
    return outs


@torch.no_grad()
def stock_logits(model, ids, prompt_len, chunks=None):
    """The unmodified model with its own dense cache (no quantization)."""
    from transformers import DynamicCache

    try:
        cache = DynamicCache(config=model.config)
    except TypeError:
        cache = DynamicCache()
    outs = []
    steps = _steps(ids, prompt_len, chunks)
    for chunk in steps:
        out = model(input_ids=chunk, past_key_values=cache, use_cache=True)
        outs.append(out.logits[:, -1].float())
    return outs


class CheckedManager:
    """A real (CUDA) ``PackedKVManager`` driving the model, with every commit
    mirrored into an :class:`OracleManager` and every attention call checked
    against the oracle on the same inputs: the kernels' fp32 output (before
    the cast to the query dtype) against the reference's dense packed
    attention.  ``worst`` holds the largest max-abs error and the smallest
    cosine seen; ``calls`` counts decode calls."""

    def __init__(self, real, oracle):
        self.real, self.oracle = real, oracle
        self.worst = (0.0, 1.0)
        self.calls = 0
        self.tokens = 0

    def __getattr__(self, name):
        return getattr(self.real, name)

    @property
    def seq_len(self):
        return self.real.seq_len

    def reset(self) -> None:
        self.real.reset()
        self.oracle.reset()

    def commit(self, layer_idx, key, value) -> None:
        self.real.commit(layer_idx, key, value)
        self.oracle.commit(layer_idx, key, value)

    def attend(self, layer_idx, query, key_new, value_new, scaling):
        from logitfill_b200.packed.attention import decode_into

        out = torch.empty(query.shape, dtype=torch.float32, device=query.device)
        decode_into(self.real.cache, layer_idx, query, key_new, value_new, scaling, out)
        want = orc.reference_attention(self.oracle.layers[layer_idx].layer, _np(query[0]), _np(key_new[0]),
                                       _np(value_new[0]), scaling)
        got = out[0].cpu().numpy().astype(np.float64)
        err = float(np.abs(got - want).max())
        cos = float(np.min(np.sum(got * want, -1) / (np.linalg.norm(got, axis=-1) * np.linalg.norm(want, axis=-1))))
        self.worst = (max(self.worst[0], err), min(self.worst[1], cos))
        self.calls += 1
        self.tokens += query.shape[2]
        return out.to(query.dtype)
