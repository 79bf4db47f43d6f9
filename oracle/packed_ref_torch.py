"""Torch CPU restatement of the reference's dense packed-attention path.

TEST AND BASELINE INFRASTRUCTURE ONLY.  Imported by ``tests/`` and by the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``, never by the
product package.

The reference runs its packed path on PyTorch: ``reference_attention``
(src/logitfill/packed/reference.py:30-56) dequantizes the whole packed
history on every call (``_LayerStore.dequantize``, cache.py:83-90, through
``dequantize_key`` / ``dequantize_value``, layout.py:132-182: a Python loop
over tiers and heads of integer unpacking and ``code * scale + min``),
concatenates the original-dtype tail and the new tokens, expands the KV heads
(``repeat_kv``, reference.py:10-15) and calls fp32
``F.scaled_dot_product_attention``.  This module does the same torch
operations in the same order over an :class:`oracle.packed_ref.OracleLayer`
store, so its CPU cost is the reference's and its result equals the numpy
oracle's to fp32 rounding.  The reference itself is Python under a read-only
source tree that does not exist on the GPU box; this port is what the CPU
baseline times there.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from oracle.packed_ref import TIER_BITS, OracleLayer


def _unpack(words: torch.Tensor, count: int, bits: int) -> torch.Tensor:
    """layout.py:38-46: first ``count`` codes of each packed int32 row."""
    per = 32 // bits
    slots = torch.arange(count)
    gathered = words[..., slots // per].to(torch.int64) & 0xFFFFFFFF
    return (gathered >> ((slots % per) * bits)) & ((1 << bits) - 1)


def dequantize_key(tokens: int, table: dict, packed: dict, group_size: int) -> torch.Tensor:
    """layout.py:132-167 in torch: per tier, per head, codes * scale + min
    (separately rounded) scattered to channel order; the FP16 tier upcast."""
    tier = torch.as_tensor(table["tier"])
    heads, dim = tier.shape
    out = torch.zeros(heads, tokens, dim, dtype=torch.float32)
    groups = torch.arange(tokens) // group_size
    for code, bits in TIER_BITS:
        index = torch.as_tensor(table[code]["index"], dtype=torch.int64)
        count = table[code]["count"]
        block = packed[code]
        for h in range(heads):
            used = int(count[h])
            if used == 0:
                continue
            codes = _unpack(torch.as_tensor(block["code"][h, :tokens]), used, bits).float()
            scale = torch.as_tensor(block["scale"][h, :used]).float()[:, groups].T
            minimum = torch.as_tensor(block["min"][h, :used]).float()[:, groups].T
            out[h][:, index[h, :used]] = codes * scale + minimum
    index = torch.as_tensor(table[3]["index"], dtype=torch.int64)
    for h in range(heads):
        used = int(table[3]["count"][h])
        if used:
            out[h][:, index[h, :used]] = torch.as_tensor(packed[3]["value"][h, :tokens, :used]).float()
    return out


def dequantize_value(packed: dict, tokens: int, dim: int, bits: int, group_size: int) -> torch.Tensor:
    """layout.py:170-182 in torch."""
    codes = _unpack(torch.as_tensor(packed["code"][:, :tokens]), dim, bits).float()
    groups = torch.arange(dim) // group_size
    scale = torch.as_tensor(packed["scale"][:, :tokens]).float()[:, :, groups]
    minimum = torch.as_tensor(packed["min"][:, :tokens]).float()[:, :, groups]
    return codes * scale + minimum


def reference_attention(layer: OracleLayer, query, key_new, value_new, scaling: float) -> torch.Tensor:
    """reference.py:30-56 for one sequence: ``query`` ``[n_q, q_len, D]``,
    ``key_new``/``value_new`` ``[n_kv, q_len, D]`` (fp32) -> fp32
    ``[n_q, q_len, D]``, causal mask aligned to the right edge when q_len > 1
    (reference.py:18-27)."""
    heads, dim = layer.table["tier"].shape
    parts_k, parts_v = [], []
    if layer.hist_len:
        parts_k.append(dequantize_key(layer.hist_len, layer.table, layer.hist_k, layer.k_group_size))
        parts_v.append(dequantize_value(layer.hist_v, layer.hist_len, dim, layer.bit_v, layer.v_group_size))
    if layer.tail_k is not None:
        parts_k.append(torch.as_tensor(layer.tail_k))
        parts_v.append(torch.as_tensor(layer.tail_v))
    parts_k.append(torch.as_tensor(np.asarray(key_new, np.float32)))
    parts_v.append(torch.as_tensor(np.asarray(value_new, np.float32)))
    k = torch.cat(parts_k, dim=1)[None]
    v = torch.cat(parts_v, dim=1)[None]
    q = torch.as_tensor(np.asarray(query, np.float32))[None]
    rep = q.shape[1] // heads
    k = k[:, :, None].expand(1, heads, rep, k.shape[2], dim).reshape(1, heads * rep, k.shape[2], dim)
    v = v[:, :, None].expand(1, heads, rep, v.shape[2], dim).reshape(1, heads * rep, v.shape[2], dim)
    q_len, T = q.shape[2], k.shape[2]
    mask = None
    if q_len > 1:
        pos = torch.arange(T)[None, :]
        last = T - q_len + torch.arange(q_len)[:, None]
        mask = pos <= last
    return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=float(scaling))[0]
