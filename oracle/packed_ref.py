"""CPU oracle for the LogitFill packed-cache hot path (numpy restatement).

TEST INFRASTRUCTURE ONLY.  This module is the checker the CUDA path is compared
against; it is imported by ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` and by nothing
else.  The product package ``logitfill_b200`` never imports it and has no CPU
fallback.

It restates, in numpy, the reference's packed layout codec and its dense
packed-attention path.  Every function names the reference lines it follows
(paths relative to the GASSFY/Logitfill project root):

* ``src/logitfill/packed/layout.py``      -- codec (codes, packing, tier tables,
  page quantizers, dequantizers)
* ``src/logitfill/packed/cache.py``       -- page-delayed history store
* ``src/logitfill/packed/reference.py``   -- dense attention over the history

Arithmetic follows the reference bit for bit where it is integer or IEEE
single precision: fp32 subtraction and division, round-half-to-even,
fp32->fp16 round-to-nearest-even, separate multiply and add in dequantization
(no fused multiply-add).  Attention is evaluated in float64 from the fp32
dequantized history; the reference evaluates it in fp32, the two agree to
~1e-6, far inside the 2e-3 parity tolerance.

Parity is pinned against the reference itself: ``tests/golden/make_golden.py``
runs the reference packer and attention on seeded inputs and stores the
results in ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this
module against them.
"""
from __future__ import annotations

import numpy as np

TIER_BITS = ((0, 2), (1, 4), (2, 8))  # layout.py:78 -- (level code, bits)


# ---------------------------------------------------------------- codec ----
def asymmetric_codes(grouped: np.ndarray, bits: int):
    """layout.py:12-18.  ``grouped`` is fp32 ``[..., group]``.

    scale = clamp((max - min) / (2^b - 1), 1e-5, 1e5) in fp32 (IEEE divide);
    codes = clamp(rint((x - min) / scale), 0, 2^b - 1) using the fp32 scale.
    """
    g = np.asarray(grouped, dtype=np.float32)
    high = g.max(axis=-1, keepdims=True)
    low = g.min(axis=-1, keepdims=True)
    qmax = np.float32((1 << bits) - 1)
    scale = np.clip((high - low) / qmax, np.float32(1e-5), np.float32(1e5)).astype(np.float32)
    codes = np.clip(np.rint((g - low) / scale), 0, (1 << bits) - 1).astype(np.int32)
    return codes, scale[..., 0], low[..., 0]


def pack_ints(codes: np.ndarray, bits: int) -> np.ndarray:
    """layout.py:21-35.  Pads the last axis to a multiple of 32/bits with 0 and
    ORs ``code << (slot * bits)`` into int32 words, slot 0 in the low bits."""
    codes = np.asarray(codes, dtype=np.int64)
    if codes.shape[-1] == 0:
        return np.zeros(codes.shape[:-1] + (0,), dtype=np.int32)
    per = 32 // int(bits)
    pad = (-codes.shape[-1]) % per
    if pad:
        codes = np.concatenate([codes, np.zeros(codes.shape[:-1] + (pad,), np.int64)], axis=-1)
    view = codes.reshape(codes.shape[:-1] + (codes.shape[-1] // per, per))
    packed = np.zeros(view.shape[:-1], dtype=np.uint64)
    for slot in range(per):
        packed |= view[..., slot].astype(np.uint64) << np.uint64(slot * bits)
    return (packed & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.int32)


def unpack_ints(packed: np.ndarray, count: int, bits: int) -> np.ndarray:
    """layout.py:38-46.  First ``count`` codes of each packed row."""
    packed = np.asarray(packed, dtype=np.int32)
    if count == 0:
        return np.zeros(packed.shape[:-1] + (0,), dtype=np.int32)
    per = 32 // int(bits)
    slots = np.arange(count)
    words = packed.view(np.uint32)[..., slots // per]
    return ((words >> ((slots % per) * bits).astype(np.uint32)) & np.uint32((1 << bits) - 1)).astype(np.int32)


def tier_tables(levels: np.ndarray) -> dict:
    """layout.py:49-68.  Per tier: ascending channel ``index`` padded to the
    tier ``width`` (max count over heads), ``count`` per head, ``local``
    position of each channel inside its tier (-1 elsewhere); ``tier`` = levels."""
    levels = np.asarray(levels, dtype=np.int64)
    heads, dim = levels.shape
    tiers = {}
    for code in (0, 1, 2, 3):
        rows = [np.nonzero(levels[h] == code)[0] for h in range(heads)]
        width = max((len(r) for r in rows), default=0)
        index = np.zeros((heads, width), dtype=np.int32)
        count = np.zeros(heads, dtype=np.int32)
        local = np.full((heads, dim), -1, dtype=np.int32)
        for h, row in enumerate(rows):
            count[h] = len(row)
            index[h, : len(row)] = row
            local[h, row] = np.arange(len(row), dtype=np.int32)
        tiers[code] = {"index": index, "count": count, "local": local, "width": width}
    tiers["tier"] = levels.astype(np.int32)
    return tiers


def quantize_key_page(page: np.ndarray, table: dict, group_size: int) -> dict:
    """layout.py:71-112.  ``page`` fp32 ``[heads, tokens, dim]``.

    INT2/4/8 tiers: per head, the tier's channels are grouped along tokens,
    quantized, padded to the tier width with code 0 and packed along channels;
    scale/min are fp16 ``[heads, width, groups]`` initialised to 1.0 / 0.0.
    FP16 tier: the channels gathered and rounded to fp16."""
    page = np.asarray(page, dtype=np.float32)
    heads, tokens, _ = page.shape
    if tokens % group_size:
        raise ValueError(f"Key page length {tokens} is not a multiple of {group_size}")
    groups = tokens // group_size
    out = {}
    for code, bits in TIER_BITS:
        index, count, width = table[code]["index"], table[code]["count"], int(table[code]["width"])
        per = 32 // bits
        words = (width + per - 1) // per if width else 0
        code_out = np.zeros((heads, tokens, words), dtype=np.int32)
        scale = np.ones((heads, width, groups), dtype=np.float16)
        minimum = np.zeros((heads, width, groups), dtype=np.float16)
        for h in range(heads):
            used = int(count[h])
            if used == 0:
                continue
            channels = index[h, :used]
            grouped = page[h][:, channels].T.reshape(used, groups, group_size)
            codes, sc, low = asymmetric_codes(grouped, bits)
            padded = np.zeros((tokens, width), dtype=np.int32)
            padded[:, :used] = codes.reshape(used, tokens).T
            code_out[h] = pack_ints(padded, bits)
            scale[h, :used] = sc.astype(np.float16)
            minimum[h, :used] = low.astype(np.float16)
        out[code] = {"code": code_out, "scale": scale, "min": minimum}
    index, count, width = table[3]["index"], table[3]["count"], int(table[3]["width"])
    values = np.zeros((heads, tokens, width), dtype=np.float16)
    for h in range(heads):
        used = int(count[h])
        if used:
            with np.errstate(over="ignore"):  # values beyond fp16 range become inf, as in torch
                values[h, :, :used] = page[h][:, index[h, :used]].astype(np.float16)
    out[3] = {"value": values}
    return out


def quantize_value_page(page: np.ndarray, bits: int, group_size: int) -> dict:
    """layout.py:115-129.  Per-token groups of ``group_size`` channels."""
    page = np.asarray(page, dtype=np.float32)
    heads, tokens, dim = page.shape
    if bits >= 16:
        return {"value": page.astype(np.float16)}
    if dim % group_size:
        raise ValueError(f"head dim {dim} is not divisible by value group {group_size}")
    grouped = page.reshape(heads, tokens, dim // group_size, group_size)
    codes, scale, low = asymmetric_codes(grouped, bits)
    return {
        "code": pack_ints(codes.reshape(heads, tokens, dim), bits),
        "scale": scale.astype(np.float16),
        "min": low.astype(np.float16),
    }


def dequantize_key(tokens: int, table: dict, packed: dict, group_size: int) -> np.ndarray:
    """layout.py:132-167.  ``code * scale + min`` in fp32 as a separately
    rounded multiply and add, scattered back to channel order."""
    tier = table["tier"]
    heads, dim = tier.shape
    out = np.zeros((heads, tokens, dim), dtype=np.float32)
    if tokens == 0:
        return out
    groups = np.arange(tokens) // group_size
    for code, bits in TIER_BITS:
        index, count, block = table[code]["index"], table[code]["count"], packed[code]
        for h in range(heads):
            used = int(count[h])
            if used == 0:
                continue
            codes = unpack_ints(block["code"][h, :tokens], used, bits).astype(np.float32)
            scale = block["scale"][h, :used].astype(np.float32)[:, groups].T
            minimum = block["min"][h, :used].astype(np.float32)[:, groups].T
            prod = (codes * scale).astype(np.float32)
            out[h][:, index[h, :used]] = (prod + minimum).astype(np.float32)
    index, count = table[3]["index"], table[3]["count"]
    for h in range(heads):
        used = int(count[h])
        if used:
            out[h][:, index[h, :used]] = packed[3]["value"][h, :tokens, :used].astype(np.float32)
    return out


def dequantize_value(packed: dict, tokens: int, dim: int, bits: int, group_size: int) -> np.ndarray:
    """layout.py:170-182."""
    if bits >= 16:
        return packed["value"][:, :tokens].astype(np.float32)
    heads = packed["code"].shape[0]
    if tokens == 0:
        return np.zeros((heads, 0, dim), dtype=np.float32)
    codes = unpack_ints(packed["code"][:, :tokens], dim, bits).astype(np.float32)
    groups = np.arange(dim) // group_size
    scale = packed["scale"][:, :tokens].astype(np.float32)[:, :, groups]
    minimum = packed["min"][:, :tokens].astype(np.float32)[:, :, groups]
    return ((codes * scale).astype(np.float32) + minimum).astype(np.float32)


# ---------------------------------------------------------------- store ----
class OracleLayer:
    """cache.py:16-90 (``_LayerStore``): original-dtype tail, page flushes
    packed and concatenated onto the history after attention."""

    def __init__(self, levels, page_size: int, k_group_size: int, v_group_size: int, bit_v: int):
        self.page_size, self.k_group_size = int(page_size), int(k_group_size)
        self.v_group_size, self.bit_v = int(v_group_size), int(bit_v)
        self.table = tier_tables(levels)
        self.hist_k = None
        self.hist_v = None
        self.hist_len = 0
        self.tail_k = None  # fp32 [H, n, D] (exact upcast of the caller's dtype)
        self.tail_v = None

    @property
    def tail_len(self) -> int:
        return 0 if self.tail_k is None else int(self.tail_k.shape[1])

    @property
    def length(self) -> int:
        return self.hist_len + self.tail_len

    def append(self, key: np.ndarray, value: np.ndarray) -> None:
        """cache.py:48-62."""
        key = np.asarray(key, np.float32)
        value = np.asarray(value, np.float32)
        self.tail_k = key if self.tail_k is None else np.concatenate([self.tail_k, key], axis=1)
        self.tail_v = value if self.tail_v is None else np.concatenate([self.tail_v, value], axis=1)
        while self.tail_len >= self.page_size:
            pk, pv = self.tail_k[:, : self.page_size], self.tail_v[:, : self.page_size]
            self.tail_k, self.tail_v = self.tail_k[:, self.page_size :], self.tail_v[:, self.page_size :]
            if self.tail_k.shape[1] == 0:
                self.tail_k = self.tail_v = None
            self._flush(pk, pv)

    def _flush(self, key, value) -> None:
        """cache.py:64-81."""
        pk = quantize_key_page(key, self.table, self.k_group_size)
        pv = quantize_value_page(value, self.bit_v, self.v_group_size)
        if self.hist_k is None:
            self.hist_k, self.hist_v = pk, pv
        else:
            for code in (0, 1, 2):
                h = self.hist_k[code]
                h["code"] = np.concatenate([h["code"], pk[code]["code"]], axis=1)
                h["scale"] = np.concatenate([h["scale"], pk[code]["scale"]], axis=2)
                h["min"] = np.concatenate([h["min"], pk[code]["min"]], axis=2)
            self.hist_k[3]["value"] = np.concatenate([self.hist_k[3]["value"], pk[3]["value"]], axis=1)
            for name in self.hist_v:
                self.hist_v[name] = np.concatenate([self.hist_v[name], pv[name]], axis=1)
        self.hist_len += int(key.shape[1])

    def dequantize(self):
        """cache.py:83-90."""
        heads, dim = self.table["tier"].shape
        if self.hist_k is None:
            empty = np.zeros((heads, 0, dim), np.float32)
            return empty, empty
        k = dequantize_key(self.hist_len, self.table, self.hist_k, self.k_group_size)
        v = dequantize_value(self.hist_v, self.hist_len, dim, self.bit_v, self.v_group_size)
        return k, v


# ------------------------------------------------------------ attention ----
def attention_over(key: np.ndarray, value: np.ndarray, query: np.ndarray, scaling: float) -> np.ndarray:
    """Softmax attention of ``query`` ``[n_q, q_len, D]`` over ``key``/``value``
    ``[n_kv, T, D]`` with GQA repeat (reference.py:10-15,45-47), causal mask
    aligned to the right edge when q_len > 1 (reference.py:18-27).  float64."""
    n_kv, T, D = key.shape
    n_q, q_len, _ = query.shape
    rep = n_q // n_kv
    # q-head h*rep + j reads KV head h: the repeat_kv expansion as a grouped product.
    qg = query.astype(np.float64).reshape(n_kv, rep, q_len, D).reshape(n_kv, rep * q_len, D)
    k = key.astype(np.float64)
    v = value.astype(np.float64)
    s = (qg @ k.transpose(0, 2, 1)).reshape(n_kv, rep, q_len, T) * float(scaling)
    if q_len > 1:
        for i in range(q_len):
            visible = T - q_len + i + 1
            s[:, :, i, visible:] = -np.inf
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    out = p.reshape(n_kv, rep * q_len, T) @ v
    return out.reshape(n_kv, rep, q_len, D).reshape(n_q, q_len, D)


def reference_attention(layer: OracleLayer, query: np.ndarray, key_new: np.ndarray,
                        value_new: np.ndarray, scaling: float) -> np.ndarray:
    """reference.py:30-56 for one sequence.  ``query`` ``[n_q, q_len, D]``,
    ``key_new``/``value_new`` ``[n_kv, q_len, D]``; history dequantized
    (cache.py:83-90), tail and new tokens appended in fp32.  Returns float64
    ``[n_q, q_len, D]``."""
    kh, vh = layer.dequantize()
    ks, vs = [kh], [vh]
    if layer.tail_k is not None:
        ks.append(layer.tail_k)
        vs.append(layer.tail_v)
    ks.append(np.asarray(key_new, np.float32))
    vs.append(np.asarray(value_new, np.float32))
    return attention_over(np.concatenate(ks, axis=1), np.concatenate(vs, axis=1), query, scaling)


# -------------------------------------------------------------- helpers ----
def bf16_to_f32(bits_u16: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns (uint16) to float32, exactly."""
    return (np.asarray(bits_u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 to bfloat16 bit patterns, round-to-nearest-even (finite inputs)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)
