"""Packed decode attention: the reference's ``packed_attention`` call and its
batched form, both running K2 (split-K GQA decode) + K3 (split merge).

Replaces ``src/logitfill/packed/reference.py:59-116``: there is no dense
fallback.  Unsupported cases raise (``NotImplementedError`` for geometry the
kernels do not implement, ``ValueError`` for malformed inputs).
"""
from __future__ import annotations

import ctypes
import math

import torch

from logitfill_b200 import _lib
from logitfill_b200.packed.cache import PackedKVCache, PackedKVManager

MAX_PAGES_PER_SPLIT = 64  # largest work item the tensor-core kernel accepts


def chunk_heads(gq: int, q_len: int) -> int:
    """(q-head, query token) pairs one K2 CTA computes: the largest divisor of
    gq * q_len that is at most 8 (the rule of ``lf_decode.cu:chunk_heads``)."""
    n = gq * q_len
    return next((c for c in range(8, 1, -1) if n % c == 0), 1)


def plan_pages_per_split(pages: int, pairs: int, resid_items: int, sms: int, occupancy) -> int:
    """The planner's cost model, free of the GPU: ``pairs`` (sequence, KV head,
    head chunk) histories of ``pages`` pages each, ``resid_items`` residual
    items in all, ``sms`` SMs and ``occupancy(pps)`` the K2 CTAs per SM (<= 0:
    pps not launchable).  Returns the pps of least (waves of page items) x
    (pps + 1.5), see ``pages_per_split``.  One refinement, when the residual
    items fit beside the page items (a quarter of the slots at most): if all
    full-length items fit in one wave and only the pairs' shorter last items
    overflow, the overflow runs in the slots the first wave's short items free,
    so the cost is max(pps + 1.5, 2 (rem + 1.5)) with rem their length."""
    if pages <= 1:
        return 1
    best, best_cost = 1, None
    for pps in range(1, min(pages, MAX_PAGES_PER_SPLIT) + 1):
        occ = occupancy(pps)
        if occ <= 0:
            continue
        ctas = pairs * (-(-pages // pps))
        resid_fit = 4 * resid_items <= sms * occ
        per_wave = sms * (occ if resid_fit else min(occ, 3))
        waves = max(1, math.ceil(ctas / per_wave - 0.02))
        cost = waves * (pps + 1.5)
        full, rem = pages // pps, pages % pps
        if resid_fit and waves > 1 and rem and pairs * full <= per_wave and ctas - per_wave <= pairs:
            cost = max(pps + 1.5, 2 * (rem + 1.5))
        if best_cost is None or cost < best_cost - 1e-9:
            best, best_cost = pps, cost
    return best


def pages_per_split(cache: PackedKVCache, layer_idx: int = 0, q_len: int = 1) -> int:
    """Pages per K2 work item.  Every (sequence, KV head, head chunk) history
    is cut into ceil(pages / pps) items, plus the short residual items that
    launch after all of them.  An item costs about pps pages plus a fixed
    start (query staging, first copy) worth ~1.5 pages; the choice minimises
    (waves of page items) x (pps + 1.5), i.e. it balances the page items
    over the SMs instead of just making the grid large.  A wave is three page
    items per SM at most (fewer if fewer fit) while the residual items are
    many: measured on B200, a fourth co-resident page item slows the other
    three and takes the slot the residual items would use, so with four
    residual items per pair at 8k histories (B 16) three per SM ran fastest
    (8 pages per item instead of 10: 8 % slower).  When the residual items
    fit in a quarter of the slots, a wave is every slot: they then run on the
    kernel's tail, and at 32k histories (B 8, 4 CTAs per SM) 15 pages per
    item ran 3 % faster than 19.  A wave overfull by up to 2 % still counts
    as one.  Memoised per layer by (pages, q_len)."""
    layer = cache.layers[layer_idx]
    P = cache.page_size
    pages = int(layer.hist_len.max()) // P if layer.hist_len.size else 0
    if pages <= 1:
        return 1
    key = (pages, q_len)
    if key in layer.pps_memo:
        return layer.pps_memo[key]
    so = _lib.lib()
    sms = torch.cuda.get_device_properties(cache.device).multi_processor_count
    gq = cache.n_q // cache.n_kv
    pairs = cache.batch * cache.n_kv * (gq * q_len // chunk_heads(gq, q_len))
    resid_items = pairs * so.lf_decode_max_splits_multi(0, 1, P, q_len)

    def occ_of(pps: int) -> int:
        return so.lf_decode_occupancy(ctypes.byref(layer.layout.c), cache.n_q * q_len, pps)

    best = plan_pages_per_split(pages, pairs, resid_items, sms, occ_of)
    layer.pps_memo[key] = best
    return best


class DecodeCall:
    """Validated arguments of one layer's K2 + K3 launch.  ``query`` is
    ``[B, n_q, D]`` (one token per sequence) or ``[B, n_q, q_len, D]``;
    ``key_new``/``value_new`` ``[B, n_kv, D]`` / ``[B, n_kv, q_len, D]`` or
    None; ``out`` has the query's shape.  ``launch`` enqueues K2 + K3 on the
    current stream; ``launch_partial`` and ``launch_merge`` the two kernels
    separately (one token per sequence only)."""

    def __init__(self, cache: PackedKVCache, layer_idx: int, query: torch.Tensor, key_new, value_new,
                 scaling: float, out: torch.Tensor, pps: int | None = None):
        layer = cache.layers[layer_idx]
        if query.dim() not in (3, 4):
            raise ValueError(f"query must be [B, n_q, D] or [B, n_q, q_len, D], got {tuple(query.shape)}")
        B, n_q, D = query.shape[0], query.shape[1], query.shape[-1]
        q_len = 1 if query.dim() == 3 else query.shape[2]
        if B != cache.batch or n_q != cache.n_q or D != cache.head_dim or q_len < 1:
            raise ValueError(f"query {tuple(query.shape)} does not match the cache "
                             f"[{cache.batch}, {cache.n_q}, q_len, {cache.head_dim}]")
        if not query.is_cuda:
            raise RuntimeError("packed attention needs CUDA tensors (no CPU fallback)")
        if out.shape != query.shape:
            raise ValueError(f"out must be {tuple(query.shape)}, got {tuple(out.shape)}")
        if query.stride(-1) != 1 or out.stride(-1) != 1:
            raise ValueError("channel stride must be 1")
        resid_dtype = layer.tail_k.dtype if layer.tail_k is not None else (
            key_new.dtype if key_new is not None else torch.bfloat16)
        layer.ensure_residual(resid_dtype)
        if key_new is not None:
            want = (B, cache.n_kv, D) if query.dim() == 3 else (B, cache.n_kv, q_len, D)
            if tuple(key_new.shape) != want or value_new.shape != key_new.shape:
                raise ValueError(f"new Key/Value must be {list(want)}")
            key_new = key_new.to(resid_dtype)
            value_new = value_new.to(resid_dtype)
            if key_new.stride() != value_new.stride() or key_new.stride(-1) != 1:
                key_new, value_new = key_new.contiguous(), value_new.contiguous()
        self.cache, self.layer = cache, layer
        self.query, self.key_new, self.value_new, self.out = query, key_new, value_new, out
        self.q_len = q_len
        self.scaling = float(scaling)
        self.resid_dtype = resid_dtype
        self.pps = pages_per_split(cache, layer_idx, q_len) if pps is None else int(pps)
        self.max_splits = _lib.lib().lf_decode_max_splits_multi(cache.row_cap // cache.page_size, self.pps,
                                                                cache.page_size, q_len)
        self.ws = cache.workspace(self.max_splits, q_len)

    def launch_partial(self) -> None:
        so, L, c = _lib.lib(), self.layer, self.cache
        tk, kn = L.tail_k, self.key_new
        _lib.check(so.lf_decode_partial(
            ctypes.byref(L.layout.c), _lib.ptr(L.rows), _lib.ptr(L.kmeta), _lib.ptr(L.layout.slot_chan),
            _lib.ptr(L.dev_hist), _lib.ptr(tk), _lib.ptr(L.tail_v), tk.stride(0), tk.stride(1),
            _lib.ptr(L.dev_tail), _lib.dtype_code(self.resid_dtype), _lib.ptr(kn), _lib.ptr(self.value_new),
            kn.stride(0) if kn is not None else 0, kn.stride(1) if kn is not None else 0,
            _lib.ptr(self.query), _lib.dtype_code(self.query.dtype), self.query.stride(0), self.query.stride(1),
            c.batch, c.n_q, self.scaling, self.pps, self.max_splits, _lib.ptr(self.ws), _lib.ptr(c.status),
            _lib.stream_handle(self.query.device)), "lf_decode_partial")

    def launch(self) -> None:
        """K2 then K3 in one library call (lf_decode / lf_decode_multi) on the current stream."""
        if self.query.dim() == 4:
            self._launch_multi()
            return
        so, L, c, out = _lib.lib(), self.layer, self.cache, self.out
        tk, kn = L.tail_k, self.key_new
        _lib.check(so.lf_decode(
            ctypes.byref(L.layout.c), _lib.ptr(L.rows), _lib.ptr(L.kmeta), _lib.ptr(L.layout.slot_chan),
            _lib.ptr(L.dev_hist), _lib.ptr(tk), _lib.ptr(L.tail_v), tk.stride(0), tk.stride(1),
            _lib.ptr(L.dev_tail), _lib.dtype_code(self.resid_dtype), _lib.ptr(kn), _lib.ptr(self.value_new),
            kn.stride(0) if kn is not None else 0, kn.stride(1) if kn is not None else 0,
            _lib.ptr(self.query), _lib.dtype_code(self.query.dtype), self.query.stride(0), self.query.stride(1),
            c.batch, c.n_q, self.scaling, self.pps, self.max_splits, _lib.ptr(self.ws), _lib.ptr(out),
            _lib.dtype_code(out.dtype), out.stride(0), out.stride(1), _lib.ptr(c.status),
            _lib.stream_handle(self.query.device)), "lf_decode")

    def _launch_multi(self) -> None:
        so, L, c, out, q = _lib.lib(), self.layer, self.cache, self.out, self.query
        tk, kn = L.tail_k, self.key_new
        _lib.check(so.lf_decode_multi(
            ctypes.byref(L.layout.c), _lib.ptr(L.rows), _lib.ptr(L.kmeta), _lib.ptr(L.layout.slot_chan),
            _lib.ptr(L.dev_hist), _lib.ptr(tk), _lib.ptr(L.tail_v), tk.stride(0), tk.stride(1),
            _lib.ptr(L.dev_tail), _lib.dtype_code(self.resid_dtype), _lib.ptr(kn), _lib.ptr(self.value_new),
            kn.stride(0) if kn is not None else 0, kn.stride(1) if kn is not None else 0,
            kn.stride(2) if kn is not None else 0,
            _lib.ptr(q), _lib.dtype_code(q.dtype), q.stride(0), q.stride(1), q.stride(2), self.q_len,
            c.batch, c.n_q, self.scaling, self.pps, self.max_splits, _lib.ptr(self.ws), _lib.ptr(out),
            _lib.dtype_code(out.dtype), out.stride(0), out.stride(1), out.stride(2), _lib.ptr(c.status),
            _lib.stream_handle(q.device)), "lf_decode_multi")

    def launch_merge(self) -> None:
        so, c, out = _lib.lib(), self.cache, self.out
        _lib.check(so.lf_decode_merge(
            _lib.ptr(self.ws), _lib.ptr(self.layer.dev_hist), c.batch, c.n_kv, c.n_q, c.head_dim, c.page_size,
            self.pps, self.max_splits, _lib.ptr(out), _lib.dtype_code(out.dtype), out.stride(0), out.stride(1),
            _lib.stream_handle(out.device)), "lf_decode_merge")


def decode_into(cache: PackedKVCache, layer_idx: int, query: torch.Tensor, key_new, value_new,
                scaling: float, out: torch.Tensor, pps: int | None = None) -> torch.Tensor:
    """Attention of ``query`` ``[B, n_q, D]`` over each sequence's packed
    history, residual page and (optionally) the new token ``[B, n_kv, D]``,
    written to ``out`` ``[B, n_q, D]``.  Launches K2 then K3 on the current stream."""
    call = DecodeCall(cache, layer_idx, query, key_new, value_new, scaling, out, pps)
    call.launch()
    return out


def packed_attention_batched(cache: PackedKVCache, layer_idx: int, query: torch.Tensor,
                             key_new: torch.Tensor | None, value_new: torch.Tensor | None,
                             scaling: float, out_dtype=None) -> torch.Tensor:
    """Batched attention over the packed caches: ``query`` ``[B, n_q, D]``
    with ``key_new``/``value_new`` ``[B, n_kv, D]`` (a decode step), or
    ``query`` ``[B, n_q, q_len, D]`` with ``[B, n_kv, q_len, D]`` (query token
    i sees new tokens 0..i) -> the query's shape in ``out_dtype`` (default
    ``query.dtype``)."""
    out = torch.empty(query.shape, dtype=out_dtype or query.dtype, device=query.device)
    return decode_into(cache, layer_idx, query, key_new, value_new, scaling, out)


def packed_attention(manager: PackedKVManager, layer_idx: int, query: torch.Tensor,
                     key_new: torch.Tensor, value_new: torch.Tensor, scaling: float) -> torch.Tensor:
    """reference.py:112-116: ``query`` ``[1, n_q, q_len, D]``,
    ``key_new``/``value_new`` ``[1, n_kv, q_len, D]`` -> ``[1, n_q, q_len, D]`` in
    ``query.dtype``.  Attends over the packed history, the residual tail and
    the new tokens with the right-aligned causal mask (reference.py:18-56),
    accumulating in fp32.  q_len 1 is a decode step; a longer call (chunked
    prefill after the first) runs the same kernels, which the reference
    leaves to its dense path."""
    if query.dim() != 4 or query.shape[0] != 1:
        raise NotImplementedError("packed attention supports batch size 1 per manager")
    if manager.bit_v != 2:
        raise NotImplementedError("packed decode needs bit_v == 2")
    q_len = query.shape[2]
    if q_len == 1:
        out = torch.empty(1, manager.n_q, manager.head_dim, dtype=torch.float32, device=query.device)
        decode_into(manager.cache, layer_idx, query[:, :, 0], key_new[:, :, 0], value_new[:, :, 0], scaling, out)
        return out.to(query.dtype).view(1, manager.n_q, 1, manager.head_dim)
    out = torch.empty(query.shape, dtype=torch.float32, device=query.device)
    decode_into(manager.cache, layer_idx, query, key_new, value_new, scaling, out)
    return out.to(query.dtype)
