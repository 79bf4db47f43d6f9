"""Packed decode attention: the reference's ``packed_attention`` call and its
batched form, both running K2 (split-K GQA decode) + K3 (split merge).

Replaces ``src/logitfill/packed/reference.py:59-116``: there is no dense
fallback.  Unsupported cases raise (``NotImplementedError`` for geometry the
kernels do not implement, ``ValueError`` for malformed inputs).
"""
from __future__ import annotations

import ctypes

import torch

from logitfill_b200 import _lib
from logitfill_b200.packed.cache import PackedKVCache, PackedKVManager

MAX_PAGES_PER_SPLIT = 64  # largest work item the tensor-core kernel accepts


def pages_per_split(cache: PackedKVCache, layer_idx: int = 0) -> int:
    """Pages per K2 work item.  Every (sequence, KV head) history is cut into
    ceil(pages / pps) items, plus up to ceil(page/32) short residual items
    that launch after all of them.  An item costs about pps pages plus a fixed
    start (query staging, first copy) worth ~1.5 pages; the choice minimises
    (waves of resident CTAs) x (pps + 1.5), i.e. it balances the page items
    over the SMs instead of just making the grid large."""
    layer = cache.layers[layer_idx]
    P = cache.page_size
    pages = int(layer.hist_len.max()) // P if layer.hist_len.size else 0
    if pages <= 1:
        return 1
    so = _lib.lib()
    sms = torch.cuda.get_device_properties(cache.device).multi_processor_count
    pairs = cache.batch * cache.n_kv
    best, best_cost = 1, None
    for pps in range(1, min(pages, MAX_PAGES_PER_SPLIT) + 1):
        occ = so.lf_decode_occupancy(ctypes.byref(layer.layout.c), cache.n_q, pps)
        if occ <= 0:
            continue
        ctas = pairs * (-(-pages // pps))
        waves = -(-ctas // (sms * occ))
        cost = waves * (pps + 1.5)
        if best_cost is None or cost < best_cost - 1e-9:
            best, best_cost = pps, cost
    return best


class DecodeCall:
    """Validated arguments of one layer's K2 + K3 launch.  ``launch_partial``
    and ``launch_merge`` enqueue the two kernels on the current stream."""

    def __init__(self, cache: PackedKVCache, layer_idx: int, query: torch.Tensor, key_new, value_new,
                 scaling: float, out: torch.Tensor, pps: int | None = None):
        layer = cache.layers[layer_idx]
        B, n_q, D = query.shape
        if B != cache.batch or n_q != cache.n_q or D != cache.head_dim:
            raise ValueError(f"query {tuple(query.shape)} does not match the cache "
                             f"[{cache.batch}, {cache.n_q}, {cache.head_dim}]")
        if not query.is_cuda:
            raise RuntimeError("packed attention needs CUDA tensors (no CPU fallback)")
        if out.shape != query.shape:
            raise ValueError(f"out must be {tuple(query.shape)}, got {tuple(out.shape)}")
        if query.stride(2) != 1 or out.stride(2) != 1:
            raise ValueError("channel stride must be 1")
        resid_dtype = layer.tail_k.dtype if layer.tail_k is not None else (
            key_new.dtype if key_new is not None else torch.bfloat16)
        layer.ensure_residual(resid_dtype)
        if key_new is not None:
            if key_new.shape != (B, cache.n_kv, D) or value_new.shape != key_new.shape:
                raise ValueError(f"new token Key/Value must be [{B}, {cache.n_kv}, {D}]")
            key_new = key_new.to(resid_dtype)
            value_new = value_new.to(resid_dtype)
            if key_new.stride() != value_new.stride() or key_new.stride(2) != 1:
                key_new, value_new = key_new.contiguous(), value_new.contiguous()
        self.cache, self.layer = cache, layer
        self.query, self.key_new, self.value_new, self.out = query, key_new, value_new, out
        self.scaling = float(scaling)
        self.resid_dtype = resid_dtype
        self.pps = pages_per_split(cache, layer_idx) if pps is None else int(pps)
        self.max_splits = _lib.lib().lf_decode_max_splits(cache.row_cap // cache.page_size, self.pps, cache.page_size)
        self.ws = cache.workspace(self.max_splits)

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
        """K2 then K3 in one library call (lf_decode) on the current stream."""
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
    """Batched decode: ``query`` ``[B, n_q, D]`` (or ``[B, n_q, 1, D]``),
    ``key_new``/``value_new`` ``[B, n_kv, D]`` (or ``[B, n_kv, 1, D]``) ->
    ``[B, n_q, D]`` in ``out_dtype`` (default ``query.dtype``)."""
    if query.dim() == 4:
        if query.shape[2] != 1:
            raise NotImplementedError("packed decode handles one query token per sequence")
        query = query[:, :, 0]
    if key_new is not None and key_new.dim() == 4:
        key_new, value_new = key_new[:, :, 0], value_new[:, :, 0]
    out = torch.empty(query.shape, dtype=out_dtype or query.dtype, device=query.device)
    return decode_into(cache, layer_idx, query, key_new, value_new, scaling, out)


def packed_attention(manager: PackedKVManager, layer_idx: int, query: torch.Tensor,
                     key_new: torch.Tensor, value_new: torch.Tensor, scaling: float) -> torch.Tensor:
    """reference.py:112-116: ``query`` ``[1, n_q, 1, D]``, ``key_new``/``value_new``
    ``[1, n_kv, 1, D]`` -> ``[1, n_q, 1, D]`` in ``query.dtype``.  Attends over
    the packed history, the residual tail and the new token (reference.py:30-56),
    accumulating in fp32."""
    if query.dim() != 4 or query.shape[0] != 1:
        raise NotImplementedError("packed attention supports batch size 1 per manager")
    if query.shape[2] != 1:
        raise NotImplementedError(
            "packed decode handles q_len == 1; prefill runs dense attention (qwen2_attention.py:240-243)")
    if manager.bit_v != 2:
        raise NotImplementedError("packed decode needs bit_v == 2")
    out = torch.empty(1, manager.n_q, manager.head_dim, dtype=torch.float32, device=query.device)
    decode_into(manager.cache, layer_idx, query[:, :, 0], key_new[:, :, 0], value_new[:, :, 0], scaling, out)
    return out.to(query.dtype).view(1, manager.n_q, 1, manager.head_dim)
