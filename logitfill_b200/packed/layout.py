"""Packed layout: tier tables, the B200 history layout and reference views.

Mirrors ``src/logitfill/packed/layout.py`` of the reference.  The channel
tables (:func:`tier_tables`, layout.py:49-68) are built once per level map
and device, with vectorised torch, by :class:`logitfill_b200.policy.TierTables`
and shared by every layer and cache that uses the map.  Storage differs: instead of per-tier tensors
concatenated on every flush (cache.py:64-81), one layer keeps two
preallocated buffers per batch,

* ``rows``  int32 ``[B, H, row_cap, row_words]`` -- per token: INT2 | INT4 |
  INT8 Key codes, Value codes, then fp16 FP16-tier Key, Value scale, Value min;
* ``kmeta`` fp16  ``[B, H, group_cap, meta_halves]`` -- per Key group: scale
  and min of each INT2/INT4/INT8 tier channel, then the group's largest
  scale (the decoder's fixed-point exponent for the page);

and every reference array is a strided view of them (:meth:`LayerLayout.hist_k_views`),
so a sequence's history has the reference's shapes and bytes with no copy.
``quantize_key_page`` / ``quantize_value_page`` keep the reference signatures
and run the K1 CUDA kernel.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from logitfill_b200 import _lib
from logitfill_b200.policy import TierTables

TIER_BITS = ((0, 2), (1, 4), (2, 8))


def tier_tables(levels: torch.Tensor) -> dict:
    """layout.py:49-68: per tier ``index`` (channels ascending, padded to the
    tier ``width``), ``count`` per head, ``local`` position of each channel in
    its tier (-1 elsewhere); ``tier`` = the levels as int32.  Built by the
    shared :class:`~logitfill_b200.policy.TierTables` on the levels' device."""
    lv = torch.as_tensor(levels)
    tt = TierTables.get(lv.detach().cpu(), lv.device)
    return {"tiers": {t: dict(tt.table[t]) for t in range(4)}, "tier": tt.table["tier"]}


class LayerLayout:
    """History layout of one layer plus its device channel tables (shared,
    per level map and device, through :class:`~logitfill_b200.policy.TierTables`)."""

    def __init__(self, levels, *, head_dim: int, page_size: int, k_group_size: int,
                 v_group_size: int, bit_v: int, row_cap: int, device):
        self.device = torch.device(device)
        lv = torch.as_tensor(levels, dtype=torch.int64)
        if lv.dim() != 2 or lv.shape[1] != head_dim:
            raise ValueError(f"levels must be [n_kv, {head_dim}], got {tuple(lv.shape)}")
        tables = TierTables.get(lv.cpu(), self.device)
        self.tables = tables
        self.levels = tables.levels
        self.kv_heads = int(lv.shape[0])
        self.head_dim = int(head_dim)
        self.page_size = int(page_size)
        self.k_group_size = int(k_group_size)
        self.v_group_size = int(v_group_size)
        self.bit_v = int(bit_v)
        self._counts = tables.counts
        self.c = _lib.LfLayout()
        self.set_capacity(row_cap)
        self.chan_code = tables.chan_code
        self.slot_chan = tables.slot_chan
        # Reference-shaped tables (layout.py:49-68 + cache.py:22-24).
        self.table = tables.table

    def set_capacity(self, row_cap: int) -> None:
        if row_cap % self.page_size:
            raise ValueError("row capacity must be a multiple of page_size")
        group_cap = row_cap // self.k_group_size
        _lib.check(_lib.lib().lf_layout_init(
            ctypes.byref(self.c), self.kv_heads, self.head_dim, self.page_size, self.k_group_size,
            self.v_group_size, self.bit_v, self._counts.ctypes.data, row_cap, group_cap), "lf_layout_init")

    # ---- geometry --------------------------------------------------------
    @property
    def row_cap(self) -> int:
        return int(self.c.row_cap)

    @property
    def group_cap(self) -> int:
        return int(self.c.group_cap)

    @property
    def row_words(self) -> int:
        return int(self.c.row_words)

    @property
    def meta_halves(self) -> int:
        return int(self.c.meta_halves)

    def width(self, code: int) -> int:
        return int(self.c.width[code])

    def words(self, code: int) -> int:
        return int(self.c.words[code])

    def alloc(self, batch: int):
        """Zeroed ``rows`` and ``kmeta`` buffers for ``batch`` sequences."""
        rows = torch.zeros(batch, self.kv_heads, self.row_cap, self.row_words, dtype=torch.int32,
                           device=self.device)
        kmeta = torch.zeros(batch, self.kv_heads, self.group_cap, max(self.meta_halves, 8),
                            dtype=torch.float16, device=self.device)
        return rows, kmeta

    # ---- reference-shaped views (layout.py:71-129 / cache.py:64-81) -----
    def hist_k_views(self, rows_b: torch.Tensor, kmeta_b: torch.Tensor, tokens: int) -> dict:
        """``rows_b`` ``[H, row_cap, R]``, ``kmeta_b`` ``[H, group_cap, M]`` of one
        sequence -> the reference's ``hist_k`` dict for ``tokens`` history tokens."""
        groups = tokens // self.k_group_size
        L = self.c
        out = {}
        for code in (0, 1, 2):
            o, n, w = int(L.code_off[code]), int(L.words[code]), int(L.width[code])
            so, mo = int(L.scale_off[code]), int(L.min_off[code])
            out[code] = {
                "code": rows_b[:, :tokens, o:o + n],
                "scale": kmeta_b[:, :groups, so:so + w].transpose(1, 2),
                "min": kmeta_b[:, :groups, mo:mo + w].transpose(1, 2),
            }
        r16 = rows_b.view(torch.float16)
        h0 = 2 * int(L.half_off)
        out[3] = {"value": r16[:, :tokens, h0:h0 + int(L.width[3])]}
        return out

    def hist_v_views(self, rows_b: torch.Tensor, tokens: int) -> dict:
        L = self.c
        nv = self.head_dim // self.v_group_size
        r16 = rows_b.view(torch.float16)
        h0 = 2 * int(L.half_off) + int(L.width[3])
        vo, vw = int(L.vcode_off), int(L.vcode_words)
        return {
            "code": rows_b[:, :tokens, vo:vo + vw],
            "scale": r16[:, :tokens, h0:h0 + nv],
            "min": r16[:, :tokens, h0 + nv:h0 + 2 * nv],
        }


# ---------------------------------------------------------------- K1 -------
def pack_pages(layout: LayerLayout, rows: torch.Tensor, kmeta: torch.Tensor, key: torch.Tensor,
               value: torch.Tensor, jobs, *, status: torch.Tensor | None = None) -> None:
    """Quantize and pack pages of ``key``/``value`` ``[S, H, T, D]`` into the
    history buffers.  ``jobs`` rows are (src_seq, src_token0, dst_seq, dst_page)."""
    if not key.is_cuda:
        raise RuntimeError("pack_pages needs CUDA tensors (the packed backend has no CPU path)")
    if key.shape != value.shape or key.dtype != value.dtype or key.stride() != value.stride():
        raise ValueError("key and value pages must match in shape, dtype and strides")
    if key.dim() != 4 or key.shape[1] != layout.kv_heads or key.shape[3] != layout.head_dim:
        raise ValueError(f"expected [S, {layout.kv_heads}, T, {layout.head_dim}], got {tuple(key.shape)}")
    if key.stride(3) != 1:
        raise ValueError("channel stride must be 1")
    jobs_np = np.asarray(jobs, dtype=np.int32).reshape(-1, 4)
    if jobs_np.shape[0] == 0:
        return
    P = layout.page_size
    S, _, T, _ = key.shape
    B = rows.shape[0]
    if (jobs_np[:, 0] < 0).any() or (jobs_np[:, 0] >= S).any() or (jobs_np[:, 1] < 0).any() \
            or (jobs_np[:, 1] + P > T).any():
        raise ValueError("pack job reads outside the source")
    if (jobs_np[:, 2] < 0).any() or (jobs_np[:, 2] >= B).any() or (jobs_np[:, 3] < 0).any() \
            or ((jobs_np[:, 3] + 1) * P > layout.row_cap).any():
        raise ValueError("pack job writes outside the history capacity")
    # Pinned, non-blocking upload: the host does not wait for the kernels
    # already queued (the pinned block is not reused before the copy ends).
    jobs_dev = torch.from_numpy(jobs_np).pin_memory().to(key.device, non_blocking=True)
    so = _lib.lib()
    _lib.check(so.lf_pack_pages(
        ctypes.byref(layout.c), _lib.ptr(key), _lib.ptr(value), _lib.dtype_code(key.dtype),
        key.stride(0), key.stride(1), key.stride(2), _lib.ptr(jobs_dev), int(jobs_np.shape[0]), B,
        _lib.ptr(layout.chan_code), _lib.ptr(rows), _lib.ptr(kmeta), _lib.ptr(status),
        _lib.stream_handle(key.device)), "lf_pack_pages")


def _one_page_layout(table: dict, page_shape, group_size: int, v_group: int, device) -> LayerLayout:
    heads, tokens, dim = page_shape
    return LayerLayout(table["tier"].to(torch.int64).cpu(), head_dim=dim, page_size=tokens,
                       k_group_size=group_size, v_group_size=v_group, bit_v=2, row_cap=tokens,
                       device=device)


def quantize_key_page(page: torch.Tensor, table: dict, group_size: int) -> dict:
    """layout.py:71-112 on the GPU (K1).  ``page`` ``[heads, tokens, dim]``."""
    heads, tokens, dim = page.shape
    if tokens % group_size:
        raise ValueError(f"Key page length {tokens} is not a multiple of {group_size}")
    lay = _one_page_layout(table, page.shape, group_size, dim, page.device)
    rows, kmeta = lay.alloc(1)
    pack_pages(lay, rows, kmeta, page[None], page[None], [(0, 0, 0, 0)])
    views = lay.hist_k_views(rows[0], kmeta[0], tokens)
    return {code: {k: v.contiguous() for k, v in d.items()} for code, d in views.items()}


def quantize_value_page(page: torch.Tensor, bits: int, group_size: int) -> dict:
    """layout.py:115-129 on the GPU (K1).  ``page`` ``[heads, tokens, dim]``."""
    heads, tokens, dim = page.shape
    if bits >= 16:
        return {"value": page.to(torch.float16)}
    if bits != 2:
        raise NotImplementedError("the packed backend stores Value at 2 bits")
    if dim % group_size:
        raise ValueError(f"head dim {dim} is not divisible by value group {group_size}")
    levels = torch.zeros(heads, dim, dtype=torch.int64)
    lay = LayerLayout(levels, head_dim=dim, page_size=tokens, k_group_size=tokens,
                      v_group_size=group_size, bit_v=2, row_cap=tokens, device=page.device)
    rows, kmeta = lay.alloc(1)
    pack_pages(lay, rows, kmeta, page[None], page[None], [(0, 0, 0, 0)])
    return {k: v.contiguous() for k, v in lay.hist_v_views(rows[0], tokens).items()}
