"""Packed history cache plus the original-dtype residual page.

Mirrors ``src/logitfill/packed/cache.py``.  :class:`PackedKVCache` is the
batched B200 store: per layer, preallocated ``rows``/``kmeta`` history
buffers (see :mod:`logitfill_b200.packed.layout`), a residual page
``[B, H, page, D]`` in the caller's dtype, and per-sequence lengths kept on the
host (authoritative) and on the device (read by the kernels).
:class:`PackedKVManager` is the reference's single-sequence manager with the
same constructor and methods, built on a one-sequence :class:`PackedKVCache`;
``manager.layers[i]`` exposes ``table``, ``hist_k``, ``hist_v``, ``hist_len``,
``tail_k``, ``tail_v`` in the reference's shapes and dtypes (views, no copies).

Page flushes run the K1 kernel (bit-exact with ``layout.py:71-129``) and write
straight into the preallocated history, replacing the O(T) ``torch.cat`` of
``cache.py:71-80``.  Capacity grows by doubling when a commit needs it.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from logitfill_b200 import _lib
from logitfill_b200.packed.layout import LayerLayout, pack_pages

DEFAULT_CAPACITY = 1024


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class _Layer:
    """One layer of a batched cache."""

    def __init__(self, levels, cache: "PackedKVCache"):
        c = cache
        self.cache = c
        self.layout = LayerLayout(levels, head_dim=c.head_dim, page_size=c.page_size,
                                  k_group_size=c.k_group_size, v_group_size=c.v_group_size,
                                  bit_v=c.bit_v, row_cap=c.row_cap, device=c.device)
        if self.layout.kv_heads != c.n_kv:
            raise ValueError(f"level map has {self.layout.kv_heads} heads, expected {c.n_kv}")
        self.rows, self.kmeta = self.layout.alloc(c.batch)
        self.hist_len = np.zeros(c.batch, np.int64)   # host, authoritative
        self.tail_len = np.zeros(c.batch, np.int64)
        self.tail_k: Optional[torch.Tensor] = None    # [B, H, page, D], allocated at first commit
        self.tail_v: Optional[torch.Tensor] = None
        self.dev_hist = torch.zeros(c.batch, dtype=torch.int32, device=c.device)
        self.dev_tail = torch.zeros(c.batch, dtype=torch.int32, device=c.device)
        self.pps_memo: dict = {}  # (pages, q_len) -> pages per K2 work item

    # -- state -------------------------------------------------------------
    def reset(self) -> None:
        self.hist_len[:] = 0
        self.tail_len[:] = 0
        self.sync_lengths()

    def sync_lengths(self) -> None:
        # Pinned, non-blocking uploads: ordered on the stream before every later
        # kernel, without making the host wait for the kernels already queued.
        both = torch.from_numpy(np.concatenate([self.hist_len, self.tail_len]).astype(np.int32)).pin_memory()
        n = self.hist_len.shape[0]
        self.dev_hist.copy_(both[:n], non_blocking=True)
        self.dev_tail.copy_(both[n:], non_blocking=True)

    def ensure_residual(self, dtype) -> None:
        c = self.cache
        if self.tail_k is None:
            shape = (c.batch, c.n_kv, c.page_size, c.head_dim)
            self.tail_k = torch.zeros(shape, dtype=dtype, device=c.device)
            self.tail_v = torch.zeros(shape, dtype=dtype, device=c.device)
        elif self.tail_k.dtype != dtype:
            raise TypeError(f"residual page holds {self.tail_k.dtype}, got {dtype}")

    def grow(self, row_cap: int) -> None:
        old_rows, old_meta = self.rows, self.kmeta
        old_cap, old_gcap = self.layout.row_cap, self.layout.group_cap
        self.layout.set_capacity(row_cap)
        self.rows, self.kmeta = self.layout.alloc(self.cache.batch)
        self.rows[:, :, :old_cap].copy_(old_rows)
        self.kmeta[:, :, :old_gcap].copy_(old_meta)

    # -- commit (cache.py:48-62) ------------------------------------------
    def append(self, key: torch.Tensor, value: torch.Tensor, seqs=None) -> None:
        """Append ``key``/``value`` ``[S, H, T, D]`` to sequences ``seqs``
        (default: all) and flush every page that fills."""
        c = self.cache
        S, H, T, D = key.shape
        if value.shape != key.shape:
            raise ValueError("Key and Value pages do not match")
        if H != c.n_kv or D != c.head_dim:
            raise ValueError(f"expected [*, {c.n_kv}, T, {c.head_dim}], got {tuple(key.shape)}")
        seqs = list(range(S)) if seqs is None else [int(s) for s in seqs]
        if len(seqs) != S:
            raise ValueError("one sequence index per batch row is required")
        if T == 0:
            return
        if key.device != c.device:
            raise RuntimeError(f"tensors must be on {c.device} (the packed backend has no CPU path)")
        self.ensure_residual(key.dtype)
        value = value.to(key.dtype)
        if key.stride() != value.stride() or key.stride(3) != 1:
            # K1 reads both pages with one set of strides.
            key, value = key.contiguous(), value.contiguous()
        P = c.page_size
        need = max(self.hist_len[b] + ((self.tail_len[b] + T) // P) * P for b in seqs)
        if need > self.layout.row_cap:
            c.grow_to(need)
        tail_jobs, src_jobs = [], []
        moves = []  # (seq, src_row, src_t0, dst_t0, n) copies into the residual page
        for i, b in enumerate(seqs):
            tl, pos = int(self.tail_len[b]), 0
            if tl + T >= P:
                fill = P - tl
                if tl > 0:
                    self.tail_k[b, :, tl:P].copy_(key[i, :, :fill])
                    self.tail_v[b, :, tl:P].copy_(value[i, :, :fill])
                    tail_jobs.append((b, 0, b, int(self.hist_len[b]) // P))
                    self.hist_len[b] += P
                    pos = fill
                    tl = 0
                while T - pos >= P:
                    src_jobs.append((i, pos, b, int(self.hist_len[b]) // P))
                    self.hist_len[b] += P
                    pos += P
            if pos < T:
                moves.append((b, i, pos, tl, T - pos))
                tl += T - pos
            self.tail_len[b] = tl
        if tail_jobs:
            pack_pages(self.layout, self.rows, self.kmeta, self.tail_k, self.tail_v, tail_jobs)
        if src_jobs:
            pack_pages(self.layout, self.rows, self.kmeta, key, value, src_jobs)
        for b, i, s0, d0, n in moves:
            self.tail_k[b, :, d0:d0 + n].copy_(key[i, :, s0:s0 + n])
            self.tail_v[b, :, d0:d0 + n].copy_(value[i, :, s0:s0 + n])
        self.sync_lengths()

    # -- device-side commit of one token per sequence --------------------
    def commit_token_device(self, key: torch.Tensor, value: torch.Tensor) -> None:
        """Launch ``lf_commit_token`` for ``key``/``value`` ``[B, H, D]`` (one
        new token for every sequence of the cache): append to the residual
        page, pack the page when it fills, advance the device lengths.  The
        host lengths are not touched; :meth:`advance_host` mirrors the step.
        Graph-capturable: no host decision depends on the lengths."""
        c = self.cache
        B, H, D = key.shape
        if (B, H, D) != (c.batch, c.n_kv, c.head_dim) or value.shape != key.shape:
            raise ValueError(f"token Key/Value must be [{c.batch}, {c.n_kv}, {c.head_dim}]")
        self.ensure_residual(key.dtype)
        value = value.to(key.dtype)
        if key.stride() != value.stride() or key.stride(2) != 1:
            key, value = key.contiguous(), value.contiguous()
        if c._commit_jobs is None:
            c._commit_jobs = torch.empty(4 * c.batch, dtype=torch.int32, device=c.device)
        tk = self.tail_k
        _lib.check(_lib.lib().lf_commit_token(
            ctypes.byref(self.layout.c), _lib.ptr(self.rows), _lib.ptr(self.kmeta), _lib.ptr(self.layout.chan_code),
            _lib.ptr(tk), _lib.ptr(self.tail_v), tk.stride(0), tk.stride(1), _lib.ptr(self.dev_hist),
            _lib.ptr(self.dev_tail), _lib.dtype_code(key.dtype), _lib.ptr(key), _lib.ptr(value), key.stride(0),
            key.stride(1), c.batch, _lib.ptr(c._commit_jobs), _lib.ptr(c.status), _lib.stream_handle(c.device)),
            "lf_commit_token")

    def advance_host(self) -> None:
        """Mirror one device-side token commit in the host lengths."""
        P = self.cache.page_size
        t = self.tail_len + 1
        full = t == P
        self.hist_len[full] += P
        self.tail_len[:] = np.where(full, 0, t)

    def dequantize(self, b: int):
        """cache.py:83-90 via the CUDA dequantizer: fp32 ``[H, hist_len, D]``."""
        c = self.cache
        T = int(self.hist_len[b])
        k = torch.empty(c.n_kv, T, c.head_dim, dtype=torch.float32, device=c.device)
        v = torch.empty_like(k)
        if T:
            _lib.check(_lib.lib().lf_dequantize(
                ctypes.byref(self.layout.c), _lib.ptr(self.rows), _lib.ptr(self.kmeta),
                _lib.ptr(self.layout.chan_code), int(b), T, _lib.ptr(k), _lib.ptr(v),
                _lib.stream_handle(c.device)), "lf_dequantize")
        return k, v


class PackedKVCache:
    """Batched packed KV cache for ``batch`` sequences, one store per layer.

    ``levels`` is a list (per layer) of ``[n_kv, head_dim]`` tier maps
    (0=INT2, 1=INT4, 2=INT8, 3=FP16) or ``None`` (all INT2), as the reference's
    ``PackedKVManager`` takes them (cache.py:93-120)."""

    def __init__(self, levels, batch: int, n_q: int, n_kv: int, head_dim: int, page_size: int = 128,
                 k_group_size: int = 128, v_group_size: int = 128, bit_v: int = 2, device="cuda",
                 capacity: int = DEFAULT_CAPACITY):
        self.batch = int(batch)
        self.n_q, self.n_kv, self.head_dim = int(n_q), int(n_kv), int(head_dim)
        self.page_size, self.k_group_size = int(page_size), int(k_group_size)
        self.v_group_size, self.bit_v = int(v_group_size), int(bit_v)
        if self.bit_v != 2:
            raise NotImplementedError("the packed backend stores Value at 2 bits (bit_v=2)")
        if self.n_q % self.n_kv:
            raise ValueError("query heads must divide into KV heads")
        if self.page_size % self.k_group_size:
            raise ValueError(f"page_size {page_size} must be a multiple of k_group_size {k_group_size}")
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.row_cap = _round_up(max(int(capacity), self.page_size), self.page_size)
        self.layers = []
        for level in levels:
            lv = torch.zeros(self.n_kv, self.head_dim, dtype=torch.int64) if level is None \
                else torch.as_tensor(level, dtype=torch.int64).cpu()
            self.layers.append(_Layer(lv, self))
        self._workspace: Optional[torch.Tensor] = None
        self._commit_jobs: Optional[torch.Tensor] = None  # device job rows of lf_commit_token
        # Device status word written by kernels whose bounded waits expire.
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    @property
    def n_layers(self) -> int:
        return len(self.layers)

    def grow_to(self, tokens: int) -> None:
        new_cap = self.row_cap
        while new_cap < tokens:
            new_cap *= 2
        if new_cap == self.row_cap:
            return
        self.row_cap = new_cap
        for layer in self.layers:
            layer.grow(new_cap)
        self._workspace = None

    def reset(self) -> None:
        for layer in self.layers:
            layer.reset()

    def commit(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor, seqs=None) -> None:
        """Append ``key``/``value`` ``[S, n_kv, T, D]`` after attention (cache.py:135-140)."""
        self.layers[layer_idx].append(key.detach(), value.detach(), seqs)

    def prefill(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor, lengths) -> None:
        """Ragged prefill: sequence ``b`` takes its first ``lengths[b]`` tokens
        of ``key``/``value`` ``[B, n_kv, T, D]``."""
        lengths = [int(x) for x in lengths]
        for b, n in enumerate(lengths):
            if n:
                self.commit(layer_idx, key[b:b + 1, :, :n], value[b:b + 1, :, :n], seqs=[b])

    def workspace(self, max_splits: int, q_len: int = 1) -> torch.Tensor:
        need = _lib.lib().lf_decode_workspace_bytes(self.batch, self.n_kv, self.n_q * q_len, self.head_dim,
                                                    max_splits)
        if self._workspace is None or self._workspace.numel() * 4 < need:
            self._workspace = torch.empty(need // 4, dtype=torch.float32, device=self.device)
        return self._workspace

    def check_status(self) -> None:
        """Raise if a kernel reported a device-side failure (synchronises)."""
        code = int(self.status.item())
        if code:
            self.status.zero_()
            _lib.check(code, "packed KV kernel")

    def length(self, b: int = 0, layer_idx: int = 0) -> int:
        layer = self.layers[layer_idx]
        return int(layer.hist_len[b] + layer.tail_len[b])


class _LayerStore:
    """One sequence's view of one layer, with the reference ``_LayerStore``
    fields (cache.py:16-90)."""

    def __init__(self, cache: PackedKVCache, layer_idx: int, seq: int):
        self._cache, self._layer, self._seq = cache, cache.layers[layer_idx], int(seq)
        self.page_size = cache.page_size
        self.k_group_size = cache.k_group_size
        self.v_group_size = cache.v_group_size
        self.bit_v = cache.bit_v

    @property
    def table(self) -> dict:
        return self._layer.layout.table

    @property
    def hist_len(self) -> int:
        return int(self._layer.hist_len[self._seq])

    @property
    def tail_len(self) -> int:
        return int(self._layer.tail_len[self._seq])

    @property
    def length(self) -> int:
        return self.hist_len + self.tail_len

    @property
    def hist_k(self):
        if self.hist_len == 0:
            return None
        L = self._layer
        return L.layout.hist_k_views(L.rows[self._seq], L.kmeta[self._seq], self.hist_len)

    @property
    def hist_v(self):
        if self.hist_len == 0:
            return None
        L = self._layer
        return L.layout.hist_v_views(L.rows[self._seq], self.hist_len)

    @property
    def tail_k(self):
        n = self.tail_len
        return None if n == 0 else self._layer.tail_k[self._seq, :, :n]

    @property
    def tail_v(self):
        n = self.tail_len
        return None if n == 0 else self._layer.tail_v[self._seq, :, :n]

    def reset(self) -> None:
        self._layer.hist_len[self._seq] = 0
        self._layer.tail_len[self._seq] = 0
        self._layer.sync_lengths()

    def append(self, key: torch.Tensor, value: torch.Tensor) -> None:
        self._layer.append(key[None], value[None], seqs=[self._seq])

    def dequantize(self):
        return self._layer.dequantize(self._seq)


class PackedKVManager:
    """Per-layer packed KV for one sequence (cache.py:93-140), on the GPU."""

    def __init__(self, levels, n_q: int, n_kv: int, head_dim: int, page_size: int, k_group_size: int,
                 v_group_size: int, bit_v: int, device, capacity: int = DEFAULT_CAPACITY):
        self.n_q, self.n_kv, self.head_dim = int(n_q), int(n_kv), int(head_dim)
        self.page_size, self.k_group_size = int(page_size), int(k_group_size)
        self.v_group_size, self.bit_v = int(v_group_size), int(bit_v)
        self.device = device
        self.seq_len = 0
        self.cache = PackedKVCache(levels, 1, n_q, n_kv, head_dim, page_size, k_group_size,
                                   v_group_size, bit_v, device, capacity)
        self.layers = [_LayerStore(self.cache, i, 0) for i in range(self.cache.n_layers)]

    def reset(self) -> None:
        self.seq_len = 0
        self.cache.reset()

    def layer_length(self, layer_idx: int) -> int:
        return self.layers[layer_idx].length

    def commit(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor) -> None:
        if key.shape[0] != 1:
            raise NotImplementedError("packed KV supports one sequence at a time")
        self.cache.commit(layer_idx, key, value)
        if layer_idx == len(self.layers) - 1:
            self.seq_len = self.layers[layer_idx].length

    def commit_token(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor, advance_host: bool = True) -> None:
        """Device-side commit of one token (``key``/``value`` ``[1, H, 1, D]``):
        ``lf_commit_token``.  With ``advance_host=False`` the host lengths
        stay as they are (a captured step; call :meth:`advance_host` after
        each replay)."""
        if key.shape[0] != 1 or key.shape[2] != 1:
            raise NotImplementedError("commit_token takes one token of one sequence")
        layer = self.cache.layers[layer_idx]
        if layer.hist_len[0] + layer.tail_len[0] + 1 > self.cache.row_cap:
            raise RuntimeError("packed history capacity exceeded; grow the cache before capturing")
        layer.commit_token_device(key[:, :, 0], value[:, :, 0])
        if advance_host:
            layer.advance_host()
            if layer_idx == len(self.layers) - 1:
                self.seq_len = self.layers[layer_idx].length

    def advance_host(self) -> None:
        """Mirror one captured decode step (every layer) in the host lengths."""
        for layer in self.cache.layers:
            layer.advance_host()
        self.seq_len = self.layers[-1].length

    def attend(self, layer_idx: int, query: torch.Tensor, key_new: torch.Tensor, value_new: torch.Tensor,
               scaling: float) -> torch.Tensor:
        """``packed_attention(self, ...)`` (reference.py:112-116): K2 + K3 over
        this layer's packed history, residual page and the new token."""
        from logitfill_b200.packed.attention import packed_attention

        return packed_attention(self, layer_idx, query, key_new, value_new, scaling)


try:
    from transformers.cache_utils import Cache as _TransformersCache
except ImportError:  # pragma: no cover - transformers absent
    _TransformersCache = object


class LogitFillCache(_TransformersCache):
    """HF ``Cache`` shim so ``generate`` can read the packed length (cache.py:149-183)."""

    def __init__(self, manager: PackedKVManager):
        # transformers >= 4.56 wants the layer list (empty here: the packed
        # store lives in the manager); older versions take no arguments.
        try:
            super().__init__(layers=[])
        except TypeError:
            try:
                super().__init__()
            except TypeError:
                pass
        self.manager = manager
        self.key_cache = []
        self.value_cache = []

    def get_seq_length(self, layer_idx: int = 0) -> int:
        del layer_idx
        return int(self.manager.seq_len)

    def get_max_cache_shape(self):
        return None

    def get_mask_sizes(self, cache_position, layer_idx: int = 0):
        """(kv_length, kv_offset); transformers 4.x passes the query's
        ``cache_position`` tensor, 5.x its length."""
        del layer_idx
        q_len = int(cache_position) if isinstance(cache_position, int) else int(cache_position.shape[0])
        return self.manager.seq_len + q_len, 0

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        raise RuntimeError("packed attention writes the LogitFill manager directly")

    def reset(self) -> None:
        self.manager.reset()

    def note_layer(self, layer_idx: int, seq_len: int) -> None:
        del layer_idx, seq_len

    def reorder_cache(self, beam_idx: torch.Tensor) -> None:
        raise NotImplementedError("packed LogitFill cache does not support beam search")
