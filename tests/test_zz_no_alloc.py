"""GPU test of lf_decode_noalloc, the decode entry point that allocates nothing.

Callers that cannot allocate device memory (allocator callbacks, runtimes
that plan every allocation up front, hosts that link only the library) call
lf_decode_noalloc instead of lf_decode_partial + lf_decode_merge: the split
partials live in a fixed 8 MiB array inside the library.  This test calls it
through the C ABI twice in a row and checks each output against the
workspace-based entry point (lf_decode) on the same inputs: the same kernels
run on the same data, so the outputs must be equal bit for bit.  The second
call has fewer splits than the first, so a read of a partial left in the
shared array by the first call would change its output.  It also checks that
the calls allocate no device memory, and that an oversized request is
rejected before any launch.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from logitfill_b200 import _lib
from logitfill_b200.packed import PackedKVCache
from logitfill_b200.packed.attention import DecodeCall
from logitfill_b200.synthetic import synthetic_kv, synthetic_levels

pytestmark = pytest.mark.gpu
NOALLOC_LIMIT = 8 << 20


def _setup(batch, history, n_kv=4, n_q=28, head_dim=128, seed=21):
    levels = synthetic_levels(1, n_kv, head_dim, 2.5, seed=seed)[0]
    T = max(history) + 1
    k, v = synthetic_kv(batch, n_kv, T, head_dim, seed=seed, layer=0, device="cuda")
    cache = PackedKVCache([levels], batch, n_q, n_kv, head_dim, device="cuda", capacity=max(1024, T + 127))
    cache.prefill(0, k, v, list(history))
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(batch, n_q, head_dim, generator=g, device="cuda").to(torch.bfloat16)
    kn = torch.stack([k[b, :, n] for b, n in enumerate(history)]).contiguous()
    vn = torch.stack([v[b, :, n] for b, n in enumerate(history)]).contiguous()
    return cache, q, kn, vn


def _noalloc(call: DecodeCall, out: torch.Tensor, splits_override=None) -> int:
    so, L, c = _lib.lib(), call.layer, call.cache
    tk, kn = L.tail_k, call.key_new
    return so.lf_decode_noalloc(
        ctypes.byref(L.layout.c), _lib.ptr(L.rows), _lib.ptr(L.kmeta), _lib.ptr(L.layout.slot_chan),
        _lib.ptr(L.dev_hist), _lib.ptr(tk), _lib.ptr(L.tail_v), tk.stride(0), tk.stride(1), _lib.ptr(L.dev_tail),
        _lib.dtype_code(call.resid_dtype), _lib.ptr(kn), _lib.ptr(call.value_new), kn.stride(0), kn.stride(1),
        _lib.ptr(call.query), _lib.dtype_code(call.query.dtype), call.query.stride(0), call.query.stride(1),
        c.batch, c.n_q, call.scaling, call.pps, splits_override or call.max_splits,
        _lib.ptr(out), _lib.dtype_code(out.dtype), out.stride(0), out.stride(1), _lib.ptr(c.status),
        _lib.stream_handle(out.device))


def _case(batch, history, pps, seed):
    """A decode call, its output from the workspace path, and a NaN-filled
    output buffer for the allocation-free call."""
    cache, q, kn, vn = _setup(batch, history, seed=seed)
    ref = torch.empty(q.shape, dtype=torch.float32, device="cuda")
    call = DecodeCall(cache, 0, q, kn, vn, 128 ** -0.5, ref, pps=pps)
    call.launch()
    need = _lib.lib().lf_decode_workspace_bytes(cache.batch, cache.n_kv, cache.n_q, cache.head_dim, call.max_splits)
    assert 0 < need <= NOALLOC_LIMIT
    out = torch.full(q.shape, float("nan"), dtype=torch.float32, device="cuda")
    return cache, call, ref, out


def test_noalloc_matches_workspace_path_twice():
    # First call: many splits (3 sequences, up to 9 pages, 1 page per split);
    # second call: fewer splits over other data (1 sequence, 2 pages, 2 per split).
    big = _case(3, (1024 + 37, 700, 128 * 9), pps=1, seed=21)
    small = _case(1, (2 * 128 + 5,), pps=2, seed=22)
    assert small[1].max_splits < big[1].max_splits
    torch.cuda.synchronize()
    for cache, call, ref, out in (big, small):
        _lib.check(_noalloc(call, out), "lf_decode_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(out, ref), float((out - ref).abs().max())
        cache.check_status()


def test_noalloc_allocates_nothing():
    cache, call, ref, out = _case(2, (1024 + 3, 500), pps=3, seed=23)
    _lib.check(_noalloc(call, out), "lf_decode_noalloc")  # first call in this context: address lookup
    torch.cuda.synchronize()
    stats0 = torch.cuda.memory_stats()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        _lib.check(_noalloc(call, out), "lf_decode_noalloc")
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    stats1 = torch.cuda.memory_stats()
    assert free1 == free0
    for key in ("allocation.all.allocated", "segment.all.allocated", "reserved_bytes.all.current"):
        assert stats1.get(key, 0) == stats0.get(key, 0), key
    assert torch.equal(out, ref)


def test_noalloc_rejects_oversized_partials():
    cache, q, kn, vn = _setup(1, (1024 + 37,))
    out = torch.empty(q.shape, dtype=torch.float32, device="cuda")
    call = DecodeCall(cache, 0, q, kn, vn, 128 ** -0.5, out)
    per_split = _lib.lib().lf_decode_workspace_bytes(1, cache.n_kv, cache.n_q, cache.head_dim, 1)
    too_many = NOALLOC_LIMIT // per_split + 1
    status = _noalloc(call, out, splits_override=too_many)
    assert status == _lib.LF_ERR_INVALID_ARGUMENT
    assert b"scratch" in _lib.lib().lf_last_error()
