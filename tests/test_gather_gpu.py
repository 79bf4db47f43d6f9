"""The fused split merge + output gather on one GPU (``lf_decode_merge_gather``,
``lf_gather_wait``), through the C ABI with this GPU as the only rank.

* The merge-gather's block equals ``lf_decode_merge`` bit for bit (the same
  arithmetic, stored to the gathered buffer instead of ``out``), the wait
  returns with the layer's count and takes it back (the counter is 0 again).
* A wait for a counter that nothing signals gives up after its limit with
  LF_ERR_DEVICE_TIMEOUT in the status word; the context stays usable.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from logitfill_b200 import _lib
from logitfill_b200.packed import PackedKVCache
from logitfill_b200.packed.attention import DecodeCall
from logitfill_b200.synthetic import synthetic_kv, synthetic_levels

pytestmark = pytest.mark.gpu


def _alloc(nbytes: int) -> int:
    p = ctypes.c_void_p()
    _lib.check(_lib.lib().lf_ipc_alloc(nbytes, ctypes.byref(p)), "lf_ipc_alloc")
    return p.value


def _free(ptr: int) -> None:
    _lib.check(_lib.lib().lf_ipc_free(ctypes.c_void_p(ptr)), "lf_ipc_free")


def _read(ptr: int, count: int, dtype) -> torch.Tensor:
    """Copy ``count`` elements at a raw device address into a new tensor."""
    t = torch.empty(count, dtype=dtype, device="cuda")
    torch.cuda.synchronize()
    view = torch.as_tensor(_View(ptr, count * t.element_size()), device="cuda").view(dtype)
    t.copy_(view)
    return t


class _View:
    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                         "strides": None}


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_merge_gather_single_rank_equals_merge(out_dtype):
    B, H, NQ, D, T = 3, 4, 28, 128, 1500
    levels = synthetic_levels(1, H, D, 2.5, seed=21)[0]
    lengths = [T, T - 300, 777]
    k, v = synthetic_kv(B, H, T + 8, D, seed=21, layer=0, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(22)
    q = torch.randn(B, NQ, D, generator=g, device="cuda").to(torch.bfloat16)
    kn = torch.stack([k[b, :, n] for b, n in enumerate(lengths)]).contiguous()
    vn = torch.stack([v[b, :, n] for b, n in enumerate(lengths)]).contiguous()
    cache = PackedKVCache([levels], B, NQ, H, D, device="cuda", capacity=T + 128)
    cache.prefill(0, k, v, lengths)
    want = torch.empty(B, NQ, D, dtype=out_dtype, device="cuda")
    call = DecodeCall(cache, 0, q, kn, vn, D ** -0.5, want, pps=3)
    call.launch_partial()
    call.launch_merge()
    so = _lib.lib()
    n = B * NQ * D
    esz = want.element_size()
    layers, layer = 3, 2
    buf, flags = _alloc(layers * n * esz), _alloc(4 * layers)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    try:
        peer_out = torch.tensor(np.array([buf], np.uint64).view(np.int64), device="cuda")
        peer_flags = torch.tensor(np.array([flags], np.uint64).view(np.int64), device="cuda")
        _lib.check(so.lf_decode_merge_gather(
            _lib.ptr(call.ws), _lib.ptr(cache.layers[0].dev_hist), B, H, NQ, D, cache.page_size, call.pps,
            call.max_splits, _lib.ptr(peer_out), _lib.ptr(peer_flags), layer, 0, 1, _lib.dtype_code(out_dtype),
            _lib.stream_handle(torch.device("cuda"))), "lf_decode_merge_gather")
        expected = so.lf_gather_signals(B, NQ, 1)
        assert expected == (B * NQ + 3) // 4
        _lib.check(so.lf_gather_wait(ctypes.c_void_p(flags), layer, expected, 2_000_000_000, _lib.ptr(status),
                                     _lib.stream_handle(torch.device("cuda"))), "lf_gather_wait")
        torch.cuda.synchronize()
        cache.check_status()
        assert int(status.item()) == 0
        got = _read(buf + layer * n * esz, n, out_dtype).view(B, NQ, D)
        assert torch.equal(got, want)
        counters = _read(flags, layers, torch.int32)
        assert counters.tolist() == [0, 0, 0]
    finally:
        torch.cuda.synchronize()
        _free(buf)
        _free(flags)


def test_gather_wait_gives_up_on_a_silent_counter():
    so = _lib.lib()
    flags = _alloc(4 * 2)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    try:
        _lib.check(so.lf_gather_wait(ctypes.c_void_p(flags), 1, 4, 1_000_000, _lib.ptr(status),
                                     _lib.stream_handle(torch.device("cuda"))), "lf_gather_wait")
        torch.cuda.synchronize()
        assert int(status.item()) == _lib.LF_ERR_DEVICE_TIMEOUT
        assert _read(flags, 2, torch.int32).tolist() == [0, 0]  # nothing taken back
        # the context is still usable
        x = torch.arange(10, device="cuda")
        assert int(x.sum().item()) == 45
    finally:
        torch.cuda.synchronize()
        _free(flags)
