"""Multi-GPU placement of the packed decode path (one process per GPU).

The path shards with no exchange inside the kernels:

* **by sequence** -- every rank holds whole sequences (all layers, all KV
  heads) and decodes them alone; nothing is communicated;
* **by KV head** -- every rank holds ``n_kv / world`` KV heads of every
  sequence together with their ``n_q / world`` query heads (the GQA groups of
  ``repeat_kv``, reference.py:10-15, stay on one rank), runs K1/K2/K3 on
  them, and the ``[B, n_q / world, D]`` attention outputs of one layer are
  gathered over NCCL (``all_gather_into_tensor``) so every rank holds the
  layer's full output.

This module holds the host-side rules of the KV-head split and two ways of
gathering: a plain NCCL collective on the caller's stream (no library kernel
reads a peer's memory), or :class:`PeerGather`, where the split merge itself
stores each rank's rows into every rank's buffer over NVLink
(``lf_decode_merge_gather``) and one bounded wait per layer
(``lf_gather_wait``) marks the layer complete.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch


def kv_head_range(n_kv: int, n_q: int, world: int, rank: int) -> tuple[int, int, int, int]:
    """(first KV head, end KV head, first q-head, end q-head) of ``rank``.
    KV heads are split evenly and contiguously; q-head h * gq + j belongs to
    KV head h, so each rank's q-heads are contiguous too."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if n_kv % world:
        raise ValueError(f"{n_kv} KV heads do not split over {world} ranks")
    if n_q % n_kv:
        raise ValueError("query heads must divide into KV heads")
    per = n_kv // world
    gq = n_q // n_kv
    h0 = rank * per
    return h0, h0 + per, h0 * gq, (h0 + per) * gq


def shard_levels(levels, n_kv: int, world: int, rank: int):
    """The rank's rows of per-layer ``[n_kv, head_dim]`` tier maps (a list, one
    map or None per layer, as ``PackedKVCache`` takes them)."""
    h0, h1, _, _ = kv_head_range(n_kv, n_kv, world, rank)
    return [None if lv is None else torch.as_tensor(lv)[h0:h1] for lv in levels]


def gather_heads(local: torch.Tensor, gathered: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather one layer's head-sharded output.  ``local`` ``[B, n_q/world,
    D]`` (contiguous) -> ``gathered`` ``[world, B, n_q/world, D]``, rank r's
    block at index r, on the current stream.  Returns ``gathered``."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    if gathered.shape != (world,) + tuple(local.shape) or not local.is_contiguous():
        raise ValueError(f"gather buffer {tuple(gathered.shape)} does not hold {world} x {tuple(local.shape)}")
    if world == 1:
        gathered[0].copy_(local)
        return gathered
    # the concatenated form [world * B, ...] (both NCCL and gloo take it)
    dist.all_gather_into_tensor(gathered.view((world * local.shape[0],) + tuple(local.shape[1:])), local, group=group)
    return gathered


def assemble_heads(gathered: torch.Tensor) -> torch.Tensor:
    """``[world, B, n_q/world, D]`` -> ``[B, n_q, D]`` in q-head order."""
    world, B, hq, D = gathered.shape
    return gathered.permute(1, 0, 2, 3).reshape(B, world * hq, D)


class _DeviceArray:
    """A torch view of raw device memory (``__cuda_array_interface__``); the
    memory is owned elsewhere."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes // 2,), "typestr": "<u2", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerGather:
    """Output gather of the KV-head split through peer memory.

    Every rank allocates a gathered buffer ``[layers, world, B, n_q_local, D]``
    and ``layers`` uint32 counters (``lf_ipc_alloc``) and exchanges their CUDA
    IPC handles over the process group; the peers' buffers are opened with
    peer access.  :meth:`merge` launches the fused split merge for one layer
    (this rank's block stored into every rank's buffer, then one signal per
    CTA to every rank), :meth:`wait` the bounded wait for that layer's
    signals from all ranks.  Collective: every rank constructs it, and
    :meth:`close` is collective too.  ``gathered`` is a view of memory that
    :meth:`close` frees: copy what must outlive it."""

    def __init__(self, layers: int, batch: int, n_q_local: int, head_dim: int, dtype, device, group=None,
                 limit_ns: int = 2_000_000_000):
        import torch.distributed as dist

        from logitfill_b200 import _lib

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.group = group
        self.layers, self.batch, self.nq, self.D = layers, batch, n_q_local, head_dim
        self.dtype = dtype
        self.device = torch.device(device)
        self.limit_ns = int(limit_ns)
        so = _lib.lib()
        self._so = so
        esz = torch.empty(0, dtype=dtype).element_size()
        self.block = layers * self.world * batch * n_q_local * head_dim
        self._out_bytes = self.block * esz
        own_out, own_flags = ctypes.c_void_p(), ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(so.lf_ipc_alloc(self._out_bytes, ctypes.byref(own_out)), "lf_ipc_alloc")
            _lib.check(so.lf_ipc_alloc(4 * layers, ctypes.byref(own_flags)), "lf_ipc_alloc")
        self._own = [own_out.value, own_flags.value]
        handles = []
        for ptr in self._own:
            buf = ctypes.create_string_buffer(64)
            _lib.check(so.lf_ipc_handle(ctypes.c_void_p(ptr), buf), "lf_ipc_handle")
            handles.append(buf.raw)
        every = [None] * self.world
        dist.all_gather_object(every, handles, group=group)
        self._opened = []
        outs, flags = [], []
        with torch.cuda.device(self.device):
            for r, (ho, hf) in enumerate(every):
                if r == self.rank:
                    outs.append(self._own[0])
                    flags.append(self._own[1])
                    continue
                po, pf = ctypes.c_void_p(), ctypes.c_void_p()
                _lib.check(so.lf_ipc_open(ctypes.create_string_buffer(ho, 64), ctypes.byref(po)), "lf_ipc_open")
                self._opened.append(po.value)
                _lib.check(so.lf_ipc_open(ctypes.create_string_buffer(hf, 64), ctypes.byref(pf)), "lf_ipc_open")
                self._opened.append(pf.value)
                outs.append(po.value)
                flags.append(pf.value)
        self.peer_out = torch.tensor(np.array(outs, dtype=np.uint64).view(np.int64), device=self.device)
        self.peer_flags = torch.tensor(np.array(flags, dtype=np.uint64).view(np.int64), device=self.device)
        self.expected = so.lf_gather_signals(batch, n_q_local, self.world)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        view = torch.as_tensor(_DeviceArray(self._own[0], self._out_bytes), device=self.device)
        self.gathered = view.view(dtype).view(layers, self.world, batch, n_q_local, head_dim)
        dist.barrier(group=group)

    def merge(self, call, layer: int) -> None:
        """This rank's split merge of ``call`` (a one-token ``DecodeCall``
        whose K2 has been launched) stored as block ``rank`` of ``layer`` in
        every rank's gathered buffer, on the current stream."""
        from logitfill_b200 import _lib

        c = call.cache
        _lib.check(self._so.lf_decode_merge_gather(
            _lib.ptr(call.ws), _lib.ptr(call.layer.dev_hist), c.batch, c.n_kv, c.n_q, c.head_dim, c.page_size,
            call.pps, call.max_splits, _lib.ptr(self.peer_out), _lib.ptr(self.peer_flags), int(layer), self.rank,
            self.world, _lib.dtype_code(self.dtype), _lib.stream_handle(self.device)), "lf_decode_merge_gather")

    def wait(self, layer: int) -> None:
        """Bounded wait (on the current stream) for every rank's block of ``layer``."""
        from logitfill_b200 import _lib

        _lib.check(self._so.lf_gather_wait(
            ctypes.c_void_p(self._own[1]), int(layer), self.expected, self.limit_ns, _lib.ptr(self.status),
            _lib.stream_handle(self.device)), "lf_gather_wait")

    def check_status(self) -> None:
        """Raise if a wait gave up (synchronises)."""
        from logitfill_b200 import _lib

        code = int(self.status.item())
        if code:
            self.status.zero_()
            _lib.check(code, "lf_gather_wait")

    def close(self) -> None:
        """Collective: close the peers' buffers, then free this rank's."""
        import torch.distributed as dist

        from logitfill_b200 import _lib

        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                _lib.check(self._so.lf_ipc_close(ctypes.c_void_p(ptr)), "lf_ipc_close")
            self._opened = []
        dist.barrier(group=self.group)
        self.gathered = None
        with torch.cuda.device(self.device):
            for ptr in self._own:
                _lib.check(self._so.lf_ipc_free(ctypes.c_void_p(ptr)), "lf_ipc_free")
        self._own = None
