"""KV-head sharding on 2 GPUs: the gathered output equals the 1-GPU output.

Two NCCL ranks (child processes, one GPU each) hold 4 of the 8 KV heads of a
config-4-shaped layer (40 q / 8 KV heads, GQA 5) with their 20 query heads,
run K2 + K3 on them and gather the head-sharded outputs, either with an NCCL
all-gather (``logitfill_b200.sharding.gather_heads``) or through peer memory
(``PeerGather``: the split merge stores each rank's heads into both ranks'
buffers over NVLink, then a bounded wait per layer; run for two steps so the
layer counter must have been taken back in between).  Rank 0 also decodes the
whole layer on its GPU; the reassembled output must equal it (the same kernels
run on the same heads with the same split plan; max-abs 1e-6 allowed for the
wider tier padding of the full layer), and the two gathers must agree bit for
bit.  Skipped on a box with fewer than two GPUs.  NVLS is off for the
collective (NCCL_NVLS_ENABLE=0); no multicast object is created.

Failure detection without a fault: rank 1 then leaves one layer unmerged (it
stays alive and in step); rank 0's wait for that layer gives up after 0.1 s
with LF_ERR_DEVICE_TIMEOUT in its status word and its context stays usable.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data(dev):
    from logitfill_b200.synthetic import synthetic_kv, synthetic_levels

    B, H, NQ, D, T = 3, 8, 40, 128, 2048
    levels = synthetic_levels(1, H, D, 2.5, seed=14)[0]
    lengths = [T + 5, T - 128 * 3 + 64, 900]
    k, v = synthetic_kv(B, H, T + 8, D, seed=14, layer=0, device=dev)
    g = torch.Generator(device=dev).manual_seed(15)
    q = torch.randn(B, NQ, D, generator=g, device=dev).to(torch.bfloat16)
    kn = torch.stack([k[b, :, n] for b, n in enumerate(lengths)]).contiguous()
    vn = torch.stack([v[b, :, n] for b, n in enumerate(lengths)]).contiguous()
    return levels, lengths, k, v, q, kn, vn, (B, H, NQ, D, T)


def _decode(levels, lengths, k, v, q, kn, vn, dims, dev, pps=4):
    from logitfill_b200.packed import PackedKVCache
    from logitfill_b200.packed.attention import decode_into

    B, H, NQ, D, T = dims
    cache = PackedKVCache([levels], B, NQ, H, D, device=dev, capacity=T + 128)
    cache.prefill(0, k, v, lengths)
    out = torch.empty(B, NQ, D, dtype=torch.float32, device=dev)
    decode_into(cache, 0, q, kn, vn, D ** -0.5, out, pps=pps)
    cache.check_status()
    return out


def _peer_gather(levels, lengths, k, v, q, kn, vn, dims, dev, pps=4, steps=2):
    """The rank's layer decoded with K2, then gathered by the fused split
    merge through peer memory; the gathered ``[world, B, n_q/world, D]`` of
    every step."""
    from logitfill_b200.packed import PackedKVCache
    from logitfill_b200.packed.attention import DecodeCall
    from logitfill_b200.sharding import PeerGather

    B, H, NQ, D, T = dims
    cache = PackedKVCache([levels], B, NQ, H, D, device=dev, capacity=T + 128)
    cache.prefill(0, k, v, lengths)
    out = torch.empty(B, NQ, D, dtype=torch.float32, device=dev)
    call = DecodeCall(cache, 0, q, kn, vn, D ** -0.5, out, pps=pps)
    peer = PeerGather(1, B, NQ, D, torch.float32, dev, limit_ns=5_000_000_000)
    got = []
    try:
        for _ in range(steps):
            call.launch_partial()
            peer.merge(call, 0)
            peer.wait(0)
            torch.cuda.synchronize(dev)
            cache.check_status()
            peer.check_status()
            got.append(peer.gathered[0].clone())
    finally:
        peer.close()
    return got


def _silent_rank(levels, lengths, k, v, q, kn, vn, dims, dev, rank: int) -> int:
    """Rank 1 decodes but never merges or signals the layer; rank 0's bounded
    wait (0.1 s) must give up.  Returns rank 0's status code (0 on rank 1)."""
    from logitfill_b200.packed import PackedKVCache
    from logitfill_b200.packed.attention import DecodeCall
    from logitfill_b200.sharding import PeerGather

    B, H, NQ, D, T = dims
    cache = PackedKVCache([levels], B, NQ, H, D, device=dev, capacity=T + 128)
    cache.prefill(0, k, v, lengths)
    out = torch.empty(B, NQ, D, dtype=torch.float32, device=dev)
    call = DecodeCall(cache, 0, q, kn, vn, D ** -0.5, out, pps=4)
    peer = PeerGather(1, B, NQ, D, torch.float32, dev, limit_ns=100_000_000)
    code = 0
    try:
        call.launch_partial()
        if rank == 0:
            peer.merge(call, 0)
            peer.wait(0)
        torch.cuda.synchronize(dev)
        code = int(peer.status.item())
        peer.status.zero_()
        assert int(torch.arange(10, device=dev).sum().item()) == 45  # the context is still usable
    finally:
        peer.close()
    return code


def _worker(rank: int, world: int, port: int, out) -> None:
    import datetime

    import torch.distributed as dist

    from logitfill_b200.sharding import assemble_heads, gather_heads, kv_head_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        levels, lengths, k, v, q, kn, vn, dims = _data(dev)
        B, H, NQ, D, T = dims
        h0, h1, q0, q1 = kv_head_range(H, NQ, world, rank)
        local = _decode(levels[h0:h1], lengths, k[:, h0:h1].contiguous(), v[:, h0:h1].contiguous(),
                        q[:, q0:q1].contiguous(), kn[:, h0:h1].contiguous(), vn[:, h0:h1].contiguous(),
                        (B, h1 - h0, q1 - q0, D, T), dev)
        gathered = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=dev)
        gather_heads(local, gathered)
        full_sharded = assemble_heads(gathered)
        p2p = _peer_gather(levels[h0:h1], lengths, k[:, h0:h1].contiguous(), v[:, h0:h1].contiguous(),
                           q[:, q0:q1].contiguous(), kn[:, h0:h1].contiguous(), vn[:, h0:h1].contiguous(),
                           (B, h1 - h0, q1 - q0, D, T), dev)
        same = all(bool(torch.equal(assemble_heads(g), full_sharded)) for g in p2p)
        silent = _silent_rank(levels[h0:h1], lengths, k[:, h0:h1].contiguous(), v[:, h0:h1].contiguous(),
                              q[:, q0:q1].contiguous(), kn[:, h0:h1].contiguous(), vn[:, h0:h1].contiguous(),
                              (B, h1 - h0, q1 - q0, D, T), dev, rank)
        if rank == 0:
            full = _decode(levels, lengths, k, v, q, kn, vn, dims, dev)
            diff = float((full_sharded - full).abs().max())
            out.put((rank, diff, same, silent))
        else:
            out.put((rank, 0.0, same, silent))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_kv_sharded_two_gpus_equals_one_gpu():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(out.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    (_, diff, same0, silent0), (_, _, same1, _) = results
    assert diff <= 1e-6, diff
    assert same0 and same1, "the NVLink merge-gather differs from the NCCL all-gather"
    from logitfill_b200._lib import LF_ERR_DEVICE_TIMEOUT

    assert silent0 == LF_ERR_DEVICE_TIMEOUT, silent0  # the wait for a rank that never signalled gave up
