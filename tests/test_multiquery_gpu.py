"""GPU parity of multi-token attention over the packed cache (q_len > 1: a
chunked prefill after the first) and of GQA groups above 8 (several CTAs per
KV head), against the oracle's dense packed attention with the right-aligned
causal mask (reference.py:18-56).

Tolerance (north star): max-abs 2e-3 and cosine >= 0.9999 per query token.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from logitfill_b200.packed import PackedKVCache, PackedKVManager
from logitfill_b200.packed.attention import packed_attention, packed_attention_batched
from logitfill_b200.synthetic import synthetic_kv, synthetic_levels
from oracle import packed_ref as orc
from tests.gpu_cases import attention_close

pytestmark = pytest.mark.gpu


def _oracle(levels, page, D, k, v, n, q, kn, vn, scaling):
    ref = orc.OracleLayer(levels, page, page, D, 2)
    if n:
        ref.append(k[:, :n].float().cpu().numpy(), v[:, :n].float().cpu().numpy())
    return orc.reference_attention(ref, q.float().cpu().numpy(), kn.float().cpu().numpy(),
                                   vn.float().cpu().numpy(), scaling)


# (n_q, n_kv, head_dim, page): tensor-core geometry (GQA 7) and the CUDA-core one.
GEOMS = [(28, 4, 128, 128), (8, 2, 64, 64)]


@pytest.mark.parametrize("geom", GEOMS, ids=["tc", "simt"])
@pytest.mark.parametrize("q_len", [2, 5, 16, 130])
def test_multi_token_matches_oracle(geom, q_len):
    n_q, H, D, P = geom
    B, T = 2, 6 * P
    levels = synthetic_levels(1, H, D, 2.5, seed=q_len)[0]
    k, v = synthetic_kv(B, H, T + 200 + q_len, D, seed=q_len, layer=0, device="cuda")
    lengths = [T + 3, T - 1]                          # ragged: tails 3 and P-1
    cache = PackedKVCache([levels], B, n_q, H, D, page_size=P, k_group_size=P, v_group_size=D, device="cuda",
                          capacity=T + P)
    cache.prefill(0, k, v, lengths)
    g = torch.Generator(device="cuda").manual_seed(q_len)
    q = torch.randn(B, n_q, q_len, D, generator=g, device="cuda").to(torch.bfloat16)
    kn = torch.stack([k[b, :, n:n + q_len] for b, n in enumerate(lengths)])
    vn = torch.stack([v[b, :, n:n + q_len] for b, n in enumerate(lengths)])
    out = packed_attention_batched(cache, 0, q, kn, vn, D ** -0.5, out_dtype=torch.float32)
    cache.check_status()
    assert out.shape == (B, n_q, q_len, D)
    for b, n in enumerate(lengths):
        want = _oracle(levels, P, D, k[b], v[b], n, q[b], kn[b], vn[b], D ** -0.5)
        got = out[b].cpu().numpy()
        for i in range(q_len):
            ok, err, cos = attention_close(got[:, i], want[:, i])
            assert ok, (b, i, err, cos)


def test_multi_token_one_is_the_decode_step():
    """q_len 1 through the multi-token entry point equals the decode call."""
    n_q, H, D = 28, 4, 128
    levels = synthetic_levels(1, H, D, 3.0, seed=7)[0]
    k, v = synthetic_kv(3, H, 1200, D, seed=7, layer=0, device="cuda")
    cache = PackedKVCache([levels], 3, n_q, H, D, device="cuda", capacity=1280)
    cache.prefill(0, k, v, [1100, 700, 129])
    q = torch.randn(3, n_q, D, device="cuda").to(torch.bfloat16)
    kn, vn = k[:, :, 1150], v[:, :, 1150]
    one = packed_attention_batched(cache, 0, q, kn, vn, D ** -0.5, out_dtype=torch.float32)
    multi = packed_attention_batched(cache, 0, q[:, :, None], kn[:, :, None], vn[:, :, None], D ** -0.5,
                                     out_dtype=torch.float32)
    assert torch.equal(one, multi[:, :, 0])


def test_gqa_above_eight():
    """GQA 16 (two CTAs of 8 q-heads per KV head) on both kernels."""
    for D, P in ((128, 128), (64, 64)):
        n_q, H = 32, 2
        levels = synthetic_levels(1, H, D, 2.5, seed=9)[0]
        k, v = synthetic_kv(1, H, 5 * P, D, seed=9, layer=0, device="cuda")
        n = 4 * P + 17
        cache = PackedKVCache([levels], 1, n_q, H, D, page_size=P, k_group_size=P, v_group_size=D, device="cuda",
                              capacity=5 * P)
        cache.prefill(0, k, v, [n])
        q = torch.randn(1, n_q, D, device="cuda").to(torch.bfloat16)
        out = packed_attention_batched(cache, 0, q, k[:, :, n], v[:, :, n], D ** -0.5, out_dtype=torch.float32)
        want = _oracle(levels, P, D, k[0], v[0], n, q[0][:, None], k[0, :, n:n + 1], v[0, :, n:n + 1], D ** -0.5)
        ok, err, cos = attention_close(out[0].cpu().numpy(), want[:, 0])
        assert ok, (D, err, cos)


def test_manager_api_multi_token():
    """The reference-signature ``packed_attention(manager, ...)`` with q_len > 1
    (reference.py:112-116 routes this to its dense path)."""
    n_q, H, D = 28, 4, 128
    levels = synthetic_levels(1, H, D, 2.5, seed=11)[0]
    k, v = synthetic_kv(1, H, 700, D, seed=11, layer=0, device="cuda")
    mgr = PackedKVManager([torch.as_tensor(levels)], n_q, H, D, 128, 128, 128, 2, "cuda")
    mgr.commit(0, k[:, :, :450], v[:, :, :450])
    q = torch.randn(1, n_q, 24, D, device="cuda").to(torch.bfloat16)
    out = packed_attention(mgr, 0, q, k[:, :, 450:474], v[:, :, 450:474], D ** -0.5)
    assert out.shape == q.shape and out.dtype == torch.bfloat16
    want = _oracle(levels, 128, D, k[0], v[0], 450, q[0], k[0, :, 450:474], v[0, :, 450:474], D ** -0.5)
    got = out[0].float().cpu().numpy()
    assert np.abs(got - want).max() < 2e-3 + 2 ** -8 * np.abs(want).max()  # plus the bf16 output rounding
