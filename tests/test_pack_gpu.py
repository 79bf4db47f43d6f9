"""GPU parity of K1 (page quantize+pack) and the dequantizer against the oracle.

Bit-exact: packed codes, fp16 scale/min bytes, the FP16 Key tier, Value
codes/scale/min, and the dequantized round trip (layout.py:71-182), read back
through the reference-shaped views of the B200 store.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from logitfill_b200.packed.layout import quantize_key_page, quantize_value_page, tier_tables
from logitfill_b200.synthetic import synthetic_kv, synthetic_levels
from oracle import packed_ref as orc
from tests.golden import cases
from tests.gpu_cases import bit_equal, manager_for, store_arrays
from tests.oracle_runner import layer_arrays, oracle_layer_for, small_case

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def small():
    return dict(np.load(GOLDEN / "golden_small.npz"))


def _check_store(mgr, case):
    ref = oracle_layer_for(case)
    got = store_arrays(mgr.layers[0])
    want = layer_arrays(ref)
    assert set(got) == set(want)
    for key in want:
        assert bit_equal(got[key], want[key]), key
    assert mgr.layers[0].hist_len == ref.hist_len and mgr.layers[0].tail_len == ref.tail_len
    if ref.tail_k is not None:
        np.testing.assert_array_equal(mgr.layers[0].tail_k.float().cpu().numpy(), ref.tail_k)
    k, v = mgr.layers[0].dequantize()
    rk, rv = ref.dequantize()
    assert bit_equal(k.cpu().numpy(), rk) and bit_equal(v.cpu().numpy(), rv)


def test_reference_unit_case_layout(small):
    """tests/test_logitfill_offline.py:127-145 through the reference-signature API."""
    page = torch.as_tensor(small["layout_page"]).cuda()
    built = tier_tables(torch.zeros(2, 8, dtype=torch.int64))
    table = built["tiers"]
    table["tier"] = built["tier"]
    pk = quantize_key_page(page, table, group_size=8)
    pv = quantize_value_page(page, bits=2, group_size=8)
    for name in ("code", "scale", "min"):
        assert bit_equal(pk[0][name].cpu().numpy(), small[f"layout_k0_{name}"]), name
        assert bit_equal(pv[name].cpu().numpy(), small[f"layout_v_{name}"]), name


def test_pack_edge_page(small):
    edge = cases.pack_edge_page()
    built = tier_tables(torch.as_tensor(edge["levels"]))
    table = built["tiers"]
    table["tier"] = built["tier"]
    page = torch.as_tensor(edge["k"]).to(torch.bfloat16).cuda()
    vpage = torch.as_tensor(edge["v"]).to(torch.bfloat16).cuda()
    pk = quantize_key_page(page, table, 128)
    pv = quantize_value_page(vpage, 2, 128)
    for code in (0, 1, 2):
        for name in ("code", "scale", "min"):
            assert bit_equal(pk[code][name].cpu().numpy(), small[f"edge_k{code}_{name}"]), (code, name)
    assert bit_equal(pk[3]["value"].cpu().numpy(), small["edge_k3_value"])
    for name in ("code", "scale", "min"):
        assert bit_equal(pv[name].cpu().numpy(), small[f"edge_v_{name}"]), name


@pytest.mark.parametrize("name", ["cuda", "mixed"])
def test_small_cases_store(small, name):
    case = small_case(small, name)
    _check_store(manager_for(case), case)


@pytest.mark.parametrize("name", sorted(cases.CONFIG0_VARIANTS))
def test_config0_store(name):
    hist, tail = cases.CONFIG0_VARIANTS[name]
    case = cases.config0_like(hist, tail)
    _check_store(manager_for(case), case)


def test_group_max_scale_field():
    """K1 also writes, at ``kmax_off`` of each meta row, the Key group's
    largest stored INT2/INT4/INT8 scale over the head's channels (the decode
    kernel's fixed-point exponent for the page): checked against the oracle's
    scales, padding channels excluded."""
    case = cases.config0_like(1024, 37)
    mgr = manager_for(case)
    ref = oracle_layer_for(case)
    layer = mgr.cache.layers[0]
    off = int(layer.layout.c.kmax_off)
    got = layer.kmeta[0, :, : ref.hist_len // 128, off].cpu().numpy().view(np.uint16)
    H = got.shape[0]
    want = np.zeros_like(got)
    for h in range(H):
        for code in range(3):
            cnt = int(ref.table[code]["count"][h])
            if cnt:
                sc = np.asarray(ref.hist_k[code]["scale"], np.float16)[h, :cnt].view(np.uint16)  # [cnt, G]
                want[h] = np.maximum(want[h], sc.max(axis=0))
    np.testing.assert_array_equal(got, want)


def test_capacity_growth_keeps_history():
    """Commits beyond the initial capacity reallocate and keep every byte."""
    case = cases.config0_like(1024, 37)
    mgr = manager_for(case, capacity=128)
    assert mgr.cache.row_cap >= 1024  # packed pages only; the tail lives in the residual page
    _check_store(mgr, case)


@pytest.mark.parametrize("dtype", ["float32", "float16"])
def test_other_input_dtypes(dtype):
    rng = np.random.default_rng(7)
    k = rng.standard_normal((2, 300, 64), dtype=np.float32)
    v = rng.standard_normal((2, 300, 64), dtype=np.float32)
    if dtype == "float16":
        k, v = k.astype(np.float16).astype(np.float32), v.astype(np.float16).astype(np.float32)
    case = {"dtype": dtype, "n_q": 4, "n_kv": 2, "head_dim": 64, "page": 64, "k_group": 32, "v_group": 32,
            "levels": rng.integers(0, 4, size=(2, 64)), "commits": [(k[:, :70], v[:, :70]), (k[:, 70:], v[:, 70:])]}
    _check_store(manager_for(case), case)


def test_prefill_pack_full_size_sampled():
    """Config-3 geometry (28 layers x B 16 x 4096-token prefill -> 32 pages):
    two sampled (sequence, layer) pairs bit-exact against the oracle, and the
    batched prefill equals per-sequence commits byte for byte."""
    from logitfill_b200.packed import PackedKVCache

    B, H, T, D = 16, 4, 4096, 128
    levels = synthetic_levels(28, H, D, 2.5, seed=3)
    for layer in (0, 27):
        k, v = synthetic_kv(B, H, T, D, seed=3, layer=layer, device="cuda")
        cache = PackedKVCache([levels[layer]], B, 28, H, D, device="cuda", capacity=T)
        cache.commit(0, k, v)
        for b in (0, B - 1):
            ref = orc.OracleLayer(levels[layer], 128, 128, 128, 2)
            ref.append(k[b].float().cpu().numpy(), v[b].float().cpu().numpy())
            from logitfill_b200.packed.cache import _LayerStore
            got = store_arrays(_LayerStore(cache, 0, b))
            want = layer_arrays(ref)
            for key in want:
                assert bit_equal(got[key], want[key]), (layer, b, key)
        one = PackedKVCache([levels[layer]], B, 28, H, D, device="cuda", capacity=T)
        for b in range(B):
            one.commit(0, k[b:b + 1], v[b:b + 1], seqs=[b])
        assert torch.equal(one.layers[0].rows, cache.layers[0].rows)
        assert torch.equal(one.layers[0].kmeta.view(torch.int16), cache.layers[0].kmeta.view(torch.int16))


def test_decode_flush_sequence():
    """Token-by-token commits (256 decode steps after a 4096-token prefill,
    flushing at every 128th) give the same store as one bulk commit."""
    from logitfill_b200.packed import PackedKVCache

    B, H, D = 2, 4, 128
    levels = synthetic_levels(1, H, D, 2.5, seed=4)[0]
    k, v = synthetic_kv(B, H, 4096 + 256, D, seed=4, layer=0, device="cuda")
    step = PackedKVCache([levels], B, 28, H, D, device="cuda", capacity=4096)
    step.commit(0, k[:, :, :4096], v[:, :, :4096])
    for t in range(4096, 4096 + 256):
        step.commit(0, k[:, :, t:t + 1], v[:, :, t:t + 1])
    bulk = PackedKVCache([levels], B, 28, H, D, device="cuda", capacity=8192)
    bulk.commit(0, k, v)
    n = 4096 + 256
    assert step.layers[0].hist_len.tolist() == [n, n] and step.layers[0].tail_len.tolist() == [0, 0]
    assert torch.equal(step.layers[0].rows[:, :, :n], bulk.layers[0].rows[:, :, :n])
    g = n // 128
    assert torch.equal(step.layers[0].kmeta[:, :, :g].view(torch.int16), bulk.layers[0].kmeta[:, :, :g].view(torch.int16))


def test_codes_at_rounding_boundaries():
    """Quotients (x - min) / scale placed within a few ulps of every half
    integer, where rounding the quotient differently would flip the code: K1
    (which divides by Markstein's method, RN(1/scale) and one FMA correction)
    must give the oracle's IEEE-division codes bit for bit, for the Key tiers
    and the Value codes."""
    rng = np.random.default_rng(11)
    H, D, P = 2, 64, 64
    levels = np.tile(np.repeat(np.array([0, 1, 2, 3]), D // 4), (H, 1))
    k = np.zeros((H, P, D), np.float32)
    v = np.zeros((H, P, D), np.float32)
    ulp_steps = np.array([-3, -2, -1, 0, 1, 2, 3], np.float32)
    for h in range(H):
        for c in range(D):
            bits = (2, 4, 8, 8)[levels[h, c]]
            qmax = np.float32(2 ** bits - 1)
            hi = np.float32(rng.uniform(0.5, 40.0))
            scale = np.float32(hi / qmax)
            k[h, 0, c], k[h, 1, c] = 0.0, hi
            half = (rng.integers(0, int(qmax), P - 2) + np.float32(0.5)).astype(np.float32)
            x = (half * scale).astype(np.float32)
            step = ulp_steps[rng.integers(0, len(ulp_steps), P - 2)]
            k[h, 2:, c] = x + step * np.spacing(x).astype(np.float32)
        for t in range(P):
            hi = np.float32(rng.uniform(0.5, 40.0))
            scale = np.float32(hi / np.float32(3))
            v[h, t, 0], v[h, t, 1] = 0.0, hi
            half = (rng.integers(0, 3, D - 2) + np.float32(0.5)).astype(np.float32)
            x = (half * scale).astype(np.float32)
            step = ulp_steps[rng.integers(0, len(ulp_steps), D - 2)]
            v[h, t, 2:] = x + step * np.spacing(x).astype(np.float32)
    k, v = k.astype(np.float32), v.astype(np.float32)
    case = {"dtype": "float32", "n_q": 2, "n_kv": H, "head_dim": D, "page": P, "k_group": P, "v_group": D,
            "levels": levels, "commits": [(k, v)]}
    _check_store(manager_for(case), case)
