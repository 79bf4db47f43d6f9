"""Pin the numpy oracle to the reference's own outputs (CPU only).

The fixtures in ``tests/golden/`` were produced by ``make_golden.py`` running
the reference packer (``src/logitfill/packed/layout.py``), its history store
(``cache.py``) and its dense attention (``reference.py:30-56``).  Packing and
the dequantized round trip must match bit for bit; attention within 1e-5.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import packed_ref as orc
from tests.golden import cases
from tests.oracle_runner import run_case, small_case

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def small():
    return dict(np.load(GOLDEN / "golden_small.npz"))


@pytest.fixture(scope="module")
def big():
    return dict(np.load(GOLDEN / "golden_config0.npz"))


def _bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint8) if a.dtype != np.bool_ else a


def assert_bit_equal(a, b, what=""):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape, (what, a.shape, b.shape)
    assert a.dtype == b.dtype, (what, a.dtype, b.dtype)
    assert np.array_equal(_bits(a), _bits(b)), what


def test_layout_round_trip_matches_reference(small):
    """Reference unit test shape (tests/test_logitfill_offline.py:127-145)."""
    page = small["layout_page"]
    table = orc.tier_tables(np.zeros((2, 8), np.int64))
    pk = orc.quantize_key_page(page, table, 8)
    pv = orc.quantize_value_page(page, 2, 8)
    for name in ("code", "scale", "min"):
        assert_bit_equal(pk[0][name], small[f"layout_k0_{name}"], f"k {name}")
        assert_bit_equal(pv[name], small[f"layout_v_{name}"], f"v {name}")
    assert_bit_equal(orc.dequantize_key(16, table, pk, 8), small["layout_deq_k"], "deq k")
    assert_bit_equal(orc.dequantize_value(pv, 16, 8, 2, 8), small["layout_deq_v"], "deq v")


@pytest.mark.parametrize("name", ["cuda", "mixed"])
def test_small_cases_match_reference(small, name):
    res = run_case(small_case(small, name))
    for key, arr in res.items():
        ref = small[f"{name}_{key}"]
        if key == "attn":
            np.testing.assert_allclose(arr, ref, atol=1e-5, rtol=0)
        else:
            assert_bit_equal(arr, ref, f"{name} {key}")


def test_pack_edge_page_matches_reference(small):
    edge = cases.pack_edge_page()
    assert [cases.sha(edge["k"]), cases.sha(edge["v"])] == list(small["edge_input_sha"])
    table = orc.tier_tables(edge["levels"])
    pk = orc.quantize_key_page(edge["k"], table, 128)
    pv = orc.quantize_value_page(edge["v"], 2, 128)
    for code in (0, 1, 2):
        for name in ("code", "scale", "min"):
            assert_bit_equal(pk[code][name], small[f"edge_k{code}_{name}"], f"edge k{code} {name}")
    assert_bit_equal(pk[3]["value"], small["edge_k3_value"], "edge fp16 tier")
    for name in ("code", "scale", "min"):
        assert_bit_equal(pv[name], small[f"edge_v_{name}"], f"edge v {name}")


@pytest.mark.parametrize("name", sorted(cases.CONFIG0_VARIANTS))
def test_config0_cases_match_reference(big, name):
    hist, tail = cases.CONFIG0_VARIANTS[name]
    case = cases.config0_like(hist, tail)
    want_inputs = list(big[f"{name}_input_sha"])
    got_inputs = ([cases.sha(case["levels"]), cases.sha(case["query"])]
                  + [cases.sha(k) for k, _ in case["commits"]] + [cases.sha(v) for _, v in case["commits"]])
    assert got_inputs == want_inputs, "seeded input generator drifted; regenerate the fixtures"
    res = run_case(case)
    assert int(res["hist_len"]) == int(big[f"{name}_hist_len"])
    assert int(res["tail_len"]) == int(big[f"{name}_tail_len"])
    for key, arr in res.items():
        if key in ("attn", "hist_len", "tail_len"):
            continue
        assert cases.sha(arr) == str(big[f"{name}_{key}_sha"]), f"{name} {key}"
    np.testing.assert_allclose(res["attn"], big[f"{name}_attn"], atol=1e-5, rtol=0)


def test_oracle_pack_roundtrip_property():
    """Unpack(pack(codes)) is the identity for every tier width."""
    rng = np.random.default_rng(3)
    for bits in (2, 4, 8):
        for n in (0, 1, 15, 16, 17, 88, 128):
            codes = rng.integers(0, 1 << bits, size=(3, 5, n))
            packed = orc.pack_ints(codes, bits)
            assert packed.shape[-1] == (n * bits + 31) // 32
            np.testing.assert_array_equal(orc.unpack_ints(packed, n, bits), codes)


def test_torch_port_matches_reference_outputs(small, big):
    """The torch restatement of reference.py:30-56 (what the CPU baseline
    times) reproduces the reference's own stored attention outputs."""
    from oracle import packed_ref_torch as orct
    from tests.oracle_runner import oracle_layer_for

    for name in ("cuda", "mixed"):
        case = small_case(small, name)
        layer = oracle_layer_for(case)
        got = orct.reference_attention(layer, case["query"], case["key_new"], case["value_new"], case["scaling"])
        assert np.allclose(got.numpy(), small[f"{name}_attn"], atol=1e-5, rtol=1e-5), name
    case = cases.config0_like(1024, 37)
    layer = oracle_layer_for(case)
    got = orct.reference_attention(layer, case["query"], case["key_new"], case["value_new"], case["scaling"])
    assert np.allclose(got.numpy(), big["config0_attn"], atol=1e-5, rtol=1e-5)
    # the dequantized history equals the numpy oracle's bit for bit
    kt = orct.dequantize_key(layer.hist_len, layer.table, layer.hist_k, layer.k_group_size).numpy()
    kn, vn = layer.dequantize()
    vt = orct.dequantize_value(layer.hist_v, layer.hist_len, 128, 2, 128).numpy()
    assert_bit_equal(kt, kn, "torch deq k")
    assert_bit_equal(vt, vn, "torch deq v")
