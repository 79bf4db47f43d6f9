"""CPU tests of the C ABI and the host logic (no GPU calls).

* the shared library loads and exports every ``LF_API`` symbol of
  ``include/logitfill_b200.h``;
* ``lf_layout_init`` agrees with an independent restatement of the layout
  rules and with the reference's tier widths (layout.py:57,82);
* argument validation returns the documented status codes without touching
  the GPU;
* host tier tables equal the oracle's (layout.py:49-68).
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from logitfill_b200 import _lib
from logitfill_b200.packed.layout import LayerLayout, tier_tables
from logitfill_b200.synthetic import synthetic_levels
from oracle import packed_ref as orc

ROOT = Path(__file__).resolve().parents[1]


def header_symbols() -> list[str]:
    text = (ROOT / "include" / "logitfill_b200.h").read_text()
    return re.findall(r"LF_API\s+[\w\s\*]+?\b(lf_\w+)\s*\(", text)


def test_library_exports_every_header_symbol():
    so = _lib.lib()
    names = header_symbols()
    assert len(names) >= 9
    for name in names:
        assert hasattr(so, name), name
    assert set(names) == set(_lib.EXPORTS)


def _layout_restated(counts, D, P, kg, vg, bit_v):
    bits = (2, 4, 8)
    width = [int(max(counts[t])) for t in range(4)]
    words = [(width[t] + 32 // bits[t] - 1) // (32 // bits[t]) for t in range(3)]
    code_off = [0, words[0], words[0] + words[1]]
    vcode_off = sum(words)
    vcode_words = (D + 32 // bit_v - 1) // (32 // bit_v)
    half_off = vcode_off + vcode_words
    halves = width[3] + 2 * (D // vg)
    row_words = (half_off + (halves + 1) // 2) | 1
    meta = -(-(2 * sum(width[:3]) + 1) // 8) * 8  # scales, mins, then the group's largest scale
    return width, words, code_off, vcode_off, half_off, row_words, meta


@pytest.mark.parametrize("target_bit", [2.25, 2.5, 3.0, 4.0])
def test_layout_init_matches_restatement(target_bit):
    levels = synthetic_levels(1, 4, 128, target_bit, seed=3)[0]
    lay = LayerLayout(levels, head_dim=128, page_size=128, k_group_size=128, v_group_size=128, bit_v=2,
                      row_cap=512, device="cpu")
    table = orc.tier_tables(levels)
    counts = np.stack([table[c]["count"] for c in range(4)])
    width, words, code_off, vcode_off, half_off, row_words, meta = _layout_restated(counts, 128, 128, 128, 128, 2)
    c = lay.c
    assert list(c.width) == width == [table[t]["width"] for t in range(4)]
    assert list(c.words) == words
    assert list(c.code_off) == code_off
    assert (c.vcode_off, c.half_off, c.row_words, c.meta_halves) == (vcode_off, half_off, row_words, meta)
    assert c.row_words % 2 == 1 and c.meta_halves % 8 == 0
    assert c.kmax_off == 2 * sum(width[:3]) and list(c.min_off) == [c.scale_off[t] + width[t] for t in range(3)]
    assert (c.row_cap, c.group_cap) == (512, 4)


def test_layout_init_rejects_bad_arguments():
    so = _lib.lib()
    out = _lib.LfLayout()
    counts = np.array([[64], [32], [16], [16]], np.int32)
    assert so.lf_layout_init(ctypes.byref(out), 1, 128, 128, 96, 128, 2, counts.ctypes.data, 128, 1) \
        == _lib.LF_ERR_INVALID_ARGUMENT   # page not a multiple of k_group
    assert so.lf_layout_init(ctypes.byref(out), 1, 128, 128, 128, 128, 3, counts.ctypes.data, 128, 1) \
        == _lib.LF_ERR_UNSUPPORTED        # bit_v 3 is not a packed width
    bad = np.array([[64], [32], [16], [15]], np.int32)
    assert so.lf_layout_init(ctypes.byref(out), 1, 128, 128, 128, 128, 2, bad.ctypes.data, 128, 1) \
        == _lib.LF_ERR_INVALID_ARGUMENT   # counts do not cover head_dim
    assert b"head" in so.lf_last_error()
    with pytest.raises(ValueError):
        _lib.check(_lib.LF_ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.LF_ERR_UNSUPPORTED, "x")


def test_entry_points_validate_before_launch():
    """Null or inconsistent arguments are rejected on the host, no GPU needed."""
    so = _lib.lib()
    assert so.lf_pack_pages(None, None, None, 2, 0, 0, 0, None, 1, 1, None, None, None, None, None) \
        == _lib.LF_ERR_INVALID_ARGUMENT
    lay = LayerLayout(np.zeros((2, 64), np.int64), head_dim=64, page_size=64, k_group_size=64,
                      v_group_size=64, bit_v=2, row_cap=256, device="cpu")
    fake = 1 << 20  # never dereferenced: validation fails first
    # max_splits too small for the capacity
    st = so.lf_decode_partial(ctypes.byref(lay.c), fake, fake, fake, fake, fake, fake, 0, 0, fake, 2, None, None,
                              0, 0, fake, 2, 0, 0, 1, 2, 1.0, 1, 1, fake, None, None)
    assert st == _lib.LF_ERR_INVALID_ARGUMENT
    # GQA group of 16 exceeds what one CTA computes
    st = so.lf_decode_partial(ctypes.byref(lay.c), fake, fake, fake, fake, fake, fake, 0, 0, fake, 2, None, None,
                              0, 0, fake, 2, 0, 0, 1, 32, 1.0, 1, 10, fake, None, None)
    assert st == _lib.LF_ERR_UNSUPPORTED
    assert so.lf_decode_merge(None, None, 1, 1, 1, 64, 64, 1, 1, None, 0, 0, 0, None) == _lib.LF_ERR_INVALID_ARGUMENT
    # K2 writes partials for head_dim <= 128 only; the merge refuses larger ones
    assert so.lf_decode_merge(fake, fake, 1, 1, 1, 256, 128, 1, 1, fake, 2, 0, 0, None) == _lib.LF_ERR_UNSUPPORTED
    assert so.lf_decode_max_splits(256, 16, 128) == 16 + 4
    assert so.lf_decode_max_splits_multi(256, 16, 128, 1) == 16 + 4
    assert so.lf_decode_max_splits_multi(256, 16, 128, 16) == 16 + 5   # 127 tail + 16 new rows
    assert so.lf_decode_max_splits_multi(256, 16, 128, 0) == 0
    assert so.lf_decode_workspace_bytes(2, 4, 28, 128, 5) == 2 * 4 * 5 * 7 * 130 * 4


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_tier_tables_match_oracle(seed):
    rng = np.random.default_rng(seed)
    levels = rng.integers(0, 4, size=(3, 64))
    levels[1] = 0   # a head with a single tier
    ours = tier_tables(torch.as_tensor(levels))
    ref = orc.tier_tables(levels)
    for code in range(4):
        for key in ("index", "count", "local"):
            np.testing.assert_array_equal(ours["tiers"][code][key].numpy(), ref[code][key])
        assert ours["tiers"][code]["width"] == ref[code]["width"]
    np.testing.assert_array_equal(ours["tier"].numpy(), ref["tier"])


def test_head_chunks():
    """(q-head, query token) pairs per K2 CTA: the largest divisor <= 8."""
    from logitfill_b200.packed.attention import chunk_heads

    assert [chunk_heads(7, 1), chunk_heads(7, 2), chunk_heads(7, 16), chunk_heads(16, 1)] == [7, 7, 8, 8]
    assert [chunk_heads(5, 3), chunk_heads(1, 11), chunk_heads(1, 1), chunk_heads(3, 4)] == [5, 1, 1, 6]


def test_device_tables_are_int32_and_match_the_loop_construction():
    """The kernels read chan_code [H][D] and slot_chan [4][H][D] as int32:
    the vectorised TierTables give exactly the per-head construction
    (channel list of each tier in ascending order), in int32."""
    from logitfill_b200.policy import TierTables

    for seed, (H, D) in enumerate([(4, 128), (2, 64), (3, 8)]):
        levels = np.random.default_rng(seed).integers(0, 4, size=(H, D))
        tt = TierTables(levels, "cpu")
        assert tt.chan_code.dtype == torch.int32 and tt.slot_chan.dtype == torch.int32
        assert tt.counts.dtype == np.int32
        ref = orc.tier_tables(levels)
        chan_code = np.zeros((H, D), np.int32)
        slot_chan = np.full((4, H, D), -1, np.int32)
        for t in range(4):
            for h in range(H):
                n = int(ref[t]["count"][h])
                idx = ref[t]["index"][h, :n]
                slot_chan[t, h, :n] = idx
                chan_code[h, idx] = (t << 16) | np.arange(n)
        assert np.array_equal(tt.chan_code.numpy(), chan_code)
        assert np.array_equal(tt.slot_chan.numpy(), slot_chan)
