"""K1's per-element division against IEEE division, bit for bit, on millions
of operand pairs.

K1 forms every code as clamp(round_half_even((x - lo) / scale), 0, 2^b - 1)
(layout.py:12-18) but divides by Markstein's method (RN(1/scale), one
product, an exact FMA residual and one corrective FMA) instead of an IEEE
division.  ``lf_selftest_divide`` runs that exact device routine on given
(x, lo, scale) triples, in both forms K1 uses: one element at a time, and two
elements in packed fp32x2 arithmetic (an element whose two codes differ
comes back as -1).  This test compares its quotients and codes with numpy's
float32 IEEE subtract and divide (round to nearest even) on seeded sweeps:

* operands as K1 sees them: bf16 x and lo, scale = clamp(RN((hi - lo) / qmax),
  1e-5, 1e5) for 2-, 4- and 8-bit tiers;
* scales with all-ones significands across the clamp range;
* scales at the clamps 1e-5 and 1e5;
* dividends that put the quotient within 3 ulps of every half integer
  0.5 .. qmax - 0.5 (the rounding boundaries of the codes);
* large and tiny magnitudes, zero, and infinite differences (codes only).

Quotients are compared where the IEEE quotient is normal (a smaller one rounds
to code 0 either way); codes are compared everywhere.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from logitfill_b200 import _lib

pytestmark = pytest.mark.gpu
N = 1 << 20
TINY = np.float32(2.0 ** -126)


def _bf16(a: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (nearest even) and back."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16
    return u.astype(np.uint32).view(np.float32)


def _device(x, lo, scale, bits):
    t = [torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda() for a in (x, lo, scale)]
    q = torch.empty_like(t[0])
    c = torch.empty(t[0].shape, dtype=torch.int32, device="cuda")
    _lib.check(_lib.lib().lf_selftest_divide(_lib.ptr(t[0]), _lib.ptr(t[1]), _lib.ptr(t[2]), t[0].numel(), bits,
                                             _lib.ptr(q), _lib.ptr(c), _lib.stream_handle(q.device)),
               "lf_selftest_divide")
    torch.cuda.synchronize()
    return q.cpu().numpy(), c.cpu().numpy().astype(np.int64)


def _ieee(x, lo, scale, bits):
    with np.errstate(all="ignore"):
        q = (x.astype(np.float32) - lo.astype(np.float32)) / scale.astype(np.float32)
        c = np.clip(np.rint(q), 0, (1 << bits) - 1)
    return q.astype(np.float32), c


def _compare(x, lo, scale, bits, what):
    q, c = _device(x, lo, scale, bits)
    qr, cr = _ieee(x, lo, scale, bits)
    normal = np.isfinite(qr) & (np.abs(qr) >= TINY)
    bad_q = normal & (q.view(np.uint32) != qr.view(np.uint32))
    assert not bad_q.any(), (what, bits, int(bad_q.sum()), x[bad_q][:4], lo[bad_q][:4], scale[bad_q][:4])
    bad_c = c != cr
    assert not bad_c.any(), (what, bits, int(bad_c.sum()), x[bad_c][:4], lo[bad_c][:4], scale[bad_c][:4])
    return int(normal.sum())


def _scale_of(hi, lo, bits):
    with np.errstate(all="ignore"):
        s = (hi.astype(np.float32) - lo.astype(np.float32)) / np.float32((1 << bits) - 1)
    return np.clip(s, np.float32(1e-5), np.float32(1e5)).astype(np.float32)


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_pack_operands(bits):
    """bf16 x in [lo, hi], scale from the group's range, many magnitudes."""
    rng = np.random.default_rng(100 + bits)
    mag = np.float32(10.0) ** rng.uniform(-6, 6, N).astype(np.float32)
    lo = _bf16(-mag * rng.random(N, dtype=np.float32))
    hi = _bf16(lo + mag * rng.random(N, dtype=np.float32) * np.float32(2))
    x = _bf16(lo + (hi - lo) * rng.random(N, dtype=np.float32))
    x = np.maximum(np.minimum(x, hi), lo)
    assert _compare(x, lo, _scale_of(hi, lo, bits), bits, "pack operands") > N // 2


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_all_ones_significands_and_clamps(bits):
    rng = np.random.default_rng(200 + bits)
    qmax = (1 << bits) - 1
    e = rng.integers(-17, 17, N)                      # 2^-17 .. 2^16 covers [1e-5, 1e5]
    ones = (((e + 127) << 23) | 0x7FFFFF).astype(np.uint32).view(np.float32)
    ones = np.clip(ones, np.float32(1e-5), np.float32(1e5)).astype(np.float32)
    clamps = np.where(rng.random(N) < 0.5, np.float32(1e-5), np.float32(1e5)).astype(np.float32)
    for scale, what in ((ones, "all-ones significand"), (clamps, "clamp")):
        d = (scale * np.float32(qmax) * rng.random(N, dtype=np.float32) * np.float32(1.02)).astype(np.float32)
        lo = np.where(rng.random(N) < 0.5, np.float32(0), _bf16(-d * rng.random(N, dtype=np.float32)))
        x = (lo + d).astype(np.float32)
        assert _compare(x, lo.astype(np.float32), scale, bits, what) > N // 2


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_half_integer_boundaries(bits):
    """Quotients within 3 ulps of every half integer k + 0.5, k < qmax."""
    rng = np.random.default_rng(300 + bits)
    qmax = (1 << bits) - 1
    k = rng.integers(0, qmax, N).astype(np.float32)
    exps = rng.integers(-17, 17, N)
    mant = rng.integers(0, 1 << 23, N)
    mant[: N // 8] = 0x7FFFFF                          # all-ones significands among them
    scale = (((exps + 127) << 23) | mant).astype(np.uint32).view(np.float32)
    scale = np.clip(scale, np.float32(1e-5), np.float32(1e5)).astype(np.float32)
    d = ((k + np.float32(0.5)) * scale).astype(np.float32)
    steps = rng.integers(-3, 4, N)
    du = d.view(np.int32) + steps.astype(np.int32)
    d = du.view(np.float32)
    lo = np.zeros(N, np.float32)
    _compare(d, lo, scale, bits, "half integers")
    # the same boundaries reached through a non-zero lo (x - lo exact)
    lo2 = -np.float32(2.0) ** rng.integers(-4, 4, N).astype(np.float32)
    x2 = (d + lo2).astype(np.float32)
    exact = (x2 - lo2) == d
    _compare(x2[exact], lo2[exact], scale[exact], bits, "half integers, lo != 0")


def test_special_differences():
    """Zero, subnormal and infinite differences: codes as IEEE division gives them."""
    scale = np.array([1e-5, 1.0, 1e5, 3.0, 1e-5, 1e5, 7.5], np.float32)
    x = np.array([0.0, 1e-40, 1e-40, np.inf, 3e38, 3e38, 2.5], np.float32)
    lo = np.array([0.0, 0.0, 0.0, 0.0, -3e38, 0.0, 2.5], np.float32)
    for bits in (2, 4, 8):
        _compare(x, lo, scale, bits, "special")
