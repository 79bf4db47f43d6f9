"""Seeded inputs of the golden parity cases.

Shared by ``make_golden.py`` (which runs the reference on them, in a checkout
that has the reference importable) and by the tests (which run the oracle and
the CUDA path on them).  Inputs are either stored in the fixture (tiny cases
whose reference inputs come from torch's generator) or rebuilt here from numpy
PCG64 streams; ``golden_*.npz`` stores a SHA-256 of every rebuilt input so a
drifting generator is caught instead of silently changing the cases.

Each case is a single sequence: ``levels [n_kv, D]``, a list of commits (each
``[n_kv, T, D]`` Key/Value in the case's dtype, given as float32 values that
are exact in that dtype), then one decode query ``[n_q, 1, D]`` with the new
token's Key/Value ``[n_kv, 1, D]``.
"""
from __future__ import annotations

import hashlib

import numpy as np

from logitfill_b200.synthetic import outlier_channels, synthetic_levels


def sha(a: np.ndarray) -> str:
    a = np.ascontiguousarray(a)
    return hashlib.sha256(str(a.dtype).encode() + str(a.shape).encode() + a.tobytes()).hexdigest()


def _bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 value (RNE), returned as float32."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def config0_like(history: int = 1024, tail: int = 37, *, seed: int = 0, n_q: int = 28, n_kv: int = 4,
                 head_dim: int = 128, page: int = 128, target_bit: float = 2.5) -> dict:
    """one layer, batch 1, 28 q / 4 kv heads, D 128, a
    ``history``-token packed history plus a ``tail``-token bf16 residual and
    one new token; bf16 K/V ~ N(0,1) with 5 % outlier Key channels x10;
    policy seeded at ``target_bit``; bf16 query ~ N(0,1)."""
    rng = np.random.default_rng([seed, history, tail, 2024])
    total = history + tail + 1
    k = rng.standard_normal((n_kv, total, head_dim), dtype=np.float32)
    v = rng.standard_normal((n_kv, total, head_dim), dtype=np.float32)
    for h in range(n_kv):
        k[h][:, outlier_channels(seed, 0, h, head_dim)] *= 10.0
    k, v = _bf16_round(k), _bf16_round(v)
    q = _bf16_round(rng.standard_normal((n_q, 1, head_dim), dtype=np.float32))
    levels = synthetic_levels(1, n_kv, head_dim, target_bit, seed=seed)[0]
    body = history + tail
    return {
        "dtype": "bfloat16", "n_q": n_q, "n_kv": n_kv, "head_dim": head_dim, "page": page,
        "k_group": page, "v_group": head_dim, "levels": levels,
        "commits": [(k[:, :body], v[:, :body])] if body else [],
        "query": q, "key_new": k[:, body:], "value_new": v[:, body:],
        "scaling": head_dim ** -0.5,
    }


def pack_edge_page(seed: int = 5) -> dict:
    """One 128-token page exercising the packer's corner cases: a constant
    channel (range 0 -> scale clamped to 1e-5), exact rounding ties for each
    tier (range = 2^b - 1 so scale = 1 and x - min lands on k + 0.5), tiny and
    large magnitudes, negative values, an FP16-tier channel that overflows fp16."""
    rng = np.random.default_rng(seed)
    n_kv, page, d = 2, 128, 128
    k = rng.standard_normal((n_kv, page, d), dtype=np.float32)
    v = rng.standard_normal((n_kv, page, d), dtype=np.float32)
    levels = rng.integers(0, 4, size=(n_kv, d))
    for h in range(n_kv):
        k[h, :, 3] = 1.25                      # constant channel
        for c, b in ((10, 2), (11, 4), (12, 8)):
            levels[h, c] = {2: 0, 4: 1, 8: 2}[b]
            qmax = (1 << b) - 1
            col = rng.integers(0, qmax, size=page).astype(np.float32) + 0.5
            col[0], col[1] = 0.0, float(qmax)  # pin min / max -> scale 1
            k[h, :, c] = col
        k[h, :, 20] *= 1e-3
        k[h, :, 21] *= 3e3
        levels[h, 22] = 3
        k[h, :, 22] = 7e4 * np.sign(k[h, :, 22])   # beyond fp16 range
        v[h, 5, :] = 0.5                        # constant token row
        v[h, 6, :] = rng.integers(0, 3, size=d) + 0.5
        v[h, 6, 0], v[h, 6, 1] = 0.0, 3.0      # exact ties along channels
    return {"dtype": "bfloat16", "n_kv": n_kv, "head_dim": d, "page": page, "k_group": page,
            "v_group": d, "levels": levels, "k": _bf16_round(k), "v": _bf16_round(v)}


CONFIG0_VARIANTS = {
    # name: (history tokens, tail tokens)
    "config0": (1024, 37),
    "config0_tail0": (1024, 0),
    "config0_tail127": (1024, 127),
    "config0_nohist": (0, 37),
    "config0_onepage": (128, 1),
}
