"""Seeded synthetic Key/Value histories and Key-tier policies.

The reference measures on a model checkpoint and Long-CoT data that are not
available; these generators stand in for them with the shapes, sizes and
value distributions the benchmark configurations name:

* K, V ~ N(0, 1) stored in bf16; in every (layer, kv-head) 6 of 128 Key
  channels (5 %) are outlier channels scaled x10.
* The Key policy comes from the reference's greedy reverse water-filling
  allocator (``src/logitfill/allocators/allocate.py:91-135``, restated in
  :func:`waterfill`) run on seeded monotone distortion curves
  ``d8 = U, d4 = d8 + U, d2 = d4 + U`` (the curve form of
  ``exp/ablation/run_ablation.py:56-61``).  The outlier channels' d2/d4 are
  multiplied by 1000 and d8 of three of them as well, so all four tiers
  (INT2/INT4/INT8/FP16) occur.  At ``target_bit`` 2.5 this gives per head
  88 x INT2, 34 x INT4, 3 x INT8, 3 x FP16 (mean Key 3.0 bit).
* The per-head extra-bit budget is ``kv_history_budget`` of
  ``allocate.py:26-53``: ``round((2 * target_bit - bit_v - 2) * head_dim)``.
"""
from __future__ import annotations

import numpy as np

LEVEL_BITS = np.array([2, 4, 8, 16], dtype=np.int64)
N_OUTLIERS = 6


def extra_budget_per_head(target_bit: float, bit_v: int = 2, n_channels: int = 128) -> int:
    """allocate.py:14-19,26-53: Key bits per head above the INT2 floor."""
    target_k = 2.0 * float(target_bit) - float(bit_v)
    if target_k < 2.0 or target_k > 16.0:
        raise ValueError(f"target_bit {target_bit} with bit_v {bit_v} implies Key target {target_k}")
    return int(round((target_k - 2.0) * n_channels))


def waterfill(d2: np.ndarray, d4: np.ndarray, d8: np.ndarray, extra: int) -> np.ndarray:
    """allocate.py:91-123, vectorised.

    Greedy marginal purchase: repeatedly upgrade the channel whose next step
    (2->4 costs 2 bits, 4->8 costs 4, 8->16 costs 8) has the largest
    distortion drop per bit, scanning steps in that order and channels in
    index order, first strict maximum wins, while the budget allows it."""
    hi = np.maximum(np.asarray(d2, np.float64), 0.0)
    mid = np.minimum(np.maximum(np.asarray(d4, np.float64), 0.0), hi)
    lo = np.minimum(np.maximum(np.asarray(d8, np.float64), 0.0), mid)
    drops = np.stack([hi - mid, mid - lo, lo])  # [3, n]
    costs = np.array([2, 4, 8])
    n = hi.shape[0]
    level = np.zeros(n, dtype=np.int64)
    spent = 0
    while True:
        gains = np.full((3, n), -np.inf)
        for step in range(3):
            ok = (level == step) & (spent + costs[step] <= extra) & (drops[step] > 0)
            gains[step, ok] = drops[step, ok] / costs[step]
        flat = gains.reshape(-1)
        best = int(np.argmax(flat))
        if not flat[best] > 0.0:
            break
        step, i = divmod(best, n)
        level[i] += 1
        spent += int(costs[step])
    return level


def outlier_channels(seed: int, layer: int, head: int, head_dim: int = 128) -> np.ndarray:
    """The 5 % outlier Key channels of one (layer, kv-head), sorted."""
    rng = np.random.default_rng([int(seed), 7919, int(layer), int(head)])
    n = max(1, round(N_OUTLIERS * head_dim / 128))
    return np.sort(rng.choice(head_dim, size=n, replace=False))


def synthetic_levels(n_layers: int, n_kv: int, head_dim: int, target_bit: float,
                     seed: int = 0, bit_v: int = 2) -> np.ndarray:
    """Key tier policy ``[n_layers, n_kv, head_dim]`` (0=INT2 .. 3=FP16)."""
    extra = extra_budget_per_head(target_bit, bit_v, head_dim)
    levels = np.zeros((n_layers, n_kv, head_dim), dtype=np.int64)
    for layer in range(n_layers):
        for head in range(n_kv):
            rng = np.random.default_rng([int(seed), 104729, layer, head])
            draw = rng.random((3, head_dim))
            d8 = draw[0]
            d4 = d8 + draw[1]
            d2 = d4 + draw[2]
            out = outlier_channels(seed, layer, head, head_dim)
            d2[out] *= 1000.0
            d4[out] *= 1000.0
            d8[out[: len(out) // 2]] *= 1000.0
            levels[layer, head] = waterfill(d2, d4, d8, extra)
    return levels


def mean_key_bits(levels: np.ndarray) -> float:
    return float(LEVEL_BITS[np.asarray(levels)].mean())


def synthetic_kv(batch: int, n_kv: int, tokens: int, head_dim: int, *, seed: int, layer: int,
                 device="cpu", dtype=None):
    """Seeded K, V ``[batch, n_kv, tokens, head_dim]`` in ``dtype`` (bf16 by
    default) with the layer's outlier Key channels scaled x10."""
    import torch

    dtype = torch.bfloat16 if dtype is None else dtype
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed) * 1_000_003 + int(layer) * 7_919 + 17)
    k = torch.randn(batch, n_kv, tokens, head_dim, generator=gen, device=device, dtype=torch.float32)
    v = torch.randn(batch, n_kv, tokens, head_dim, generator=gen, device=device, dtype=torch.float32)
    for head in range(n_kv):
        out = torch.as_tensor(outlier_channels(seed, layer, head, head_dim), device=device)
        k[:, head, :, out] *= 10.0
    return k.to(dtype), v.to(dtype)
