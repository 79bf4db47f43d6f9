"""Key-tier policies on disk: the format ``DeepSeekQwenKVAdapter.load_policy`` reads.

Mirrors ``PrecisionPolicy`` of ``src/logitfill/allocators/policy.py:28-86``: a
directory holding ``policy.npz`` (``levels`` ``[layers, kv_heads, head_dim]``
int64 in {0=INT2, 1=INT4, 2=INT8, 3=FP16}, plus optional per-channel curves of
the same shape) and ``metadata.json``.  Loading checks the level range, the
shape against ``n_layers``/``n_kv``/``head_dim`` metadata and, when the
metadata carries ``target_bit`` (and does not set ``enforce_budget`` false),
the per-head Key budget of ``allocators/allocate.py:26-88``.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from logitfill_b200.synthetic import LEVEL_BITS, extra_budget_per_head

# Extra payload bits above the INT2 floor per channel at each level (allocate.py:22-23).
LEVEL_EXTRA = np.array([0, 2, 6, 14], dtype=np.int64)


def assert_history_budget(levels: np.ndarray, target_bit: float, bit_v: int = 2) -> dict:
    """allocate.py:75-88: reject a map that spends more than the per-head Key budget."""
    values = np.asarray(levels, dtype=np.int64)
    if np.any((values < 0) | (values > 3)):
        raise ValueError("levels must be in {0, 1, 2, 3}")
    n_channels = int(values.shape[-1])
    extra = extra_budget_per_head(target_bit, bit_v, n_channels)
    spent = LEVEL_EXTRA[values].sum(axis=-1)
    overflow = int(spent.max()) if spent.size else 0
    if overflow > extra:
        raise ValueError(f"waterfill spent {overflow} extra bits in a head, budget is {extra}")
    return {
        "target_bit": float(target_bit), "bit_v": int(bit_v), "target_bit_k": 2.0 * float(target_bit) - bit_v,
        "extra_budget_per_head": int(extra), "n_channels": n_channels, "extra_spent_per_head": overflow,
        "actual_bit_k": float(LEVEL_BITS[values].mean()) if values.size else float("nan"),
    }


class PrecisionPolicy:
    """Fixed per-channel Key levels plus the calibration metadata (policy.py:28-86)."""

    def __init__(self, levels, metadata: dict, curves: dict | None = None):
        self.levels = np.asarray(levels, dtype=np.int64)
        if self.levels.ndim != 3:
            raise ValueError(f"levels must be [layers, kv_heads, head_dim], got {self.levels.shape}")
        if np.any((self.levels < 0) | (self.levels > 3)):
            raise ValueError("levels must be in {0, 1, 2, 3}")
        self.metadata = dict(metadata)
        self.curves = {k: np.asarray(v) for k, v in (curves or {}).items()}
        self._check_consistency()

    def _check_consistency(self) -> None:
        axis = {"n_layers": 0, "n_kv": 1, "head_dim": 2}
        for key, dim in axis.items():
            if key in self.metadata and int(self.metadata[key]) != self.levels.shape[dim]:
                raise ValueError(f"metadata {key}={self.metadata[key]} does not match levels {self.levels.shape}")
        if self.metadata.get("enforce_budget", True) and "target_bit" in self.metadata:
            assert_history_budget(self.levels, float(self.metadata["target_bit"]),
                                  int(self.metadata.get("bit_v", 2)))
        for name, curve in self.curves.items():
            if curve.shape != self.levels.shape:
                raise ValueError(f"curve {name} has shape {curve.shape}, levels are {self.levels.shape}")

    def validate_model(self, model) -> None:
        """Raise when ``model`` cannot take this policy (policy.py:53-66)."""
        cfg = model.config
        n_q = int(cfg.num_attention_heads)
        head_dim = int(getattr(cfg, "head_dim", None) or cfg.hidden_size // n_q)
        expected = (int(cfg.num_hidden_layers), int(cfg.num_key_value_heads), head_dim)
        if tuple(self.levels.shape) != expected:
            raise ValueError(f"policy shape {self.levels.shape} does not match model {expected}")
        model_id = getattr(cfg, "name_or_path", None) or getattr(cfg, "_name_or_path", None)
        saved = self.metadata.get("model_id")
        if saved and model_id and Path(str(saved)).name != Path(str(model_id)).name and str(saved) != str(model_id):
            raise ValueError(f"policy model_id {saved} does not match loaded model {model_id}")

    def save(self, directory) -> Path:
        path = Path(directory)
        path.mkdir(parents=True, exist_ok=True)
        np.savez_compressed(path / "policy.npz", levels=self.levels, **self.curves)
        (path / "metadata.json").write_text(json.dumps(self.metadata, indent=2, sort_keys=True) + "\n",
                                            encoding="utf-8")
        return path

    @classmethod
    def load(cls, directory) -> "PrecisionPolicy":
        path = Path(directory)
        with np.load(path / "policy.npz") as packed:
            levels = packed["levels"]
            curves = {k: packed[k] for k in packed.files if k != "levels"}
        metadata = json.loads((path / "metadata.json").read_text(encoding="utf-8"))
        return cls(levels, metadata, curves)
