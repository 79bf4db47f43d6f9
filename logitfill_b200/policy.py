"""Key-tier policies: the on-disk directory and the device tier tables.

On disk (the directory LogitFill's offline calibration writes and
``DeepSeekQwenKVAdapter.load_policy`` reads, ``src/logitfill/allocators/policy.py``):

* ``policy.npz``: array ``levels`` ``[layers, kv_heads, head_dim]`` with one
  Key tier per channel (0 = INT2, 1 = INT4, 2 = INT8, 3 = FP16), plus any
  number of per-channel arrays of the same shape (calibration curves);
* ``metadata.json``: a JSON object.  The keys read here: ``n_layers``,
  ``n_kv``, ``head_dim`` (must describe ``levels``), ``bit_v``,
  ``target_bit`` with ``enforce_budget`` (the per-head Key budget is checked
  unless ``enforce_budget`` is false), ``model_id``.

:func:`read_policy` / :func:`write_policy` move a :class:`KeyPolicy`
between disk and memory; :class:`TierTables` turns one ``[kv_heads,
head_dim]`` level map into the device tables the kernels and the
reference-shaped ``layer.table`` need, built once per (map, device) with
vectorised torch and shared by every cache and manager that uses the map.
"""
from __future__ import annotations

import hashlib
import json
import threading
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np
import torch

from logitfill_b200.synthetic import LEVEL_BITS, extra_budget_per_head

N_TIERS = 4
# Key bits a channel costs above the INT2 floor, by tier.
_EXTRA_BITS = LEVEL_BITS - LEVEL_BITS[0]


def key_budget_report(levels, target_bit: float, bit_v: int = 2) -> dict:
    """Extra Key bits each head spends against the budget a history target
    of ``target_bit`` bits per element allows (Value at ``bit_v``); raises
    ``ValueError`` when a head overspends."""
    lv = np.asarray(levels, dtype=np.int64)
    if lv.size and (lv.min() < 0 or lv.max() >= N_TIERS):
        raise ValueError("Key tiers are 0 (INT2), 1 (INT4), 2 (INT8) or 3 (FP16)")
    d = int(lv.shape[-1])
    allowed = extra_budget_per_head(target_bit, bit_v, d)
    spent = _EXTRA_BITS[lv].sum(axis=-1) if lv.size else np.zeros(0, np.int64)
    worst = int(spent.max()) if spent.size else 0
    if worst > allowed:
        raise ValueError(f"a head of the level map uses {worst} Key bits above INT2; "
                         f"target_bit {target_bit} (bit_v {bit_v}) allows {allowed}")
    return {"allowed_extra_bits": allowed, "max_extra_bits": worst,
            "mean_key_bits": float(LEVEL_BITS[lv].mean()) if lv.size else float("nan")}


@dataclass
class KeyPolicy:
    """A model's Key tier map ``levels`` ``[layers, kv_heads, head_dim]``, the
    directory's metadata and its extra per-channel arrays (``curves``)."""

    levels: np.ndarray
    metadata: dict = field(default_factory=dict)
    curves: dict = field(default_factory=dict)

    def __post_init__(self):
        self.levels = np.asarray(self.levels, dtype=np.int64)
        self.metadata = dict(self.metadata)
        self.curves = {k: np.asarray(v) for k, v in self.curves.items()}
        check_policy(self)

    @classmethod
    def load(cls, directory) -> "KeyPolicy":
        return read_policy(directory)

    def save(self, directory) -> Path:
        return write_policy(directory, self)

    def validate_model(self, model) -> None:
        check_model_fit(self, model.config)


# The name LogitFill's adapter API uses for the policy object.
PrecisionPolicy = KeyPolicy


def check_policy(policy: KeyPolicy) -> None:
    """Raise ``ValueError`` unless ``policy`` is a well-formed map: 3-D, tiers
    in 0..3, the shape the metadata states, extra arrays of the same shape,
    and (when the metadata has ``target_bit`` and does not switch the check
    off) every head within its Key bit budget."""
    lv = policy.levels
    if lv.ndim != 3:
        raise ValueError(f"a policy's levels are [layers, kv_heads, head_dim]; got shape {lv.shape}")
    if lv.size and (lv.min() < 0 or lv.max() >= N_TIERS):
        raise ValueError("Key tiers are 0 (INT2), 1 (INT4), 2 (INT8) or 3 (FP16)")
    meta = policy.metadata
    for axis, key in enumerate(("n_layers", "n_kv", "head_dim")):
        if key in meta and int(meta[key]) != lv.shape[axis]:
            raise ValueError(f"metadata says {key} = {meta[key]} but the level map has shape {lv.shape}")
    for name, arr in policy.curves.items():
        if arr.shape != lv.shape:
            raise ValueError(f"policy array {name!r} has shape {arr.shape}, the level map {lv.shape}")
    if "target_bit" in meta and meta.get("enforce_budget", True):
        key_budget_report(lv, float(meta["target_bit"]), int(meta.get("bit_v", 2)))


def check_model_fit(policy: KeyPolicy, config) -> None:
    """Raise ``ValueError`` unless the map's shape is the model's (layers, KV
    heads, head_dim) and, when both name one, the model is the one the map
    was calibrated for (same id, or the same final path component)."""
    n_q = int(config.num_attention_heads)
    head_dim = int(getattr(config, "head_dim", None) or config.hidden_size // n_q)
    want = (int(config.num_hidden_layers), int(config.num_key_value_heads), head_dim)
    if tuple(policy.levels.shape) != want:
        raise ValueError(f"level map {tuple(policy.levels.shape)} does not fit the model's "
                         f"(layers, kv_heads, head_dim) = {want}")
    mine = policy.metadata.get("model_id")
    theirs = getattr(config, "name_or_path", None) or getattr(config, "_name_or_path", None)
    if mine and theirs and str(mine) != str(theirs) and Path(str(mine)).name != Path(str(theirs)).name:
        raise ValueError(f"the policy was calibrated for {mine!r}, the model is {theirs!r}")


def read_policy(directory) -> KeyPolicy:
    """Load ``policy.npz`` + ``metadata.json`` from ``directory``."""
    path = Path(directory)
    with np.load(path / "policy.npz") as npz:
        if "levels" not in npz.files:
            raise ValueError(f"{path / 'policy.npz'} has no 'levels' array")
        levels = npz["levels"]
        curves = {name: npz[name] for name in npz.files if name != "levels"}
    meta = json.loads((path / "metadata.json").read_text(encoding="utf-8"))
    if not isinstance(meta, dict):
        raise ValueError(f"{path / 'metadata.json'} does not hold a JSON object")
    return KeyPolicy(levels, meta, curves)


def write_policy(directory, policy: KeyPolicy) -> Path:
    """Write ``policy`` as ``policy.npz`` (compressed) + ``metadata.json``."""
    path = Path(directory)
    path.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(path / "policy.npz", levels=policy.levels, **policy.curves)
    (path / "metadata.json").write_text(json.dumps(policy.metadata, indent=2, sort_keys=True) + "\n",
                                        encoding="utf-8")
    return path


class TierTables:
    """Tier tables of one ``[kv_heads, head_dim]`` level map on one device.

    * ``counts`` host int32 ``[4, H]``: channels per tier and head (the input
      of ``lf_layout_init``);
    * ``chan_code`` int32 ``[H, D]``: ``tier << 16 | position in the tier``;
    * ``slot_chan`` int32 ``[4, H, D]``: the channel in tier slot ``s``
      (ascending channel order), -1 past the head's count;
    * ``table``: the reference-shaped dict of ``layer.table``
      (``src/logitfill/packed/layout.py:49-68``: per tier ``index``,
      ``count``, ``local``, ``width``; and ``tier``).

    :meth:`get` builds them once per (map, device) and returns the shared
    instance afterwards."""

    _cache: dict = {}
    _lock = threading.Lock()

    def __init__(self, levels, device):
        lv = torch.as_tensor(np.asarray(levels), dtype=torch.int64)
        if lv.dim() != 2:
            raise ValueError(f"a layer's level map is [kv_heads, head_dim]; got {tuple(lv.shape)}")
        if lv.numel() and (int(lv.min()) < 0 or int(lv.max()) >= N_TIERS):
            raise ValueError("Key tiers are 0 (INT2), 1 (INT4), 2 (INT8) or 3 (FP16)")
        dev = torch.device(device)
        H, D = lv.shape
        lv_d = lv.to(dev)
        onehot = lv_d.unsqueeze(-1) == torch.arange(N_TIERS, device=dev)      # [H, D, 4]
        # position of each channel among the channels of its tier (ascending)
        rank = onehot.to(torch.int32).cumsum(dim=1) - 1                        # [H, D, 4] (cumsum gives int64)
        local = rank.gather(2, lv_d.unsqueeze(-1)).squeeze(-1).to(torch.int32)  # [H, D]
        counts = onehot.sum(dim=1).to(torch.int32).T.contiguous()              # [4, H]
        slot_chan = torch.full((N_TIERS, H, D), -1, dtype=torch.int32, device=dev)
        heads = torch.arange(H, device=dev).unsqueeze(1).expand(H, D)
        chans = torch.arange(D, device=dev, dtype=torch.int32).unsqueeze(0).expand(H, D)
        slot_chan[lv_d, heads, local.long()] = chans
        self.chan_code = ((lv_d.to(torch.int32) << 16) | local).to(torch.int32).contiguous()
        self.slot_chan = slot_chan
        self.counts = np.ascontiguousarray(counts.cpu().numpy().astype(np.int32))
        widths = self.counts.max(axis=1) if H else np.zeros(N_TIERS, np.int32)
        table = {}
        for t in range(N_TIERS):
            w = int(widths[t])
            index = slot_chan[t, :, :w].clamp(min=0)  # the reference pads an index row with channel 0
            loc = torch.where(lv_d == t, local, torch.full_like(local, -1))
            table[t] = {"index": index.contiguous(), "count": counts[t].contiguous(), "local": loc.contiguous(),
                        "width": w}
        table["tier"] = lv_d.to(torch.int32)
        self.table = table
        self.levels = lv.clone()
        self.device = dev

    @classmethod
    def get(cls, levels, device) -> "TierTables":
        """The shared tables of ``levels`` on ``device`` (built on first use)."""
        arr = np.ascontiguousarray(np.asarray(levels if not torch.is_tensor(levels) else levels.cpu(), np.int64))
        dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        key = (hashlib.sha1(arr.tobytes()).hexdigest(), arr.shape, str(dev))
        with cls._lock:
            hit = cls._cache.get(key)
            if hit is None:
                hit = cls(arr, dev)
                cls._cache[key] = hit
            return hit


def policy_tables(policy: KeyPolicy, device) -> list:
    """Every layer's :class:`TierTables` of ``policy`` on ``device``."""
    return [TierTables.get(policy.levels[i], device) for i in range(policy.levels.shape[0])]
