"""Packed Key/Value history and its decode path (drop-in for ``logitfill.packed``)."""

from logitfill_b200.packed.cache import LogitFillCache, PackedKVCache, PackedKVManager

__all__ = ["LogitFillCache", "PackedKVCache", "PackedKVManager"]
