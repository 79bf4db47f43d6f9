"""B200-native LogitFill packed KV-cache hot path.

Drop-in for the ``packed`` backend of GASSFY/Logitfill (``logitfill.packed``):
page quantize+pack (K1), split-K GQA decode attention over packed pages plus
the residual page (K2) and the split merge (K3), hand-written for sm_100a and
called through the C ABI in ``include/logitfill_b200.h``.
"""
from logitfill_b200.packed import LogitFillCache, PackedKVCache, PackedKVManager
from logitfill_b200.packed.attention import packed_attention, packed_attention_batched

__all__ = ["LogitFillCache", "PackedKVCache", "PackedKVManager", "packed_attention", "packed_attention_batched"]
