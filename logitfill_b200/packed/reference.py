"""Import path of the reference's decode entry point (``logitfill.packed.reference``).

Only ``packed_attention`` is provided: the B200 backend has no dense fallback.
"""
from logitfill_b200.packed.attention import packed_attention, packed_attention_batched

__all__ = ["packed_attention", "packed_attention_batched"]
