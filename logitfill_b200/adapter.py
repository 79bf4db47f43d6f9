"""Model-level drop-in: the packed backend on a Hugging Face Qwen2 model.

Mirrors ``DeepSeekQwenKVAdapter`` of ``src/logitfill/models/deepseek_qwen.py:21-149``
with ``backend="packed"`` and the packed branch of the patched attention
forward (``src/logitfill/models/qwen2_attention.py:74-150,223-256``):

* the first prefill of a sequence runs the model's own dense attention in the
  original dtype; every later call with history runs the B200 decode kernels
  (K2 + K3) over the packed pages and the residual page;
* K/V of every call are committed after the attention that produced them
  (page-delayed quantization, K1 on each completed page);
* ``make_cache()`` returns the ``Cache`` handle that ``model(...)`` /
  ``generate`` read the sequence length from.

Differences from the reference, each deliberate:

* The attention forward accepts both the transformers 4.x keyword
  ``past_key_value`` and the 5.x ``past_key_values`` (the reference's forward
  names only the former, so under 5.x the cache reached it through ``**kwargs``
  and was forwarded into the dense attention call).
* A multi-token call with history returns ``[B, q_len, heads, D]`` before the
  output projection (the reference reshapes the ``[B, heads, q_len, D]``
  result directly, which interleaves heads and positions when q_len > 1).
* A decode step whose cache reports a length other than the packed history's
  raises ``ValueError`` instead of running with wrong rotary positions; pass
  ``past_key_values=adapter.make_cache()``.
* ``backend="fake"`` (fake quantization in the dense cache, the reference's
  correctness path) is not part of this package and raises
  ``NotImplementedError``; ``backend="packed"`` is the default here.

There is no dense or CPU fallback for a decode step: the CUDA library must be
present and the shapes supported, or the call raises.
"""
from __future__ import annotations

from types import MethodType
from typing import Optional

from torch import nn

from logitfill_b200.packed.cache import LogitFillCache, PackedKVManager
from logitfill_b200.policy import KeyPolicy, check_model_fit, policy_tables, read_policy

_CACHE_KEYS = ("past_key_value", "past_key_values")


def _head_dim(config) -> int:
    n_q = int(config.num_attention_heads)
    return int(getattr(config, "head_dim", None) or config.hidden_size // n_q)


def _dense_attention(attn, query, key, value, attention_mask, kwargs):
    """The model's configured attention implementation (sdpa, eager, ...)
    on ``[B, heads, T, D]`` states; returns ``[B, q_len, heads, D]``
    (qwen2_attention.py:149-185)."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    from transformers.models.qwen2.modeling_qwen2 import eager_attention_forward

    impl = getattr(attn.config, "_attn_implementation", None) or "sdpa"
    if impl == "eager":
        fn = eager_attention_forward
    elif hasattr(ALL_ATTENTION_FUNCTIONS, "get_interface"):
        fn = ALL_ATTENTION_FUNCTIONS.get_interface(impl, eager_attention_forward)
    else:
        fn = ALL_ATTENTION_FUNCTIONS.get(impl, eager_attention_forward)
    window = getattr(attn, "sliding_window", None)
    if window is None:
        cfg = attn.config
        if (getattr(cfg, "use_sliding_window", False) and getattr(cfg, "sliding_window", None) is not None
                and attn.layer_idx >= getattr(cfg, "max_window_layers", 0)):
            window = cfg.sliding_window
    out, _ = fn(attn, query, key, value, attention_mask,
                dropout=0.0 if not attn.training else attn.attention_dropout,
                scaling=attn.scaling, sliding_window=window, **kwargs)
    return out


def _make_forward(adapter: "DeepSeekQwenKVAdapter", layer_idx: int):
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    def forward(self, hidden_states, position_embeddings=None, attention_mask=None, *args, **kwargs):
        # 4.x passes the cache as ``past_key_value`` (positionally third in
        # some call sites), 5.x as ``past_key_values``; neither goes on to
        # the attention implementation.
        cache = args[0] if args else None
        for name in _CACHE_KEYS:
            given = kwargs.pop(name, None)
            if given is not None:
                cache = given
        kwargs.pop("cache_position", None)
        if position_embeddings is None:
            raise ValueError("the packed attention forward needs position_embeddings (cos, sin)")

        shape = hidden_states.shape[:-1]
        heads_shape = (*shape, -1, self.head_dim)
        query = self.q_proj(hidden_states).view(heads_shape).transpose(1, 2)
        key = self.k_proj(hidden_states).view(heads_shape).transpose(1, 2)
        value = self.v_proj(hidden_states).view(heads_shape).transpose(1, 2)
        cos, sin = position_embeddings
        query, key = apply_rotary_pos_emb(query, key, cos, sin)
        if adapter.capture:
            adapter.captured["Q"][layer_idx] = query.detach()
            adapter.captured["K"][layer_idx] = key.detach()
            adapter.captured["V"][layer_idx] = value.detach()

        replaced = adapter.k_overrides is not None and layer_idx in adapter.k_overrides
        if replaced:
            key = adapter.k_overrides[layer_idx].to(device=key.device, dtype=key.dtype)
        if adapter.skip_quant or replaced:
            # Unquantized path: the stock cache update and dense attention.
            if cache is not None:
                key, value = cache.update(key, value, self.layer_idx)
            out = _dense_attention(self, query, key, value, attention_mask, kwargs)
        else:
            out = _packed_branch(self, adapter, layer_idx, query, key, value, attention_mask, cache, kwargs)
        out = out.reshape(*shape, -1).contiguous()
        return self.o_proj(out), None

    return forward


def _packed_branch(attn, adapter, layer_idx, query, key, value, attention_mask, cache, kwargs):
    """qwen2_attention.py:223-256."""
    manager = adapter.packed_manager()
    past = manager.seq_len if layer_idx == 0 else manager.layer_length(layer_idx)
    if past == 0 and layer_idx == 0:
        manager.reset()
    if past == 0:
        out = _dense_attention(attn, query, key, value, attention_mask, kwargs)
    else:
        if layer_idx == 0 and cache is not None and not isinstance(cache, LogitFillCache):
            seen = int(cache.get_seq_length()) if hasattr(cache, "get_seq_length") else -1
            if seen != past:
                raise ValueError(
                    f"cache reports {seen} tokens but the packed history holds {past}; "
                    "pass past_key_values=adapter.make_cache()")
        out = manager.attend(layer_idx, query, key, value, attn.scaling).transpose(1, 2)
        if adapter.graph_step and query.shape[2] == 1:
            # A step being captured for replay (GraphDecoder): the token is
            # committed on the device and the host lengths advance per replay.
            manager.commit_token(layer_idx, key, value, advance_host=False)
            return out
    manager.commit(layer_idx, key, value)
    if cache is not None and hasattr(cache, "note_layer"):
        cache.note_layer(layer_idx, manager.seq_len)
    return out


class DeepSeekQwenKVAdapter:
    """Attach the packed Key/Value cache to a ``Qwen2ForCausalLM``
    (deepseek_qwen.py:21-149)."""

    def __init__(self, model: nn.Module, group_size: int = 128, page_size: Optional[int] = None,
                 v_group_size: Optional[int] = None, bit_v: int = 2, backend: str = "packed"):
        if model.__class__.__name__ != "Qwen2ForCausalLM":
            raise TypeError(f"DeepSeek-R1-Distill-Qwen-7B is Qwen2ForCausalLM, got {model.__class__.__name__}")
        if group_size < 1:
            raise ValueError("group_size must be positive")
        if backend not in ("fake", "packed"):
            raise ValueError(f"backend must be fake or packed, got {backend}")
        if backend == "fake":
            raise NotImplementedError("this package implements backend='packed' only")
        self.model = model
        self.group_size = int(group_size)
        self.page_size = self.group_size if page_size is None else int(page_size)
        self.v_group_size = self.group_size if v_group_size is None else int(v_group_size)
        self.bit_v = int(bit_v)
        self.backend = backend
        cfg = model.config
        self.n_layers = int(cfg.num_hidden_layers)
        self.n_kv = int(cfg.num_key_value_heads)
        self.n_q = int(cfg.num_attention_heads)
        self.head_dim = _head_dim(cfg)
        # apply.py:29-36
        if self.page_size % self.group_size:
            raise ValueError(f"page_size {self.page_size} must be a multiple of Key group_size {self.group_size}")
        if self.bit_v < 2 or self.bit_v > 16:
            raise ValueError(f"bit_v must be in 2..16, got {bit_v}")
        if self.bit_v < 16 and self.head_dim % self.v_group_size:
            raise ValueError(f"head_dim {self.head_dim} is not divisible by v_group_size {self.v_group_size}")
        if self.bit_v != 2:
            raise NotImplementedError("the packed backend stores Value at 2 bits (bit_v=2)")
        self.capture = False
        self.skip_quant = False
        self.graph_step = False  # set by GraphDecoder around its captured decode step
        self.captured: dict = {"Q": {}, "K": {}, "V": {}}
        self.k_overrides: Optional[dict] = None
        self.policy: Optional[KeyPolicy] = None
        self._levels: list = [None] * self.n_layers
        self._originals: list = []
        self._attached = False
        self._packed: Optional[PackedKVManager] = None

    # -- attach / detach (deepseek_qwen.py:61-86) ----------------------------
    def attach(self) -> "DeepSeekQwenKVAdapter":
        if self._attached:
            return self
        layers = self.model.model.layers
        self._originals = [layer.self_attn.forward for layer in layers]
        self.model._kv_adapter = self
        for i, layer in enumerate(layers):
            attn = layer.self_attn
            attn.k_levels = None
            attn.kv_group_size = self.group_size
            attn.v_group_size = self.v_group_size
            attn.kv_page_size = self.page_size
            attn.bit_v = self.bit_v
            attn.forward = MethodType(_make_forward(self, i), attn)
        self._attached = True
        if self.policy is not None:
            self.set_k_levels(self.policy.levels)
        return self

    def detach(self) -> None:
        if not self._attached:
            return
        for layer, original in zip(self.model.model.layers, self._originals):
            layer.self_attn.forward = original
        self._originals = []
        self._attached = False
        if getattr(self.model, "_kv_adapter", None) is self:
            self.model._kv_adapter = None

    # -- Key tier map (deepseek_qwen.py:88-121) ------------------------------
    def set_k_levels(self, levels) -> None:
        """``levels[layer]`` is ``[n_kv, head_dim]`` with 0=2bit, 1=4, 2=8,
        3=16; ``None`` puts every Key channel at 2 bit.  Changing the map
        drops the packed history (it was encoded with the old map)."""
        if not self._attached:
            raise RuntimeError("call attach() before set_k_levels()")
        layers = self.model.model.layers
        if levels is None:
            self._levels = [None] * self.n_layers
        else:
            if len(levels) != self.n_layers:
                raise ValueError(f"expected {self.n_layers} level maps, got {len(levels)}")
            for level in levels:
                if tuple(level.shape) != (self.n_kv, self.head_dim):
                    raise ValueError(f"level map {tuple(level.shape)} does not match {(self.n_kv, self.head_dim)}")
            self._levels = list(levels)
        for layer, level in zip(layers, self._levels):
            layer.self_attn.k_levels = level
        self._packed = None

    def load_policy(self, directory) -> KeyPolicy:
        """Read a policy directory (deepseek_qwen.py:111-121): check it fits
        the model and the adapter's Value bits, install its Key tier maps and
        build their device tier tables (shared with every cache that uses
        them)."""
        policy = read_policy(directory)
        check_model_fit(policy, self.model.config)
        bit_v = int(policy.metadata.get("bit_v", self.bit_v))
        if bit_v != self.bit_v:
            raise ValueError(f"the policy was calibrated with Value at {bit_v} bits, the adapter stores {self.bit_v}")
        self.policy = policy
        if self._attached:
            self.set_k_levels(policy.levels)
            policy_tables(policy, next(self.model.parameters()).device)
        return policy

    # -- packed store (deepseek_qwen.py:123-146) -----------------------------
    def packed_manager(self) -> PackedKVManager:
        if self._packed is None:
            device = next(self.model.parameters()).device
            self._packed = PackedKVManager(
                levels=self._levels, n_q=self.n_q, n_kv=self.n_kv, head_dim=self.head_dim,
                page_size=self.page_size, k_group_size=self.group_size, v_group_size=self.v_group_size,
                bit_v=self.bit_v, device=device)
        return self._packed

    def make_cache(self) -> LogitFillCache:
        """Cache object accepted by ``model(..., past_key_values=)``."""
        return LogitFillCache(self.packed_manager())

    def clear_capture(self) -> None:
        self.captured = {"Q": {}, "K": {}, "V": {}}


__all__ = ["DeepSeekQwenKVAdapter"]
