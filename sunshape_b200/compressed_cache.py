"""HF cache whose quantized layers store codeword indices instead of keys, with attention routed
through the fused decode kernel.

The reference's ``SunShapeLayer`` (``sunshape/cache.py:32-46``) quantizes keys and stores them
dequantized, so the model's native attention runs unchanged but the cache is as large as a dense
one.  ``SunShapeCompressedLayer`` keeps what the decode path actually reads:

* uint8 codeword indices ``[B, Hkv, capacity, n_blocks]`` (SunShape-Mixed heavy blocks stay dense in
  ``[B, Hkv, capacity, n_heavy, block_dim]``), appended by one encode launch per update;
* values ``[B, Hkv, capacity, Dv]`` in the model dtype,

in buffers that grow by doubling, so appends do not copy the whole cache.  ``update`` returns a
``CompressedKeys`` view (a ``SunShapeQuantizedKeys`` that also names its codec) and the value view.
The attention function registered as ``attn_implementation="sunshape"`` sends decode steps
(query length 1) to ``_apply_quantized_attention`` -- LUT build, LUT-gather scores and softmax . V
in one fused launch over the stored indices -- and prefill steps to SDPA over keys rebuilt by the
dequantize kernel.  Key storage drops from ``2 * head_dim`` bytes per token and KV head (bf16) to
``n_blocks`` bytes (16 at head_dim 128, block_dim 8).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
from transformers.cache_utils import DynamicCache, DynamicLayer

from .vllm_attn_backend import SunShapeQuantizedKeys, _apply_quantized_attention, dequantize_keys

ATTN_IMPLEMENTATION = "sunshape"


@dataclass(frozen=True)
class CompressedKeys(SunShapeQuantizedKeys):
    """Quantized keys of one cache layer, with the codec that encoded them."""

    codec: Any = None


class SunShapeCompressedLayer(DynamicLayer):
    """Cache layer storing codeword indices (+ SunShape-Mixed heavy blocks) and dense values."""

    def __init__(self, codec):
        super().__init__()
        self.codec = codec
        self.indices = self.heavy = self.values_buf = None
        self.length = 0

    # ------------------------------------------------------------------ storage
    def _reserve(self, need: int, like_keys: torch.Tensor, like_values: torch.Tensor) -> None:
        cap = 0 if self.indices is None else self.indices.shape[2]
        if need <= cap:
            return
        new_cap = max(need, 2 * cap, 64)
        B, H = like_keys.shape[:2]
        c = self.codec
        idx = torch.empty(B, H, new_cap, c.n_blocks, dtype=torch.uint8, device=like_keys.device)
        val = torch.empty(B, H, new_cap, like_values.shape[-1], dtype=like_values.dtype, device=like_values.device)
        heavy = None
        n_heavy = int(c.mixed_high_precision_blocks.sum().item()) if c.is_mixed else 0
        if n_heavy:
            hdt = torch.bfloat16 if like_keys.dtype == torch.bfloat16 else torch.float32
            heavy = torch.empty(B, H, new_cap, n_heavy, c.block_dim, dtype=hdt, device=like_keys.device)
        if self.length:
            idx[:, :, :self.length] = self.indices[:, :, :self.length]
            val[:, :, :self.length] = self.values_buf[:, :, :self.length]
            if heavy is not None:
                heavy[:, :, :self.length] = self.heavy[:, :, :self.length]
        self.indices, self.values_buf, self.heavy = idx, val, heavy

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        self.dtype, self.device = key_states.dtype, key_states.device
        self.is_initialized = True

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        S = key_states.shape[-2]
        self._reserve(self.length + S, key_states, value_states)
        a, b = self.length, self.length + S
        k = key_states if key_states.dtype in (torch.bfloat16, torch.float16) else key_states.float()
        idx, heavy = self.codec.quantize_packed(k, kv_heads=k.shape[1])
        self.indices[:, :, a:b] = idx
        if self.heavy is not None:
            self.heavy[:, :, a:b] = heavy
        self.values_buf[:, :, a:b] = value_states
        self.length = b
        return self.key_view(), self.values_buf[:, :, :b]

    def key_view(self) -> CompressedKeys:
        B, H = self.indices.shape[:2]
        c = self.codec
        return CompressedKeys(
            quantized_heads=(), batch_size=int(B), num_kv_heads=int(H), seq_len=int(self.length),
            indices=self.indices[:, :, :self.length],
            heavy=None if self.heavy is None else self.heavy[:, :, :self.length],
            passthrough_blocks=c.mixed_high_precision_blocks if c.is_mixed else None,
            head_dim=c.head_dim, block_dim=c.block_dim, codec=c)

    @property
    def keys(self) -> torch.Tensor:
        """Dense keys rebuilt by the dequantize kernel (for code that reads ``layer.keys``)."""
        if self.length == 0:
            return torch.tensor([], device=getattr(self, "device", None))
        return dequantize_keys(self.codec, self.key_view()).to(self.dtype)

    @keys.setter
    def keys(self, value) -> None:   # DynamicLayer.__init__ assigns keys; the layer derives them
        pass

    @property
    def values(self) -> torch.Tensor:
        if self.length == 0:
            return torch.tensor([], device=getattr(self, "device", None))
        return self.values_buf[:, :, :self.length]

    @values.setter
    def values(self, value) -> None:
        pass

    def get_seq_length(self) -> int:
        return self.length

    def crop(self, max_length: int) -> None:
        if max_length < 0:
            max_length = self.length - abs(max_length)
        self.length = min(self.length, max(0, max_length))

    def batch_repeat_interleave(self, repeats: int) -> None:
        if self.indices is not None:
            self.indices = self.indices.repeat_interleave(repeats, dim=0)
            self.values_buf = self.values_buf.repeat_interleave(repeats, dim=0)
            if self.heavy is not None:
                self.heavy = self.heavy.repeat_interleave(repeats, dim=0)

    def batch_select_indices(self, indices: torch.Tensor) -> None:
        if self.indices is not None:
            self.indices = self.indices[indices]
            self.values_buf = self.values_buf[indices]
            if self.heavy is not None:
                self.heavy = self.heavy[indices]

    def storage_bytes(self) -> dict:
        """Bytes per stored token (all heads of a sequence) for keys and values."""
        B, H = (self.indices.shape[:2]) if self.indices is not None else (0, 0)
        key_b = self.codec.n_blocks
        if self.heavy is not None:
            key_b += self.heavy.shape[-2] * self.heavy.shape[-1] * self.heavy.element_size()
        val_b = self.values_buf.shape[-1] * self.values_buf.element_size() if self.values_buf is not None else 0
        return {"key_bytes_per_token_head": key_b, "value_bytes_per_token_head": val_b, "kv_heads": H}


class SunShapeCompressedCache(DynamicCache):
    """DynamicCache whose selected layers are ``SunShapeCompressedLayer``s (the others stay dense).

    Run the model with ``attn_implementation="sunshape"`` (``register_attention()`` makes the name
    known to transformers) so attention reads the stored indices."""

    def __init__(self, config=None, num_layers: int | None = None, layer_codecs: dict[int, Any] | None = None,
                 **kwargs):
        register_attention()
        if config is not None:
            kwargs["config"] = config
        super().__init__(**kwargs)
        layer_codecs = layer_codecs or {}
        if len(self.layers) == 0:
            if num_layers is None:
                raise ValueError("Must provide either config or num_layers")
            for _ in range(num_layers):
                self.layers.append(DynamicLayer())
        for i in range(len(self.layers)):
            if i in layer_codecs:
                self.layers[i] = SunShapeCompressedLayer(layer_codecs[i])

    @classmethod
    def from_codecs(cls, codecs_dict: dict[int, Any], config=None, num_layers: int | None = None):
        return cls(config=config, num_layers=num_layers, layer_codecs=codecs_dict)


def _additive_mask(mask: torch.Tensor | None, dtype=torch.float32) -> torch.Tensor | None:
    if mask is None:
        return None
    if mask.dtype == torch.bool:   # True = attend (transformers' sdpa masks)
        return torch.zeros(mask.shape, dtype=dtype, device=mask.device).masked_fill_(~mask, float("-inf"))
    return mask


def sunshape_attention_forward(module, query, key, value, attention_mask, dropout: float = 0.0,
                               scaling: float | None = None, is_causal: bool | None = None, **kwargs):
    """transformers attention function: fused quantized-key decode for ``CompressedKeys`` at query
    length 1, SDPA over dequantized keys for longer queries (prefill) and for dense layers."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    if isinstance(key, CompressedKeys):
        if query.shape[2] == 1:
            mask = _additive_mask(attention_mask)
            if mask is not None:
                mask = mask[..., : key.seq_len]
            out = _apply_quantized_attention(codec=key.codec, query=query, key=key, value=value, attn_mask=mask,
                                             scale=scaling)
            return out.transpose(1, 2).contiguous(), None
        key = dequantize_keys(key.codec, key).to(query.dtype)
    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                                  is_causal=is_causal, **kwargs)


_REGISTERED = False


def register_attention() -> None:
    """Make ``attn_implementation="sunshape"`` known to transformers (attention + mask functions)."""
    global _REGISTERED
    if _REGISTERED:
        return
    from transformers import AttentionInterface
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS, sdpa_mask

    AttentionInterface.register(ATTN_IMPLEMENTATION, sunshape_attention_forward)
    ALL_MASK_ATTENTION_FUNCTIONS.register(ATTN_IMPLEMENTATION, sdpa_mask)
    _REGISTERED = True


__all__ = ["CompressedKeys", "SunShapeCompressedLayer", "SunShapeCompressedCache", "register_attention",
           "sunshape_attention_forward", "ATTN_IMPLEMENTATION"]
