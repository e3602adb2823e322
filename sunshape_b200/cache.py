"""HF cache classes (reference ``sunshape/cache.py``) with the key codec on B200 kernels.

``SunShapeLayer.update`` keeps the reference behaviour (``cache.py:32-46``): keys are
quantized and dequantized through the layer's codec before ``DynamicLayer.update``
stores them, so the model's own attention runs unmodified.  Both steps are single
CUDA launches over all ``[batch, kv_heads, seq]`` rows (per-KV-head codebooks included).
"""
from __future__ import annotations

from typing import Any

import torch
from transformers.cache_utils import DynamicCache, DynamicLayer


def fake_quantize_keys(codec, key_states: torch.Tensor) -> torch.Tensor:
    """quantize -> dequantize of key_states [B, H, S, D] (any float dtype), returned in its dtype."""
    from .vllm_attn_backend import dequantize_keys, quantize_codec_keys

    if key_states.ndim != 4:
        flat = key_states.reshape(1, 1, -1, key_states.shape[-1])
        return fake_quantize_keys(codec, flat).reshape(key_states.shape)
    # 16-bit keys go to the encoder as they are (exact in its tensor-core arithmetic; the reference
    # upcasts them to fp32 first, cache.py:41-44, which holds the same values)
    k = key_states if key_states.dtype in (torch.bfloat16, torch.float16) else key_states.float()
    payload = quantize_codec_keys(codec, k)
    return dequantize_keys(codec, payload).to(key_states.dtype)


class SunShapeLayer(DynamicLayer):
    """DynamicLayer that quantise-dequantises keys through a SunShape codec before storing them."""

    def __init__(self, codec=None):
        super().__init__()
        self.codec = codec

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if self.codec is not None:
            key_states = fake_quantize_keys(self.codec, key_states)
        return super().update(key_states, value_states, *args, **kwargs)


class IdentityLayer(DynamicLayer):
    """Control layer: same path as SunShapeLayer with identity quantization."""


class SunShapeCache(DynamicCache):
    """DynamicCache whose selected layers quantise keys via SunShape codecs (reference ``cache.py:55-104``)."""

    def __init__(self, config=None, num_layers: int | None = None, layer_codecs: dict[int, Any] | None = None,
                 identity_layers: set[int] | None = None, **kwargs):
        if config is not None:
            kwargs["config"] = config
        super().__init__(**kwargs)
        layer_codecs = layer_codecs or {}
        identity_layers = identity_layers or set()
        if len(self.layers) == 0:
            if num_layers is None:
                raise ValueError("Must provide either config or num_layers")
            for _ in range(num_layers):
                self.layers.append(DynamicLayer())
        for i in range(len(self.layers)):
            if i in layer_codecs:
                new_layer = SunShapeLayer(codec=layer_codecs[i])
            elif i in identity_layers:
                new_layer = IdentityLayer()
            else:
                continue
            sliding = getattr(self.layers[i], "sliding_window", None)
            if sliding is not None:
                new_layer.sliding_window = sliding
            self.layers[i] = new_layer

    @classmethod
    def from_codecs(cls, codecs_dict: dict[int, Any], config=None, num_layers: int | None = None) -> "SunShapeCache":
        return cls(config=config, num_layers=num_layers, layer_codecs=codecs_dict)

    @classmethod
    def from_traces(cls, traces: dict, layers: list[int], config=None, num_layers: int | None = None, **kwargs):
        """Reference ``cache.py:131-186`` fits codecs from calibration traces; fitting is offline
        calibration, not part of the decode path."""
        raise NotImplementedError(
            "SunShapeCache.from_traces fits codecs from traces (offline calibration); fit with the reference and "
            "build the cache with SunShapeCache.from_codecs or SunShapeBundle.load(...).make_cache()")

    @classmethod
    def identity(cls, patched_layers: list[int], config=None, num_layers: int | None = None) -> "SunShapeCache":
        return cls(config=config, num_layers=num_layers, identity_layers=set(patched_layers))

    def has_previous_state(self, layer_idx: int | None = None) -> bool:
        return self.get_seq_length() > 0
