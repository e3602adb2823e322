"""TurboQuant KV caches (reference ``sunshape/turbo_cache.py``) for like-for-like comparisons.

A ``TurboQuantLayer`` replaces the keys it receives by their quantize -> dequantize round trip
through a quantizer callable (any ``[rows, head_dim] -> [rows, head_dim]`` function; the reference's
layer does the same, ``turbo_cache.py:16-29``) before the dense layer stores them, so the model's own
attention sees TurboQuant keys.  ``TurboQuantCache.for_layers`` builds ``sunshape_b200.turbo.TurboQuantMSE``
quantizers per layer (seed + layer index, as ``turbo_cache.py:70-96``); the 1-bit QJL residual variant
(``turboquant_prod``) is not provided.
"""
from __future__ import annotations

from typing import Any, Callable

import torch
from transformers.cache_utils import DynamicCache, DynamicLayer


class TurboQuantLayer(DynamicLayer):
    def __init__(self, quantizer: Callable[[torch.Tensor], torch.Tensor] | None = None):
        super().__init__()
        self.quantizer = quantizer

    def _round_trip(self, key_states: torch.Tensor) -> torch.Tensor:
        rows = key_states.reshape(-1, key_states.shape[-1]).float()
        return self.quantizer(rows).reshape(key_states.shape).to(key_states.dtype)

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if self.quantizer is not None:
            key_states = self._round_trip(key_states)
        return super().update(key_states, value_states, *args, **kwargs)


class TurboQuantCache(DynamicCache):
    """DynamicCache whose layers listed in ``layer_quantizers`` fake-quantize keys with TurboQuant."""

    def __init__(self, config=None, num_layers: int | None = None, layer_quantizers: dict[int, Any] | None = None,
                 **kwargs):
        super().__init__(**({"config": config} if config is not None else {}), **kwargs)
        if not self.layers:
            if num_layers is None:
                raise ValueError("Must provide either config or num_layers")
            self.layers.extend(DynamicLayer() for _ in range(num_layers))
        for i, quantizer in (layer_quantizers or {}).items():
            if 0 <= i < len(self.layers):
                replacement = TurboQuantLayer(quantizer)
                window = getattr(self.layers[i], "sliding_window", None)
                if window is not None:
                    replacement.sliding_window = window
                self.layers[i] = replacement

    @classmethod
    def from_quantizers(cls, quantizers_dict: dict[int, Any], config=None,
                        num_layers: int | None = None) -> "TurboQuantCache":
        return cls(config=config, num_layers=num_layers, layer_quantizers=quantizers_dict)

    @classmethod
    def for_layers(cls, *, head_dims: dict[int, int], layers: list[int], config=None, num_layers: int | None = None,
                   bits: int = 3, mode: str = "turboquant_mse", seed: int = 42,
                   device: torch.device | None = None) -> "TurboQuantCache":
        if mode == "turboquant_prod":
            raise NotImplementedError("the QJL residual variant (turboquant_prod) is not provided; use turboquant_mse")
        if mode != "turboquant_mse":
            raise ValueError(f"Unsupported TurboQuant cache mode: {mode}")
        from .turbo import TurboQuantMSE

        quantizers = {int(li): TurboQuantMSE(int(head_dims[li]), bits=int(bits), seed=seed + int(li), device=device)
                      for li in layers}
        return cls.from_quantizers(quantizers, config=config, num_layers=num_layers)

    def has_previous_state(self, layer_idx: int | None = None) -> bool:
        return self.get_seq_length() > 0
