"""TurboQuant cache classes (reference ``sunshape/turbo_cache.py``), same API.

``TurboQuantLayer`` fake-quantizes keys through any quantizer callable on the flattened
``[rows, head_dim]`` fp32 keys (reference ``turbo_cache.py:16-29``); ``TurboQuantCache`` installs
it on the selected layers (``:32-99``).  The TurboQuant quantizers themselves
(``turbo_baseline.TurboQuantMSE`` / ``TurboQuantProd``) are the reference's comparison baseline,
not part of the SunShape decode path, so ``for_layers`` raises and callers pass their quantizers
through ``from_quantizers``.
"""
from __future__ import annotations

from typing import Any, Callable

import torch
from transformers.cache_utils import DynamicCache, DynamicLayer


class TurboQuantLayer(DynamicLayer):
    def __init__(self, quantizer: Callable[[torch.Tensor], torch.Tensor] | None = None):
        super().__init__()
        self.quantizer = quantizer

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if self.quantizer is not None:
            shape, dtype = key_states.shape, key_states.dtype
            flat = self.quantizer(key_states.reshape(-1, shape[-1]).float())
            key_states = flat.to(dtype).view(shape)
        return super().update(key_states, value_states, *args, **kwargs)


class TurboQuantCache(DynamicCache):
    def __init__(self, config=None, num_layers: int | None = None, layer_quantizers: dict[int, Any] | None = None,
                 **kwargs):
        if config is not None:
            kwargs["config"] = config
        super().__init__(**kwargs)
        layer_quantizers = layer_quantizers or {}
        if len(self.layers) == 0:
            if num_layers is None:
                raise ValueError("Must provide either config or num_layers")
            self.layers.extend(DynamicLayer() for _ in range(num_layers))
        for i, quantizer in layer_quantizers.items():
            if not 0 <= i < len(self.layers):
                continue
            layer = TurboQuantLayer(quantizer=quantizer)
            sliding = getattr(self.layers[i], "sliding_window", None)
            if sliding is not None:
                layer.sliding_window = sliding
            self.layers[i] = layer

    @classmethod
    def from_quantizers(cls, quantizers_dict: dict[int, Any], config=None,
                        num_layers: int | None = None) -> "TurboQuantCache":
        return cls(config=config, num_layers=num_layers, layer_quantizers=quantizers_dict)

    @classmethod
    def for_layers(cls, *, head_dims: dict[int, int], layers: list[int], config=None, num_layers: int | None = None,
                   bits: int = 3, mode: str = "turboquant_mse", seed: int = 42,
                   device: torch.device | None = None) -> "TurboQuantCache":
        if mode not in ("turboquant_mse", "turboquant_prod"):
            raise ValueError(f"Unsupported TurboQuant cache mode: {mode}")
        raise NotImplementedError(
            "the TurboQuant quantizers are the reference's comparison baseline and are not part of the B200 "
            "SunShape decode path; build them with the reference's turbo_baseline module and pass them to "
            "TurboQuantCache.from_quantizers")

    def has_previous_state(self, layer_idx: int | None = None) -> bool:
        return self.get_seq_length() > 0
