"""sunshape_b200 -- B200-native (sm_100a) SunShape quantized-key decode path.

Drop-in names of the reference package (``sunshape/__init__.py``) for the decode
hot path: codec, score entry points, attention backend, caches and bundle format.
All compute runs in ``libsunshape_b200.so`` (hand-written CUDA for sm_100a behind a
C ABI, ``include/sunshape_b200.h``); there is no CPU fallback.
"""
from .codec import SunShapeBlockCodec, SunShapeQuantized
from .kernels import _torch_attention_scores, sunshape_attention_scores, sunshape_attention_scores_strict

__version__ = "0.1.0"


def __getattr__(name):
    # heavier modules (transformers) load lazily
    if name in ("SunShapeCache", "SunShapeLayer", "IdentityLayer"):
        from . import cache
        return getattr(cache, name)
    if name in ("TurboQuantCache", "TurboQuantLayer"):
        from . import turbo_cache
        return getattr(turbo_cache, name)
    if name in ("SunShapeBundle", "SunShapeCausalLM", "SunShapeConfig", "SunShapeForCausalLM", "TraceConfig",
                "default_block_dim", "resolve_mode_alias"):
        from . import hf
        return getattr(hf, name)
    if name in ("SunShapeVLLMHandle", "SunShapeVLLMRuntimeState", "load_runtime_state", "runtime_state_from_bundle"):
        from .integration import vllm
        return getattr(vllm, name)
    if name in ("SunShapeAttentionImpl", "SunShapeQuantizedKeys", "quantize_key_states"):
        from . import vllm_attn_backend
        return getattr(vllm_attn_backend, name)
    raise AttributeError(name)


__all__ = [
    "SunShapeBlockCodec", "SunShapeQuantized", "sunshape_attention_scores", "sunshape_attention_scores_strict",
    "_torch_attention_scores", "SunShapeCache", "SunShapeBundle", "SunShapeConfig", "SunShapeForCausalLM",
    "SunShapeAttentionImpl", "SunShapeQuantizedKeys", "quantize_key_states",
]
