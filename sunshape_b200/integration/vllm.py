"""Runtime registry glue between a serving engine and the SunShape attention backend.

The decode path needs one thing from the serving side: given a layer index, the codec
that encoded that layer's keys.  The reference keeps it in a runtime-state object whose
``codec_for_layer`` the attention backend calls (``sunshape/integration/vllm.py:127-141``,
used at ``sunshape/vllm_attn_backend.py:108,295``).  This module provides that object,
built from a bundle file or an in-memory bundle, and ``install_hooks``, which loads a
bundle and registers it with the backend module in one call.

Engine launch plumbing (connector configs, environment exports, engine-argument
dictionaries) is not on the decode path and is not provided; an engine integration
only needs ``load_runtime_state`` + ``register_runtime_state``.
"""
from __future__ import annotations

import importlib
from dataclasses import dataclass, field, fields
from pathlib import Path
from typing import Any, Iterable

import torch

DEFAULT_BACKEND_MODULE = "sunshape_b200.vllm_attn_backend"


@dataclass
class SunShapeVLLMRuntimeState:
    """Per-process codec registry.  Field names follow the reference's runtime state so code that
    builds one by keyword keeps working; ``bundle`` is a ``sunshape_b200.hf.SunShapeBundle``."""

    bundle_path: str
    model_name: str
    mode: str
    bits_per_dim: float
    block_dim: int
    layers: list[int]
    bundle: Any
    device: str
    backend_module: str = DEFAULT_BACKEND_MODULE
    beta: bool = True

    def codec_for_layer(self, layer_idx: int):
        """The layer's codec, or None when the layer is not quantized."""
        return self.bundle.codecs.get(int(layer_idx))

    def supports_layer(self, layer_idx: int) -> bool:
        return self.codec_for_layer(layer_idx) is not None

    def to_dict(self) -> dict[str, Any]:
        d = {f.name: getattr(self, f.name) for f in fields(self) if f.name != "bundle"}
        d["layers"] = [int(x) for x in self.layers]
        d["trace_meta"] = dict(getattr(self.bundle, "trace_meta", {}) or {})
        return d


def runtime_state_from_bundle(bundle, *, bundle_path: str = "<memory>", device: str | None = None,
                              layers: Iterable[int] | None = None) -> SunShapeVLLMRuntimeState:
    """Runtime state around an in-memory bundle (no file round trip)."""
    if device is None:
        first = next(iter(bundle.codecs.values()), None)
        device = str(first.device) if first is not None else "cuda"
    return SunShapeVLLMRuntimeState(
        bundle_path=str(bundle_path), model_name=bundle.model_name, mode=bundle.mode,
        bits_per_dim=float(bundle.bits_per_dim), block_dim=int(bundle.block_dim),
        layers=sorted(int(x) for x in (layers if layers else bundle.layers)), bundle=bundle, device=str(device))


def load_runtime_state(*, bundle_path: str | Path, model_name: str, mode: str, bits_per_dim: float,
                       block_dim: int, layers: Iterable[int], backend_module: str = DEFAULT_BACKEND_MODULE,
                       device: str | torch.device | None = None) -> SunShapeVLLMRuntimeState:
    """Load a bundle file (the reference's format) onto ``device`` (default: the current CUDA device)."""
    from ..hf import SunShapeBundle

    path = Path(bundle_path)
    if not path.is_file():
        raise FileNotFoundError(f"SunShape vLLM bundle does not exist: {path}")
    dev = torch.device(device) if device is not None else torch.device("cuda")
    bundle = SunShapeBundle.load(path, device=dev)
    state = runtime_state_from_bundle(bundle, bundle_path=str(path), device=str(dev), layers=layers)
    state.model_name, state.mode = model_name, mode
    state.bits_per_dim, state.block_dim = float(bits_per_dim), int(block_dim)
    state.backend_module = backend_module
    return state


@dataclass
class SunShapeVLLMHandle:
    """What ``install_hooks`` returns: the registered state and where it was registered."""

    state: SunShapeVLLMRuntimeState
    backend_module: str = DEFAULT_BACKEND_MODULE
    hooks_installed: bool = False
    notes: list[str] = field(default_factory=list)

    def to_dict(self) -> dict[str, Any]:
        return {"backend_module": self.backend_module, "hooks_installed": self.hooks_installed,
                "notes": list(self.notes), "runtime": self.state.to_dict()}

    def deactivate(self) -> "SunShapeVLLMHandle":
        backend = importlib.import_module(self.backend_module)
        backend.clear_registered_runtime()
        backend.clear_registered_handle()
        self.hooks_installed = False
        return self


def install_hooks(*, bundle_path: str | Path, model_name: str, mode: str, bits_per_dim: float, block_dim: int,
                  layers: Iterable[int], backend_module: str = DEFAULT_BACKEND_MODULE,
                  device: str | torch.device | None = None) -> SunShapeVLLMHandle:
    """Load the bundle and register it (and the returned handle) with the backend module, so
    ``SunShapeAttentionImpl`` / ``quantize_key_states`` find the codecs by layer index."""
    state = load_runtime_state(bundle_path=bundle_path, model_name=model_name, mode=mode,
                               bits_per_dim=bits_per_dim, block_dim=block_dim, layers=layers,
                               backend_module=backend_module, device=device)
    backend = importlib.import_module(backend_module)
    handle = SunShapeVLLMHandle(state=state, backend_module=backend_module)
    backend.register_runtime_state(state)
    backend.register_handle(handle)
    handle.hooks_installed = True
    handle.notes.append(f"runtime state for layers {state.layers} registered with {backend_module}")
    return handle
