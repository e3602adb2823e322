"""vLLM runtime state for the SunShape backend (reference ``sunshape/integration/vllm.py``).

Only the part the decode path consumes is behavioural: ``SunShapeVLLMRuntimeState.codec_for_layer``
(reference ``:140-141``) hands the layer's codec to the attention backend.  The config / handle
dataclasses keep the reference's fields so launch scripts written for it still work; real vLLM
connector wiring is out of scope here, as it is in the reference (which only probes module names).
"""
from __future__ import annotations

import importlib
import json
import os
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Iterable

import torch

DEFAULT_CONNECTOR_NAME = "sunshape"
DEFAULT_BACKEND_MODULE = "sunshape_b200.vllm_attn_backend"


@dataclass
class SunShapeVLLMConfig:
    model_name: str
    bundle_path: str
    mode: str
    bits_per_dim: float
    block_dim: int
    layers: list[int]
    connector_name: str = DEFAULT_CONNECTOR_NAME
    backend_module: str = DEFAULT_BACKEND_MODULE
    beta: bool = True

    def runtime_entrypoint(self) -> str:
        return f"{self.backend_module}:install_sunshape_hooks"

    def launch_env(self) -> dict[str, str]:
        return {
            "SUNSHAPE_VLLM_CONNECTOR": self.connector_name,
            "SUNSHAPE_VLLM_BUNDLE_PATH": self.bundle_path,
            "SUNSHAPE_VLLM_MODE": self.mode,
            "SUNSHAPE_VLLM_BITS_PER_DIM": str(self.bits_per_dim),
            "SUNSHAPE_VLLM_BLOCK_DIM": str(self.block_dim),
            "SUNSHAPE_VLLM_LAYERS": ",".join(str(x) for x in self.layers),
            "SUNSHAPE_VLLM_BACKEND_MODULE": self.backend_module,
        }

    def engine_args(self) -> dict[str, Any]:
        return {
            "model": self.model_name,
            "kv_transfer_config": {"connector": self.connector_name, "bundle_path": self.bundle_path,
                                   "mode": self.mode, "bits_per_dim": self.bits_per_dim,
                                   "block_dim": self.block_dim, "layers": list(self.layers)},
            "sunshape_runtime": {"backend_module": self.backend_module,
                                 "install_entrypoint": self.runtime_entrypoint(), "beta": self.beta},
        }

    def to_dict(self) -> dict[str, Any]:
        return {"model_name": self.model_name, "bundle_path": self.bundle_path, "mode": self.mode,
                "bits_per_dim": self.bits_per_dim, "block_dim": self.block_dim, "layers": list(self.layers),
                "connector_name": self.connector_name, "backend_module": self.backend_module, "beta": self.beta,
                "engine_args": self.engine_args(), "launch_env": self.launch_env()}

    def save_json(self, path: str | Path) -> Path:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(json.dumps(self.to_dict(), indent=2))
        return path


@dataclass
class SunShapeVLLMHandle:
    config: SunShapeVLLMConfig
    hooks_installed: bool
    backend_module: str | None = None
    connector_registered: bool = False
    runtime_patch_available: bool = False
    vllm_version: str | None = None
    notes: list[str] = field(default_factory=list)

    def engine_args(self) -> dict[str, Any]:
        return self.config.engine_args()

    def to_dict(self) -> dict[str, Any]:
        return {"config": self.config.to_dict(), "hooks_installed": self.hooks_installed,
                "backend_module": self.backend_module, "connector_registered": self.connector_registered,
                "runtime_patch_available": self.runtime_patch_available, "vllm_version": self.vllm_version,
                "notes": list(self.notes)}

    def activate(self) -> "SunShapeVLLMHandle":
        backend = importlib.import_module(self.backend_module or self.config.backend_module)
        if hasattr(backend, "register_handle"):
            backend.register_handle(self)
            self.hooks_installed = True
            self.connector_registered = True
        return self

    def deactivate(self) -> "SunShapeVLLMHandle":
        backend = importlib.import_module(self.backend_module or self.config.backend_module)
        if hasattr(backend, "clear_registered_runtime"):
            backend.clear_registered_runtime()
        if hasattr(backend, "clear_registered_handle"):
            backend.clear_registered_handle()
        self.hooks_installed = False
        self.connector_registered = False
        return self


@dataclass
class SunShapeVLLMRuntimeState:
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
        return self.bundle.codecs.get(int(layer_idx))

    def supports_layer(self, layer_idx: int) -> bool:
        return int(layer_idx) in self.bundle.codecs

    def to_dict(self) -> dict[str, Any]:
        return {"bundle_path": self.bundle_path, "model_name": self.model_name, "mode": self.mode,
                "bits_per_dim": self.bits_per_dim, "block_dim": self.block_dim, "layers": list(self.layers),
                "device": self.device, "backend_module": self.backend_module, "beta": self.beta,
                "trace_meta": dict(getattr(self.bundle, "trace_meta", {}))}


def runtime_state_from_bundle(bundle, *, bundle_path: str = "<memory>", device: str | None = None,
                              layers: Iterable[int] | None = None) -> SunShapeVLLMRuntimeState:
    """Runtime state around an in-memory bundle (no file round trip)."""
    return SunShapeVLLMRuntimeState(
        bundle_path=str(bundle_path), model_name=bundle.model_name, mode=bundle.mode,
        bits_per_dim=float(bundle.bits_per_dim), block_dim=int(bundle.block_dim),
        layers=[int(x) for x in layers] if layers else list(bundle.layers), bundle=bundle,
        device=str(device or next(iter(bundle.codecs.values())).device if bundle.codecs else "cuda"))


def load_runtime_state(*, bundle_path: str | Path, model_name: str, mode: str, bits_per_dim: float,
                       block_dim: int, layers: Iterable[int], backend_module: str = DEFAULT_BACKEND_MODULE,
                       device: str | torch.device | None = None) -> SunShapeVLLMRuntimeState:
    from ..hf import SunShapeBundle

    bundle_path = Path(bundle_path)
    if not bundle_path.exists():
        raise FileNotFoundError(f"SunShape vLLM bundle does not exist: {bundle_path}")
    dev = torch.device(device) if device is not None else torch.device("cuda")
    bundle = SunShapeBundle.load(bundle_path, device=dev)
    return SunShapeVLLMRuntimeState(
        bundle_path=str(bundle_path), model_name=model_name, mode=mode, bits_per_dim=float(bits_per_dim),
        block_dim=int(block_dim), layers=[int(x) for x in layers] if layers else list(bundle.layers),
        bundle=bundle, device=str(dev), backend_module=backend_module, beta=True)


def build_launch_env(config: SunShapeVLLMConfig) -> dict[str, str]:
    env = dict(config.launch_env())
    env["VLLM_ATTENTION_BACKEND"] = config.connector_name
    env["SUNSHAPE_VLLM_INSTALL_ENTRYPOINT"] = config.runtime_entrypoint()
    return env


def install_hooks(*, bundle_path: str | Path, model_name: str, mode: str, bits_per_dim: float, block_dim: int,
                  layers: Iterable[int]) -> SunShapeVLLMHandle:
    """Register the runtime state with the backend module (vLLM itself is optional here)."""
    config = SunShapeVLLMConfig(model_name=model_name, bundle_path=str(bundle_path), mode=mode,
                                bits_per_dim=float(bits_per_dim), block_dim=int(block_dim),
                                layers=[int(x) for x in layers])
    handle = SunShapeVLLMHandle(config=config, hooks_installed=False, backend_module=config.backend_module)
    handle.activate()
    backend = importlib.import_module(config.backend_module)
    state = load_runtime_state(bundle_path=bundle_path, model_name=model_name, mode=mode,
                               bits_per_dim=bits_per_dim, block_dim=block_dim, layers=layers,
                               backend_module=config.backend_module)
    backend.register_runtime_state(state)
    os.environ["VLLM_ATTENTION_BACKEND"] = config.connector_name
    handle.notes.append("Registered SunShape runtime state for the B200 attention backend.")
    return handle
