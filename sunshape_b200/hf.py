"""Config, codec bundle format and HF wrapper (reference ``sunshape/hf.py:202-416``).

The bundle format is the reference's unchanged (``hf.py:273-338``): a ``torch.save``d
dict with ``format_version`` 1 and per-layer codec ``state_dict``s, so bundles fitted
by the reference load here and bundles saved here load in the reference (for codecs
with one codebook per layer; per-KV-head codebooks add a leading dim to ``centroids``).
Trace extraction and codec fitting are offline calibration and are not part of the
B200 decode path.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from pathlib import Path

import torch

from .cache import SunShapeCache
from .codec import SunShapeBlockCodec


def resolve_mode_alias(mode: str) -> str:
    aliases = {
        "sunshape_base": "profileperm_baseline",
        "profileperm_baseline": "profileperm_baseline",
        "profileperm_sigmaq": "profileperm_baseline",
        "sunshape_mixed": "profileperm_mixed_precision",
        "profileperm_mixed_precision": "profileperm_mixed_precision",
        "baseline": "identity_baseline",
        "identity_baseline": "identity_baseline",
        "sunshape_pro": "profileperm_localmetric_dsq",
        "profileperm_localmetric_dsq": "profileperm_localmetric_dsq",
        "profileperm_sigmaq_localmetric_dsq": "profileperm_localmetric_dsq",
        "rotated": "rotated",
    }
    if mode not in aliases:
        raise ValueError(f"Unknown SunShape mode alias: {mode}")
    return aliases[mode]


def default_block_dim(bits_per_dim: float) -> int:
    return 8 if bits_per_dim <= 1.0 else 2


@dataclass
class SunShapeConfig:
    layers: list[int] | None = None
    bits_per_dim: float = 4.0
    block_dim: int | None = None
    mode: str = "sunshape_base"
    cal_points: int = 4096
    dsq_steps: int = 3
    kmeans_iters: int = 15
    seed: int = 42

    @property
    def resolved_mode(self) -> str:
        return resolve_mode_alias(self.mode)

    @property
    def resolved_block_dim(self) -> int:
        return default_block_dim(self.bits_per_dim) if self.block_dim is None else int(self.block_dim)


@dataclass
class TraceConfig:
    num_samples: int = 16
    seq_len: int = 512
    dataset_name: str = "wikitext"
    dataset_config: str = "wikitext-2-raw-v1"
    split: str = "validation"


def _get_num_layers(model) -> int:
    cfg = getattr(model, "config", None)
    text = getattr(cfg, "text_config", None) or cfg
    n = getattr(text, "num_hidden_layers", None)
    if n is None:
        raise ValueError("cannot infer the number of decoder layers")
    return int(n)


@dataclass
class SunShapeBundle:
    model_name: str
    layers: list[int]
    bits_per_dim: float
    block_dim: int
    mode: str
    cal_points: int
    dsq_steps: int
    seed: int
    codecs: dict[int, SunShapeBlockCodec]
    trace_meta: dict = field(default_factory=dict)

    def make_cache(self, *, config=None, num_layers: int | None = None) -> SunShapeCache:
        return SunShapeCache.from_codecs(codecs_dict=self.codecs, config=config, num_layers=num_layers)

    def wrap_model(self, model) -> "SunShapeCausalLM":
        return SunShapeCausalLM(model=model, bundle=self)

    def state_dict(self) -> dict:
        codec_state = {}
        for layer_idx, codec in self.codecs.items():
            codec_state[str(layer_idx)] = {
                "state_dict": {k: v.detach().cpu() for k, v in codec.state_dict().items()},
                "head_dim": codec.head_dim,
                "block_dim": codec.block_dim,
                "n_centroids": codec.n_centroids,
                "c": codec.c,
                "n_refine_dsq": codec.n_refine_dsq,
                "mode": codec.mode,
            }
        return {
            "format_version": 1,
            "model_name": self.model_name,
            "layers": list(self.layers),
            "bits_per_dim": self.bits_per_dim,
            "block_dim": self.block_dim,
            "mode": self.mode,
            "cal_points": self.cal_points,
            "dsq_steps": self.dsq_steps,
            "seed": self.seed,
            "trace_meta": dict(self.trace_meta),
            "codecs": codec_state,
        }

    def save(self, path: str | Path) -> Path:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        torch.save(self.state_dict(), path)
        return path

    @classmethod
    def from_state_dict(cls, obj: dict, *, device: torch.device | None = None) -> "SunShapeBundle":
        if not isinstance(obj, dict) or "codecs" not in obj:
            raise ValueError("Invalid SunShape bundle file.")
        device = torch.device(device) if device is not None else torch.device(
            "cuda" if torch.cuda.is_available() else "cpu")
        codecs: dict[int, SunShapeBlockCodec] = {}
        for layer_idx_str, payload in obj["codecs"].items():
            sd = payload["state_dict"]
            cents = sd.get("centroids")
            kv_heads = int(cents.shape[0]) if cents is not None and cents.ndim == 4 else None
            codec = SunShapeBlockCodec(head_dim=int(payload["head_dim"]), block_dim=int(payload["block_dim"]),
                                       n_centroids=int(payload["n_centroids"]), c=float(payload.get("c", 5.0)),
                                       n_refine_dsq=int(payload.get("n_refine_dsq", 3)), mode=str(payload["mode"]),
                                       device=device, kv_heads=kv_heads)
            codec.load_state_dict(sd)
            codec.to(device)
            codecs[int(layer_idx_str)] = codec
        return cls(model_name=str(obj["model_name"]), layers=[int(x) for x in obj["layers"]],
                   bits_per_dim=float(obj["bits_per_dim"]), block_dim=int(obj["block_dim"]), mode=str(obj["mode"]),
                   cal_points=int(obj["cal_points"]), dsq_steps=int(obj["dsq_steps"]), seed=int(obj["seed"]),
                   codecs=codecs, trace_meta=dict(obj.get("trace_meta", {})))

    @classmethod
    def load(cls, path: str | Path, *, device: torch.device | None = None) -> "SunShapeBundle":
        return cls.from_state_dict(torch.load(path, map_location="cpu", weights_only=False), device=device)


class SunShapeCausalLM(torch.nn.Module):
    def __init__(self, model, bundle: SunShapeBundle):
        super().__init__()
        self.model = model
        self.bundle = bundle

    def _inject_cache(self, kwargs: dict) -> dict:
        updated = dict(kwargs)
        if updated.get("past_key_values") is None and updated.get("use_cache", True):
            updated["past_key_values"] = self.bundle.make_cache(config=self.model.config,
                                                                num_layers=_get_num_layers(self.model))
        return updated

    def forward(self, *args, **kwargs):
        return self.model(*args, **self._inject_cache(kwargs))

    def generate(self, *args, **kwargs):
        return self.model.generate(*args, **self._inject_cache(kwargs))

    def unwrap(self):
        return self.model

    def __getattr__(self, name):
        try:
            return super().__getattr__(name)
        except AttributeError:
            return getattr(self.model, name)


class SunShapeForCausalLM(SunShapeCausalLM):
    @classmethod
    def from_pretrained(cls, model_name: str, *, bundle_path: str | Path | None = None, device_map: str = "none",
                        torch_dtype: str = "float16", trust_remote_code: bool = False,
                        local_files_only: bool = False, **kwargs):
        """Load an HF causal LM and wrap it with a SunShape bundle (reference ``hf.py:372-416``).

        Returns ``(model, tokenizer, bundle)`` like the reference.  A fitted bundle
        (``bundle_path``) is required: fitting from traces is offline calibration.
        """
        if bundle_path is None:
            raise NotImplementedError("SunShapeForCausalLM.from_pretrained needs bundle_path: codec fitting is "
                                      "offline calibration and is not part of the B200 decode path")
        from transformers import AutoModelForCausalLM, AutoTokenizer

        dtype = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}[torch_dtype]
        kw = dict(trust_remote_code=trust_remote_code, local_files_only=local_files_only)
        tokenizer = AutoTokenizer.from_pretrained(model_name, **kw)
        model = AutoModelForCausalLM.from_pretrained(model_name, torch_dtype=dtype, **kw)
        if device_map == "none":
            model = model.to("cuda")
        bundle = SunShapeBundle.load(bundle_path, device=next(model.parameters()).device)
        out_path = kwargs.get("output_bundle_path")
        if out_path is not None:
            bundle.save(out_path)
        return cls(model=model, bundle=bundle), tokenizer, bundle
