"""SunShape attention backend (drop-in for ``sunshape/vllm_attn_backend.py``) on B200 kernels.

Same module-level surface as the reference: mode toggles, handle / runtime
registry, ``SunShapeQuantizedKeys``, ``quantize_key_states``,
``_apply_quantized_attention`` and ``SunShapeAttentionImpl.forward`` with the
reference signature (``vllm_attn_backend.py:271-282``).  What changes is the
body: the reference loops over (batch, kv-head) in Python and calls a score
kernel, torch softmax and a matmul per head (``:216-253``); here ONE fused CUDA
launch (LUT build + LUT-gather scores + online softmax . V, split along the KV
sequence inside the GPU) produces the whole ``[B, Hq, L, Dv]`` output.

``SunShapeQuantizedKeys`` gains an optional packed backing store
(``indices [B, Hkv, T, nb]`` uint8 and ``heavy [B, Hkv, T, n_heavy, bd]``) that
the kernels read directly; ``head(b, h)`` still returns per-head
``SunShapeQuantized`` views, so per-head callers keep working.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Any

import torch
import torch.nn.functional as F

from . import _lib
from .codec import SunShapeQuantized
from .integration.vllm import SunShapeVLLMHandle, SunShapeVLLMRuntimeState, install_hooks

MODE_ACTIVE = "active"
MODE_CAPTURE = "capture"
MODE_OFF = "off"

_MODE = MODE_OFF
_ACTIVE_HANDLE: SunShapeVLLMHandle | None = None
_RUNTIME_STATE: SunShapeVLLMRuntimeState | None = None


@dataclass(frozen=True)
class SunShapeQuantizedKeys:
    """Quantized key cache payload (reference ``vllm_attn_backend.py:38-53``).

    Either the reference form (``quantized_heads``: a tuple of per-(b, h)
    ``SunShapeQuantized``) or the packed form (``indices``/``heavy`` tensors) --
    or both.  The fused kernels consume the packed form; :meth:`packed` builds it
    from per-head payloads when needed.
    """

    quantized_heads: tuple[Any, ...]
    batch_size: int
    num_kv_heads: int
    seq_len: int
    indices: torch.Tensor | None = None         # [B, Hkv, T, nb] uint8 (T may be a view of a larger cache)
    heavy: torch.Tensor | None = None           # [B, Hkv, T, n_heavy, bd] bf16/fp32
    passthrough_blocks: torch.Tensor | None = None
    head_dim: int = 0
    block_dim: int = 0

    def head(self, batch_idx: int, kv_head_idx: int) -> Any:
        if self.quantized_heads:
            return self.quantized_heads[batch_idx * self.num_kv_heads + kv_head_idx]
        if self.indices is None:
            raise IndexError("empty SunShapeQuantizedKeys")
        idx = self.indices[batch_idx, kv_head_idx]
        nb = idx.shape[-1]
        pv = None
        if self.heavy is not None and self.passthrough_blocks is not None:
            pv = torch.zeros(idx.shape[0], nb, self.block_dim, device=idx.device, dtype=torch.float32)
            pv[:, torch.nonzero(self.passthrough_blocks).flatten()] = self.heavy[batch_idx, kv_head_idx].float()
        return SunShapeQuantized(indices=idx, head_dim=self.head_dim, block_dim=self.block_dim, n_blocks=nb,
                                 passthrough_blocks=self.passthrough_blocks, passthrough_values=pv)

    def packed(self, codec) -> tuple[torch.Tensor, torch.Tensor | None]:
        """(indices [B, Hkv, T, nb] uint8, heavy [B, Hkv, T, n_heavy, bd] or None)."""
        if self.indices is not None:
            return self.indices, self.heavy
        heads = self.quantized_heads
        idx = torch.stack([h.indices for h in heads]).view(self.batch_size, self.num_kv_heads, self.seq_len, -1)
        if idx.dtype != torch.uint8:
            idx = idx.to(torch.uint8)
        heavy = None
        if codec.is_mixed and heads[0].passthrough_blocks is not None and heads[0].passthrough_values is not None:
            ids = codec.heavy_block_ids()
            heavy = torch.stack([h.passthrough_values[:, ids] for h in heads]).float()
            heavy = heavy.view(self.batch_size, self.num_kv_heads, self.seq_len, len(ids), -1)
        return idx, heavy


def set_mode(mode: str):
    global _MODE
    _MODE = mode


def get_mode() -> str:
    return _MODE


def register_handle(handle: SunShapeVLLMHandle) -> SunShapeVLLMHandle:
    global _ACTIVE_HANDLE
    _ACTIVE_HANDLE = handle
    set_mode(MODE_ACTIVE)
    return handle


def register_runtime_state(state: SunShapeVLLMRuntimeState) -> SunShapeVLLMRuntimeState:
    global _RUNTIME_STATE
    _RUNTIME_STATE = state
    set_mode(MODE_ACTIVE)
    return state


def clear_registered_handle() -> None:
    global _ACTIVE_HANDLE
    _ACTIVE_HANDLE = None
    if _RUNTIME_STATE is None:
        set_mode(MODE_OFF)


def clear_registered_runtime() -> None:
    global _RUNTIME_STATE
    _RUNTIME_STATE = None
    if _ACTIVE_HANDLE is None:
        set_mode(MODE_OFF)


def get_registered_handle() -> SunShapeVLLMHandle | None:
    return _ACTIVE_HANDLE


def get_registered_runtime() -> SunShapeVLLMRuntimeState | None:
    return _RUNTIME_STATE


def quantize_codec_keys(codec, key_states: torch.Tensor) -> SunShapeQuantizedKeys:
    """Encode ``key_states [B, Hkv, S, D]`` with ``codec`` in one launch (packed payload)."""
    if key_states.ndim != 4:
        raise RuntimeError("quantize_key_states expects key_states with shape [batch, kv_heads, seq_len, head_dim].")
    B, Hkv, S, _ = key_states.shape
    idx, heavy = codec.quantize_packed(key_states, kv_heads=Hkv)
    return SunShapeQuantizedKeys(
        quantized_heads=(), batch_size=int(B), num_kv_heads=int(Hkv), seq_len=int(S), indices=idx, heavy=heavy,
        passthrough_blocks=codec.mixed_high_precision_blocks.detach().clone() if codec.is_mixed else None,
        head_dim=codec.head_dim, block_dim=codec.block_dim)


def quantize_key_states(layer_idx: int, key_states: torch.Tensor) -> SunShapeQuantizedKeys:
    """vllm_attn_backend.py:101-123 -- one batched encode launch instead of a per-head loop."""
    runtime = get_registered_runtime()
    if runtime is None:
        raise RuntimeError("SunShape runtime state is not registered.")
    codec = runtime.codec_for_layer(int(layer_idx))
    if codec is None:
        raise RuntimeError(f"No SunShape codec is registered for layer {layer_idx}.")
    return quantize_codec_keys(codec, key_states)


def _decode_keys_if_needed(layer_idx: int | None, key_states: torch.Tensor) -> torch.Tensor:
    runtime = get_registered_runtime()
    if runtime is None or layer_idx is None:
        return key_states
    codec = runtime.codec_for_layer(int(layer_idx))
    if codec is None or key_states.ndim < 2:
        return key_states
    if key_states.ndim == 4:      # [B, Hkv, S, D]: one launch each way, per-KV-head codebooks included
        from .cache import fake_quantize_keys

        return fake_quantize_keys(codec, key_states)
    orig_shape, orig_dtype = key_states.shape, key_states.dtype
    decoded = codec(key_states.reshape(-1, orig_shape[-1]).float())
    return decoded.to(orig_dtype).reshape(orig_shape)


def _dequantize_key_payload_if_needed(layer_idx: int | None, key_states: Any) -> Any:
    if not isinstance(key_states, SunShapeQuantizedKeys):
        return key_states
    runtime = get_registered_runtime()
    if runtime is None or layer_idx is None:
        raise RuntimeError("SunShape runtime state is required to dequantize quantized key payloads.")
    codec = runtime.codec_for_layer(int(layer_idx))
    if codec is None:
        raise RuntimeError(f"No codec is registered for layer {layer_idx}.")
    return dequantize_keys(codec, key_states)


def dequantize_keys(codec, keys: SunShapeQuantizedKeys) -> torch.Tensor:
    """All heads of a payload back to dense fp32 keys [B, Hkv, T, D] in one launch."""
    desc, keep, n_heavy = codec.kernel_desc()
    idx, heavy = keys.packed(codec)
    B, H, T = keys.batch_size, keys.num_kv_heads, keys.seq_len
    idx_c, hs = _heads_view(idx, B, H, T)
    idx_c = _lib.aligned16(idx_c)
    if idx_c is not idx and hs != T:
        idx_c, hs = _lib.aligned16(idx.contiguous()), T
    heavy_c = None
    if heavy is not None:
        heavy_c = _lib.aligned16(heavy.contiguous() if not _same_head_stride(heavy, hs, T) else heavy)
    out = torch.empty(B, H, T, codec.head_dim, device=idx.device, dtype=torch.float32)
    if B * H * T:
        kd = _lib.kv_desc(idx_c, heavy_c, None, T, hs)
        _lib.dequantize(desc, kd, B * H, H, out)
    return out


def _quantized_fast_path_unavailable_reason(*, runtime_state, layer_idx, query, key, value, attn_mask,
                                            is_causal) -> str | None:
    """vllm_attn_backend.py:159-194 (same checks and messages)."""
    if runtime_state is None or layer_idx is None:
        return "No registered runtime state for quantized attention."
    if not isinstance(key, SunShapeQuantizedKeys):
        return "Key payload is not SunShapeQuantizedKeys."
    codec = runtime_state.codec_for_layer(int(layer_idx))
    if codec is None:
        return f"No codec for layer {layer_idx}."
    if query.ndim != 4 or value.ndim != 4:
        return "Quantized attention expects query/value tensors with shape [batch, heads, seq, dim]."
    if key.batch_size != int(query.shape[0]):
        return "Quantized key batch size does not match query batch size."
    if key.batch_size != int(value.shape[0]):
        return "Quantized key batch size does not match value batch size."
    if key.num_kv_heads != int(value.shape[1]):
        return "Quantized key kv-head count does not match value kv-head count."
    if key.seq_len != int(value.shape[2]):
        return "Quantized key sequence length does not match value sequence length."
    if int(query.shape[-1]) != int(codec.head_dim):
        return "Query head_dim does not match codec head_dim."
    if int(query.shape[1]) % int(key.num_kv_heads) != 0:
        return "Query head count must be divisible by kv-head count."
    if is_causal and int(query.shape[2]) != 1:
        return "Causal quantized fast path currently targets decode (query_len == 1)."
    if attn_mask is not None and attn_mask.ndim not in {2, 3, 4}:
        return "Unsupported attention-mask rank for quantized fast path."
    return None


def _mask_view(attn_mask: torch.Tensor | None, B: int, Hq: int, L: int, T: int):
    """Strided view of the additive mask with the reference's slicing rules (vllm_attn_backend.py:197-213).

    Returns (tensor with unit stride along T, (stride_b, stride_hq, stride_l)).
    """
    if attn_mask is None:
        return None, (0, 0, 0)
    m = attn_mask
    if m.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        m = m.to(torch.float32)          # the reference adds mask.to(scores.dtype): bool -> 0/1
    if m.shape[-1] != T:
        m = m.expand(*m.shape[:-1], T)
    if m.stride(-1) != 1:
        m = m.contiguous()

    def sq(t, dim):
        return 0 if t.shape[dim] == 1 else t.stride(dim)

    if m.ndim == 2:                                   # [L|1, T] broadcast over batch and heads
        if m.shape[0] not in (1, L):
            raise RuntimeError("2-D attention mask must have shape [query_len or 1, seq_len].")
        return m, (0, 0, sq(m, 0))
    if m.ndim == 3:
        if m.shape[1] not in (1, L):
            raise RuntimeError("3-D attention mask must have shape [batch or heads, query_len or 1, seq_len].")
        if m.shape[0] == B:                           # per-batch mask
            return m, (sq(m, 0), 0, sq(m, 1))
        if m.shape[0] not in (1, Hq):
            raise RuntimeError("3-D attention mask leading dim must equal batch size or query head count.")
        return m, (0, sq(m, 0), sq(m, 1))
    if m.shape[0] not in (1, B) or m.shape[1] not in (1, Hq) or m.shape[2] not in (1, L):
        raise RuntimeError("4-D attention mask must broadcast to [batch, q_heads, query_len, seq_len].")
    return m, (sq(m, 0), sq(m, 1), sq(m, 2))


def _same_head_stride(t: torch.Tensor, hs: int, T: int) -> bool:
    """t [B, H, T, *rest]: contiguous rows with a uniform head stride of hs tokens."""
    row = 1
    for s in t.shape[3:]:
        row *= s
    if T > 1 and t.stride(2) != row:
        return False
    for d in range(3, t.ndim):
        expect = 1
        for s in t.shape[d + 1:]:
            expect *= s
        if t.shape[d] > 1 and t.stride(d) != expect:
            return False
    if t.shape[1] > 1 and t.stride(1) != hs * row:
        return False
    if t.shape[0] > 1 and t.stride(0) != t.shape[1] * hs * row:
        return False
    return True


def _heads_view(t: torch.Tensor, B: int, H: int, T: int) -> tuple[torch.Tensor, int]:
    """Return (tensor, head_stride_tokens) so head hh's token rows start at hh * head_stride."""
    row = 1
    for s in t.shape[3:]:
        row *= s
    if t.shape[1] > 1:
        hs = t.stride(1) // max(row, 1)
    elif t.shape[0] > 1:
        hs = t.stride(0) // max(row, 1)
    else:
        hs = T
    if hs >= T and _same_head_stride(t, hs, T):
        return t, hs
    return t.contiguous(), T


def _kv_layout(value, idx, heavy, B, H, T):
    """Pick one head stride (tokens) shared by values, indices and heavy rows; copy if they disagree."""
    v, hs = _heads_view(value, B, H, T)
    aligned = all(t is None or t.data_ptr() % 16 == 0 for t in (v, idx, heavy))
    if aligned and _same_head_stride(idx, hs, T) and (heavy is None or _same_head_stride(heavy, hs, T)):
        return v, idx, heavy, hs
    return (_lib.aligned16(value.contiguous()), _lib.aligned16(idx.contiguous()),
            (_lib.aligned16(heavy.contiguous()) if heavy is not None else None), T)


def _apply_quantized_attention(*, codec, query: torch.Tensor, key: SunShapeQuantizedKeys, value: torch.Tensor,
                               attn_mask: torch.Tensor | None, scale: float | None,
                               partials: torch.Tensor | None = None, out: torch.Tensor | None = None,
                               write_output: bool = True, peer_group=None):
    """vllm_attn_backend.py:216-253 as one fused launch.

    query [B, Hq, L, D], value [B, Hkv, T, Dv] -> output [B, Hq, L, Dv] in value.dtype.
    With ``partials`` ([B*Hq*L, 2 + Dv] fp32) the unnormalised (max, sum, acc) of
    the softmax over this call's tokens is also written, for KV-sequence shards.
    """
    B, Hq, L, _D = query.shape
    _, Hkv, T, Dv = value.shape
    desc, keep, n_heavy = codec.kernel_desc()
    idx, heavy = key.packed(codec)
    if T == 0:
        raise RuntimeError("quantized attention over an empty KV sequence.")
    if n_heavy and heavy is None:
        raise ValueError("Mixed-precision quantized keys are missing passthrough values.")
    if codec.n_blocks > 32 and value.dtype == torch.float32 and peer_group is None:
        return _apply_dequantized_attention(codec=codec, query=query, key=key, value=value, attn_mask=attn_mask,
                                            scale=scale, partials=partials, out=out, write_output=write_output)
    v, idx, heavy, hs = _kv_layout(value, idx, heavy, B, Hkv, T)
    if idx.dtype != torch.uint8:
        idx = idx.to(torch.uint8)
    q = query.contiguous()
    mask, mstr = _mask_view(attn_mask, B, Hq, L, T)
    if mask is not None:
        mask = mask.to(query.device)
    if out is None and write_output:
        out = torch.empty(B, Hq, L, Dv, device=query.device, dtype=value.dtype)
    if B == 0:
        return out
    kd = _lib.kv_desc(idx, heavy, v, T, hs, Dv)
    if peer_group is not None:
        _lib.decode_attention_peers(desc, kd, q, B, Hq, Hkv, L, mask, mstr, scale, out, peer_group)
    else:
        _lib.decode_attention(desc, kd, q, B, Hq, Hkv, L, mask, mstr, scale, out, partials)
    return out


def _apply_dequantized_attention(*, codec, query, key, value, attn_mask, scale, partials=None, out=None,
                                 write_output=True):
    """fp32 values with more than 32 blocks per head (the fused fp32-value kernel keeps its LUT in
    shared memory): the reference's arithmetic (vllm_attn_backend.py:216-253) on the GPU -- keys from
    the dequantize kernel, then batched matmul / softmax / matmul in fp32."""
    B, Hq, L, D = query.shape
    _, Hkv, T, Dv = value.shape
    G = Hq // Hkv
    k_hat = dequantize_keys(codec, key)                                  # [B, Hkv, T, D] fp32
    q = query if scale is None else query * float(scale)
    q = q.float().reshape(B, Hkv, G * L, D)
    s = torch.matmul(q, k_hat.transpose(-2, -1))                          # [B, Hkv, G*L, T]
    if attn_mask is not None:
        m = attn_mask.to(device=s.device, dtype=s.dtype)
        if m.ndim == 3:   # [batch, L, T] or [q_heads, L, T] (vllm_attn_backend.py:197-213 order)
            m = m[:, None] if m.shape[0] == B else m[None]
        s = (s.reshape(B, Hq, L, T) + m).reshape(B, Hkv, G * L, T)
    mx = s.amax(-1, keepdim=True)
    e = torch.exp(s - mx)
    l = e.sum(-1, keepdim=True)
    acc = torch.matmul(e, value.float())                                  # [B, Hkv, G*L, Dv]
    if partials is not None:
        pr = partials.view(B, Hkv, G * L, 2 + Dv)
        pr[..., 0:1] = mx
        pr[..., 1:2] = l
        pr[..., 2:] = acc
    if not write_output:
        return out
    res = (acc / l).reshape(B, Hq, L, Dv).to(value.dtype)
    if out is None:
        return res
    out.copy_(res)
    return out


def decode_partials(*, codec, query: torch.Tensor, key: SunShapeQuantizedKeys, value: torch.Tensor,
                    attn_mask: torch.Tensor | None = None, scale: float | None = None,
                    partials: torch.Tensor | None = None) -> torch.Tensor:
    """Unnormalised softmax partials over this call's KV tokens: [B*Hq*L, 2 + Dv] fp32 rows (m, l, acc)."""
    B, Hq, L, _ = query.shape
    Dv = value.shape[-1]
    if partials is None:
        partials = torch.empty(B * Hq * L, 2 + Dv, device=query.device, dtype=torch.float32)
    _apply_quantized_attention(codec=codec, query=query, key=key, value=value, attn_mask=attn_mask, scale=scale,
                               partials=partials, write_output=False)
    return partials


class SunShapeAttentionImpl:
    """Attention shim (reference ``vllm_attn_backend.py:256-347``) with the fused B200 fast path."""

    def __init__(self, *, delegate: Any = None, layer_idx: int | None = None,
                 runtime_state: SunShapeVLLMRuntimeState | None = None):
        self.delegate = delegate
        self.layer_idx = layer_idx
        self.runtime_state = runtime_state or get_registered_runtime()

    def forward(self, query: torch.Tensor, key: Any, value: torch.Tensor, *, attn_mask: torch.Tensor | None = None,
                is_causal: bool = False, scale: float | None = None, layer_idx: int | None = None,
                **kwargs: Any) -> torch.Tensor:
        layer = self.layer_idx if layer_idx is None else layer_idx
        runtime_state = self.runtime_state or get_registered_runtime()
        reason = _quantized_fast_path_unavailable_reason(runtime_state=runtime_state, layer_idx=layer, query=query,
                                                         key=key, value=value, attn_mask=attn_mask,
                                                         is_causal=is_causal)
        if reason is None:
            codec = runtime_state.codec_for_layer(int(layer)) if runtime_state is not None else None
            if codec is None:
                raise RuntimeError(f"No codec is registered for layer {layer}.")
            return _apply_quantized_attention(codec=codec, query=query, key=key, value=value, attn_mask=attn_mask,
                                              scale=scale)
        key = _dequantize_key_payload_if_needed(layer, key)
        key = _decode_keys_if_needed(layer, key)
        delegate = self.delegate
        if delegate is not None:
            if hasattr(delegate, "forward"):
                return delegate.forward(query, key, value, attn_mask=attn_mask, is_causal=is_causal, scale=scale,
                                        layer_idx=layer, **kwargs)
            if callable(delegate):
                return delegate(query, key, value, attn_mask=attn_mask, is_causal=is_causal, scale=scale,
                                layer_idx=layer, **kwargs)
        if query.ndim != 4 or key.ndim != 4 or value.ndim != 4:
            raise RuntimeError("SunShapeAttentionImpl fallback expects 4D [batch, heads, seq, dim] tensors "
                               "when no delegate backend is provided.")
        if scale is not None:
            query = query * float(scale)
        return F.scaled_dot_product_attention(query, key.to(query.dtype), value, attn_mask=attn_mask,
                                              is_causal=is_causal)

    __call__ = forward


class SunShapeAttentionBackend:
    backend_name = "sunshape"

    def __init__(self, *, delegate_backend: Any = None):
        self.delegate_backend = delegate_backend

    def make_impl(self, *, layer_idx: int | None = None, delegate: Any = None) -> SunShapeAttentionImpl:
        return SunShapeAttentionImpl(delegate=delegate if delegate is not None else self.delegate_backend,
                                     layer_idx=layer_idx, runtime_state=get_registered_runtime())

    def describe(self) -> dict[str, Any]:
        return describe_backend()


def get_backend_factory(*, delegate_backend: Any = None) -> SunShapeAttentionBackend:
    return SunShapeAttentionBackend(delegate_backend=delegate_backend)


def ensure_backend_registered() -> dict[str, Any]:
    return {
        "backend": "sunshape",
        "mode": get_mode(),
        "registered": get_registered_handle() is not None,
        "runtime_loaded": get_registered_runtime() is not None,
        "install_entrypoint": "sunshape_b200.vllm_attn_backend:install_sunshape_hooks",
        "env_backend": os.environ.get("VLLM_ATTENTION_BACKEND"),
    }


def describe_backend() -> dict[str, Any]:
    handle = get_registered_handle()
    if handle is None:
        return {"mode": get_mode(), "registered": False, "config": None, "runtime": None}
    d = {"mode": get_mode(), "registered": True}
    d.update(handle.to_dict())
    d["runtime"] = _RUNTIME_STATE.to_dict() if _RUNTIME_STATE is not None else None
    return d


def install_sunshape_hooks(*args, **kwargs) -> SunShapeVLLMHandle:
    """Load a bundle and register its codecs with this backend (``integration.vllm.install_hooks``)."""
    return install_hooks(*args, backend_module=__name__, **kwargs)


__all__ = [
    "MODE_ACTIVE", "MODE_CAPTURE", "MODE_OFF", "SunShapeVLLMHandle",
    "SunShapeVLLMRuntimeState", "SunShapeAttentionBackend", "SunShapeAttentionImpl", "SunShapeQuantizedKeys",
    "clear_registered_handle", "clear_registered_runtime", "describe_backend", "ensure_backend_registered",
    "get_mode", "get_registered_handle", "get_registered_runtime", "get_backend_factory", "install_sunshape_hooks",
    "quantize_key_states", "quantize_codec_keys", "dequantize_keys", "decode_partials", "register_handle", "register_runtime_state",
    "set_mode",
]
