"""Score entry points for SunShape block-VQ keys (reference ``sunshape/triton_kernels.py``).

``sunshape_attention_scores(codec, query, quantized_key)`` keeps the reference
signature (``triton_kernels.py:570-609``) but always runs the B200 LUT kernel:
the per-query LUT ``q_b . C_b[c]`` is built in shared memory and the uint8
indices are streamed from HBM and gathered against it.  Unsupported inputs
raise ``RuntimeError`` with the reason instead of silently falling back.
"""
from __future__ import annotations

import torch

from . import _lib
from .codec import SunShapeBlockCodec, SunShapeQuantized


def _fast_path_unavailable_reason(codec, query: torch.Tensor, quantized_key) -> str | None:
    """Counterpart of ``_triton_fast_path_unavailable_reason`` (triton_kernels.py:327-363)."""
    if not hasattr(quantized_key, "indices"):
        return "Quantized key must expose an .indices tensor."
    if not query.is_cuda:
        return "Query tensor must be on CUDA for the B200 fast path."
    if not quantized_key.indices.is_cuda:
        return "Quantized key indices must be on CUDA for the B200 fast path."
    if query.ndim != 2:
        return f"Expected query.ndim == 2, got {query.ndim}."
    if quantized_key.indices.ndim != 2:
        return f"Expected quantized_key.indices.ndim == 2, got {quantized_key.indices.ndim}."
    if quantized_key.indices.shape[1] != codec.n_blocks:
        return ("Quantized key block count does not match codec: "
                f"indices.shape[1]={quantized_key.indices.shape[1]}, codec.n_blocks={codec.n_blocks}.")
    if query.shape[1] != codec.head_dim:
        return f"Query head dim {query.shape[1]} does not match codec.head_dim {codec.head_dim}."
    if codec.centroids.ndim not in (3, 4):
        return f"Expected codec.centroids.ndim == 3, got {codec.centroids.ndim}."
    if query.shape[0] > 16 * 64:
        return "At most 1024 query rows per call."
    return None


def _supports_fast_path(codec, query: torch.Tensor, quantized_key) -> bool:
    return _fast_path_unavailable_reason(codec, query, quantized_key) is None


def require_fast_path(codec, query: torch.Tensor, quantized_key) -> None:
    reason = _fast_path_unavailable_reason(codec, query, quantized_key)
    if reason is not None:
        raise RuntimeError(reason)


# the reference's public name for the same check (triton_kernels.py:366-373), kept for callers
require_triton_fast_path = require_fast_path


def _heavy_compact(codec: SunShapeBlockCodec, quantized_key) -> torch.Tensor | None:
    if not codec.is_mixed or getattr(quantized_key, "passthrough_blocks", None) is None:
        return None
    if not bool(codec.mixed_high_precision_blocks.any()):
        return None
    pv = quantized_key.passthrough_values
    if pv is None:
        raise ValueError("Mixed-precision quantized keys are missing passthrough values.")
    return pv[:, codec.heavy_block_ids()].float().contiguous()


def sunshape_attention_scores_strict(codec, query: torch.Tensor, quantized_key, *,
                                     kv_head: int | None = None) -> torch.Tensor:
    """Scores [num_query_heads, num_tokens] fp32 on the B200 kernel, or raise.

    ``kv_head`` selects the codebook of a per-KV-head codec and is required for one."""
    require_fast_path(codec, query, quantized_key)
    h = codec._require_head(kv_head, "sunshape_attention_scores")
    if h is not None:
        codec = codec._head_view(h)
    if quantized_key.indices.dtype in (torch.int16, torch.int32):
        # codebooks above 256 codewords store int16 / int32 indices (codec.py:78-83)
        return _wide_or_packed_scores(codec, query, quantized_key.indices,
                                      16 if quantized_key.indices.dtype == torch.int16 else 32)
    if codec.n_blocks > 32:
        # more than 32 blocks (block_dim 2, the reference's default 4 bits/dim): a per-query LUT would
        # outgrow shared memory, so scores are the reference's own formula (triton_kernels.py:300-311)
        # on the GPU: the dequantize kernel, then one cuBLAS matmul
        return _torch_attention_scores(codec, query, quantized_key)
    desc, keep, n_heavy = codec.kernel_desc()
    idx = quantized_key.indices
    if idx.dtype != torch.uint8:
        idx = idx.to(torch.uint8)
    idx = _lib.aligned16(idx.contiguous())
    heavy = _heavy_compact(codec, quantized_key) if n_heavy else None
    q = query.contiguous()
    if q.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        q = q.float()
    n_rows, T = q.shape[0], idx.shape[0]
    out = torch.empty(n_rows, T, device=q.device, dtype=torch.float32)
    if n_rows == 0 or T == 0:
        return out
    kd = _lib.kv_desc(idx, heavy, None, T, T)
    for r0 in range(0, n_rows, 16):
        rows = min(16, n_rows - r0)
        _lib.attention_scores(desc, kd, q[r0:r0 + rows], 1, 1, rows, None, out[r0:r0 + rows])
    return out


def _wide_or_packed_scores(codec, query: torch.Tensor, indices: torch.Tensor, bits: int) -> torch.Tensor:
    desc, keep, n_heavy = codec.kernel_desc()
    if n_heavy:
        raise RuntimeError("packed / wide index scores do not take SunShape-Mixed heavy blocks.")
    q = query.contiguous()
    if q.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        q = q.float()
    idx = indices.contiguous()
    n_rows, T = q.shape[0], idx.shape[0]
    out = torch.empty(n_rows, T, device=q.device, dtype=torch.float32)
    if n_rows == 0 or T == 0:
        return out
    for r0 in range(0, n_rows, 16):
        rows = min(16, n_rows - r0)
        _lib.attention_scores_packed(desc, idx, bits, T, T, q[r0:r0 + rows], 1, 1, rows, out[r0:r0 + rows])
    return out


def sunshape_attention_scores_packed(codec, query: torch.Tensor, packed: torch.Tensor, bits: int, *,
                                     kv_head: int | None = None) -> torch.Tensor:
    """Scores [num_query_heads, num_tokens] against bit-packed indices [num_tokens, row_bytes] (1, 2 or 4
    bits per block; the reference's packed format, triton_kernels.py:213-292)."""
    if not query.is_cuda or not packed.is_cuda:
        raise RuntimeError("sunshape_b200 runs only on CUDA tensors (B200, sm_100a); there is no CPU fallback.")
    h = codec._require_head(kv_head, "sunshape_attention_scores_packed")
    if h is not None:
        codec = codec._head_view(h)
    return _wide_or_packed_scores(codec, query, packed, int(bits))


def pack_indices(indices: torch.Tensor, bits: int) -> torch.Tensor:
    """Bit-pack uint8 indices [..., n_blocks] at 1, 2 or 4 bits per block (on the GPU)."""
    return _lib.pack_indices(indices.to(torch.uint8), int(bits))


def sunshape_attention_scores(codec, query: torch.Tensor, quantized_key, *, kv_head: int | None = None) -> torch.Tensor:
    """``<query, k_hat>`` against block-quantized keys (triton_kernels.py:570-609), on the B200 kernel."""
    return sunshape_attention_scores_strict(codec, query, quantized_key, kv_head=kv_head)


def _torch_attention_scores(codec, query: torch.Tensor, quantized_key, *, kv_head: int | None = None) -> torch.Tensor:
    """Dequantize-then-matmul reference path (triton_kernels.py:300-311), dequantize on the GPU kernel."""
    k_hat = codec.dequantize(quantized_key, kv_head=kv_head)
    return torch.matmul(query.float(), k_hat.float().transpose(-2, -1))


def _precompute_query_centroid_dots(query: torch.Tensor, centroids: torch.Tensor, n_blocks: int,
                                    block_dim: int) -> torch.Tensor:
    """Host formula of the LUT (triton_kernels.py:381-408), kept for API parity and debugging."""
    q_blocks = query.view(query.shape[0], n_blocks, block_dim)
    return torch.einsum("qbd,bcd->qbc", q_blocks, centroids).contiguous()


__all__ = [
    "SunShapeQuantized",
    "sunshape_attention_scores",
    "sunshape_attention_scores_strict",
    "require_fast_path",
    "_torch_attention_scores",
    "_precompute_query_centroid_dots",
    "sunshape_attention_scores_packed",
    "pack_indices",
]
