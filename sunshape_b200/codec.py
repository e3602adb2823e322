"""SunShape block codec on B200: same buffers and methods as the reference codec.

``SunShapeBlockCodec`` keeps the reference's buffer names and shapes
(``sunshape/codec.py:230-245``) so bundles saved by the reference load
unchanged; ``quantize`` / ``dequantize`` / ``attention_scores`` run the CUDA
kernels of ``libsunshape_b200.so``.  The codebook may also be per KV head:
``centroids`` of shape ``[kv_heads, n_blocks, n_centroids, block_dim]``.

Offline calibration (``fit``: k-means, covariance permutation, DSQ) is not on
the decode hot path; codecs are loaded from bundles or have their buffers set
directly.
"""
from __future__ import annotations

import math
from typing import NamedTuple

import torch

from . import _lib

_PROFILEPERM_MODES = {"profileperm_baseline", "profileperm_localmetric_dsq", "profileperm_mixed_precision"}
_KNOWN_MODES = _PROFILEPERM_MODES | {"identity_baseline", "legacy_strict", "rotated"}


class SunShapeQuantized(NamedTuple):
    """Quantized keys of one head (reference ``codec.py:28-34``)."""

    indices: torch.Tensor
    head_dim: int
    block_dim: int
    n_blocks: int
    passthrough_blocks: torch.Tensor | None = None
    passthrough_values: torch.Tensor | None = None


def _compact_index_dtype(n_centroids: int) -> torch.dtype:
    """codec.py:78-83."""
    if n_centroids <= 256:
        return torch.uint8
    if n_centroids <= 65535:
        return torch.int16
    return torch.int32


def _invert_permutation(perm: torch.Tensor) -> torch.Tensor:
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(len(perm), device=perm.device, dtype=perm.dtype)
    return inv


class SunShapeBlockCodec(torch.nn.Module):
    """Block VQ key codec (ProfilePerm + per-block codebooks), CUDA-backed.

    Constructor arguments mirror ``sunshape/codec.py:205-216``.  Supported on the
    CUDA path: the ProfilePerm modes (``profileperm_baseline``, ``profileperm_mixed_precision``,
    and SunShape-Pro ``profileperm_localmetric_dsq``, whose block-diagonal metric ``E`` changes only
    the encode's distance) and ``identity_baseline``; ``rotated`` / ``legacy_strict`` raise.
    """

    def __init__(self, head_dim: int, block_dim: int = 8, n_centroids: int = 256, c: float = 5.0,
                 n_refine_dsq: int = 3, mode: str = "profileperm_baseline", use_rotation: bool = False,
                 rotation_seed: int = 0, device: torch.device | None = None, kv_heads: int | None = None):
        super().__init__()
        if head_dim % block_dim != 0:
            raise ValueError("head_dim must be divisible by block_dim")
        self.head_dim = head_dim
        self.block_dim = block_dim
        self.n_blocks = head_dim // block_dim
        self.n_centroids = n_centroids
        self.c = c
        self.mode = "rotated" if use_rotation else mode
        if self.mode not in _KNOWN_MODES:
            raise ValueError(f"Unknown SunShapeBlockCodec mode: {self.mode}")
        self.n_refine_dsq = 3 if n_refine_dsq is None else int(n_refine_dsq)
        self.use_rotation = self.mode == "rotated"
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda" if torch.cuda.is_available() else "cpu")
        dev = self.device
        cshape = (self.n_blocks, n_centroids, block_dim) if kv_heads is None else (
            kv_heads, self.n_blocks, n_centroids, block_dim)
        self.register_buffer("E", torch.eye(head_dim, device=dev))
        self.register_buffer("E_inv", torch.eye(head_dim, device=dev))
        self.register_buffer("centroids", torch.zeros(*cshape, device=dev))
        self.register_buffer("dsq_block_affinity", torch.ones(self.n_blocks, device=dev))
        self.register_buffer("dsq_active_blocks", torch.ones(self.n_blocks, device=dev, dtype=torch.bool))
        self.register_buffer("mixed_high_precision_blocks", torch.zeros(self.n_blocks, device=dev, dtype=torch.bool))
        self.register_buffer("mixed_block_mass", torch.zeros(self.n_blocks, device=dev))
        ident = torch.arange(head_dim, device=dev, dtype=torch.long)
        self.register_buffer("permutation", ident.clone())
        self.register_buffer("inv_permutation", ident.clone())
        self.register_buffer("rotation", torch.eye(head_dim, device=dev))
        self._desc_cache = None
        self._metric_cache = None

    # ------------------------------------------------------------------ state
    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        key = prefix + "centroids"
        if key in state_dict and state_dict[key].shape != self.centroids.shape:
            self.centroids = torch.empty_like(state_dict[key], device=self.centroids.device)
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)
        self._desc_cache = None
        self._metric_cache = None

    def _apply(self, fn, *args, **kwargs):
        out = super()._apply(fn, *args, **kwargs)
        self.device = self.E.device
        self._desc_cache = None
        self._metric_cache = None
        return out

    def invalidate(self) -> None:
        """Call after editing buffers in place (centroids, permutation, heavy mask, metric)."""
        self._desc_cache = None
        self._metric_cache = None

    @property
    def n_codebooks(self) -> int:
        return 1 if self.centroids.ndim == 3 else int(self.centroids.shape[0])

    @property
    def is_mixed(self) -> bool:
        return self.mode == "profileperm_mixed_precision"

    @property
    def is_metric(self) -> bool:
        """SunShape-Pro: nearest codeword under a block-diagonal local metric E (codec.py:375-377)."""
        return self.mode == "profileperm_localmetric_dsq"

    def _check_supported(self) -> None:
        if self.mode in ("rotated", "legacy_strict"):
            raise RuntimeError(
                f"mode {self.mode!r} uses a dense metric/rotation; the B200 kernels implement the ProfilePerm "
                "modes (profileperm_baseline, profileperm_mixed_precision, profileperm_localmetric_dsq) and "
                "identity_baseline.")

    def _metric_blocks(self) -> torch.Tensor:
        """Diagonal blocks E_b [nb, bd, bd] of the SunShape-Pro metric (permuted basis)."""
        bd, nb = self.block_dim, self.n_blocks
        e = self.E.float().view(nb, bd, nb, bd)
        return torch.stack([e[b, :, b, :] for b in range(nb)])

    def _metric_desc(self):
        """Encoder descriptor in the metric space: codewords C_b E_b^T, identity permutation."""
        dc = getattr(self, "_metric_cache", None)
        if dc is not None:
            return dc
        desc, keep, n_heavy = self.kernel_desc()
        cents = keep[0]                                                        # [n_cb, nb, C, bd]
        ct = torch.einsum("hbcd,bed->hbce", cents, self._metric_blocks()).contiguous()
        ident = torch.arange(self.head_dim, device=cents.device, dtype=torch.int64)
        mdesc = _lib.codec_desc(ct, ident, None, 0, self.head_dim, self.block_dim, None)
        self._metric_cache = (mdesc, (ct, ident))
        return self._metric_cache

    def kernel_desc(self):
        """C-ABI codec descriptor plus the tensors it points into (kept alive together)."""
        self._check_supported()
        dc = self._desc_cache
        if dc is not None:
            return dc
        if not self.centroids.is_cuda:
            raise RuntimeError("sunshape_b200 codec buffers must live on a CUDA device; there is no CPU path.")
        cents = self.centroids.float()
        if cents.ndim == 3:
            cents = cents.unsqueeze(0)
        cents = cents.contiguous()
        use_perm = self.mode in _PROFILEPERM_MODES
        perm = (self.permutation if use_perm else torch.arange(self.head_dim, device=self.E.device)).to(
            torch.int64).contiguous()
        heavy = None
        n_heavy = 0
        if self.is_mixed:
            hm = self.mixed_high_precision_blocks.to(torch.bool)
            n_heavy = int(hm.sum().item())
            if n_heavy:
                heavy = hm.to(torch.uint8).contiguous()
        # largest centroid norm per codebook: bounds |q_b . c| for the fp16 LUT scale
        norm_max = cents.norm(dim=-1).amax(dim=(1, 2)).contiguous()
        desc = _lib.codec_desc(cents, perm, heavy, n_heavy, self.head_dim, self.block_dim, norm_max)
        dc = (desc, (cents, perm, heavy, norm_max), n_heavy)
        self._desc_cache = dc
        return dc

    def heavy_block_ids(self) -> torch.Tensor:
        return torch.nonzero(self.mixed_high_precision_blocks.to(torch.bool)).flatten()

    # ------------------------------------------------------------------ transforms
    def _forward_transform(self, x: torch.Tensor) -> torch.Tensor:
        if self.mode in _PROFILEPERM_MODES:
            return x[..., self.permutation]
        if self.use_rotation:
            return x @ self.rotation.T
        return x

    def _inverse_transform(self, x: torch.Tensor) -> torch.Tensor:
        if self.mode in _PROFILEPERM_MODES:
            return x[..., self.inv_permutation]
        if self.use_rotation:
            return x @ self.rotation
        return x

    def fit(self, *args, **kwargs):
        raise NotImplementedError(
            "offline codec calibration is not part of the B200 decode path; load a bundle fitted by the "
            "reference (SunShapeBundle.load) or set the codec buffers directly")

    # ------------------------------------------------------------------ encode / decode
    def quantize_packed(self, keys: torch.Tensor, *, kv_heads: int = 1, index_dtype: torch.dtype | None = None,
                        heavy_dtype: torch.dtype | None = None):
        """Encode keys [..., H, T, D] (any leading dims, H KV heads) in one launch.

        Returns ``(indices [..., H, T, nb], heavy [..., H, T, n_heavy, bd] or None)``.
        ``heavy_dtype`` defaults to the keys' dtype for bf16 keys, else fp32, so
        heavy blocks are stored exactly.
        """
        desc, keep, n_heavy = self.kernel_desc()
        if keys.shape[-1] != self.head_dim:
            raise RuntimeError("Key head_dim does not match codec head_dim.")
        if keys.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            keys = keys.float()
        _lib.require_cuda(keys)
        T = keys.shape[-2]
        lead = keys.shape[:-2]
        k = keys.reshape(-1, T, self.head_dim)
        if k.stride(-1) != 1 or (T > 1 and k.stride(-2) != self.head_dim):
            k = k.contiguous()
        n_heads = k.shape[0]
        idt = index_dtype or _compact_index_dtype(self.n_centroids)
        idx = torch.empty(*lead, T, self.n_blocks, dtype=idt, device=keys.device)
        heavy = None
        if n_heavy:
            hdt = heavy_dtype or (torch.bfloat16 if keys.dtype == torch.bfloat16 else torch.float32)
            heavy = torch.empty(*lead, T, n_heavy, self.block_dim, dtype=hdt, device=keys.device)
        if n_heads and T:
            if self.is_metric:
                # SunShape-Pro: compare in the metric space -- key blocks (permuted) times E_b^T, one
                # fp32 GEMM over the block-diagonal E, then the encoder against the transformed codebooks
                mdesc, _ = self._metric_desc()
                kt = torch.matmul(k.float()[..., self.permutation], self.E.float().t()).contiguous()
                _lib.encode(mdesc, kt, n_heads, kv_heads, T, kt.stride(0), kt.stride(1), idx, None, T)
            else:
                _lib.encode(desc, k, n_heads, kv_heads, T, k.stride(0), k.stride(1), idx, heavy, T)
        return idx, heavy

    def _require_head(self, kv_head: int | None, what: str) -> int | None:
        """A codec holding one codebook per KV head needs to be told which head a call is for: the
        reference signatures (one codec per layer) carry no head, and silently using codebook 0 for
        every head would return wrong results without an error."""
        if self.n_codebooks == 1:
            return None
        if kv_head is None:
            raise RuntimeError(
                f"{what}: this codec holds {self.n_codebooks} per-KV-head codebooks; pass kv_head= "
                "(or use a one-codebook codec, as the reference does)")
        if not 0 <= int(kv_head) < self.n_codebooks:
            raise RuntimeError(f"{what}: kv_head {kv_head} out of range [0, {self.n_codebooks}).")
        return int(kv_head)

    def quantize(self, keys: torch.Tensor, *, kv_head: int | None = None) -> SunShapeQuantized:
        """codec.py:362-385 for one head's keys [T, D] (``kv_head`` picks a per-head codebook and is
        required when the codec holds more than one)."""
        keys = keys.to(self.device)
        if keys.dtype != torch.float32:
            keys = keys.float()
        h = self._require_head(kv_head, "quantize")
        if h is not None:
            return self._head_view(h).quantize(keys)
        idx, heavy = self.quantize_packed(keys.unsqueeze(0))
        idx = idx[0]
        pt_blocks = self.mixed_high_precision_blocks.detach().clone() if self.is_mixed else None
        pt_values = None
        if heavy is not None:
            pt_values = torch.zeros(keys.shape[0], self.n_blocks, self.block_dim, device=keys.device,
                                    dtype=torch.float32)
            pt_values[:, self.heavy_block_ids()] = heavy[0].float()
        return SunShapeQuantized(indices=idx, head_dim=self.head_dim, block_dim=self.block_dim,
                                 n_blocks=self.n_blocks, passthrough_blocks=pt_blocks, passthrough_values=pt_values)

    def _head_view(self, kv_head: int) -> "SunShapeBlockCodec":
        cache = getattr(self, "_head_views", None)
        if cache is None:
            cache = self._head_views = {}
        v = cache.get(kv_head)
        if v is None or v.centroids.data_ptr() != self.centroids[kv_head].data_ptr():
            v = SunShapeBlockCodec(self.head_dim, self.block_dim, self.n_centroids, self.c, self.n_refine_dsq,
                                   self.mode, device=self.device)
            for name, buf in self.named_buffers():
                setattr(v, name, buf[kv_head] if name == "centroids" else buf)
            cache[kv_head] = v
        return v

    def dequantize(self, quantized: SunShapeQuantized, *, kv_head: int | None = None) -> torch.Tensor:
        """codec.py:387-398: [T, nb] indices (+ passthrough) -> [T, D] fp32 in the model basis."""
        h = self._require_head(kv_head, "dequantize")
        if h is not None:
            return self._head_view(h).dequantize(quantized)
        desc, keep, n_heavy = self.kernel_desc()
        idx = quantized.indices
        if idx.dtype not in (torch.uint8, torch.int16, torch.int32):
            idx = idx.to(torch.int32)
        idx = _lib.aligned16(idx.contiguous())
        heavy = None
        if n_heavy:
            if quantized.passthrough_values is None:
                raise ValueError("Mixed-precision quantized keys are missing passthrough values.")
            heavy = _lib.aligned16(quantized.passthrough_values[:, self.heavy_block_ids()].float().contiguous())
        T = idx.shape[0]
        out = torch.empty(T, self.head_dim, device=idx.device, dtype=torch.float32)
        if T:
            kd = _lib.kv_desc(idx, heavy, None, T, T)
            _lib.dequantize(desc, kd, 1, 1, out)
        return out

    def forward(self, keys: torch.Tensor, *, kv_head: int | None = None) -> torch.Tensor:
        return self.dequantize(self.quantize(keys, kv_head=kv_head), kv_head=kv_head)

    def attention_scores(self, query: torch.Tensor, quantized: SunShapeQuantized, *,
                         kv_head: int | None = None) -> torch.Tensor:
        """codec.py:403-422 -- scores through the LUT kernel (no silent fallback)."""
        from .kernels import sunshape_attention_scores_strict

        return sunshape_attention_scores_strict(self, query.to(self.device).float(), quantized, kv_head=kv_head)

    def heldout_logit_mse(self, q_test: torch.Tensor, k_test: torch.Tensor) -> float:
        q_test = q_test.to(self.device).float()
        k_test = k_test.to(self.device).float()
        delta = k_test - self.forward(k_test)
        return ((q_test * delta).sum(dim=1).square()).mean().item()

    def kl_attention(self, q_test: torch.Tensor, k_test: torch.Tensor) -> float:
        import torch.nn.functional as F

        q_test = q_test.to(self.device).float()
        k_test = k_test.to(self.device).float()
        k_hat = self.forward(k_test)
        scale = math.sqrt(self.head_dim)
        p = F.softmax((q_test @ k_test.T) / scale, dim=-1)
        qd = F.softmax((q_test @ k_hat.T) / scale, dim=-1)
        return (p * (torch.log(p + 1e-9) - torch.log(qd + 1e-9))).sum(dim=-1).mean().item()
