"""TurboQuant-MSE counterpart (the reference's comparison baseline, ``sunshape/turbo_baseline.py``)
with its attention scores on the LUT-scores kernel of this library.

TurboQuant-MSE (Zandieh et al., arXiv 2504.19874, Algorithm 1) normalises a key, rotates it by a
random orthogonal matrix and scalar-quantizes every rotated coordinate to the nearest of 2^bits
centroids.  Scores against the compressed keys (``TurboQuantMSE.attention_scores``,
``turbo_baseline.py:171-186``) are ``norm_t * sum_d (q R^T)_d * centroid[idx_t,d]``: a block-VQ score
with block_dim 1, head_dim blocks and one shared 2^bits-entry codebook, so they run on
``sunshape_attention_scores_packed`` (per-row LUT in shared memory, indices bit-packed at 1, 2 or 4
bits or stored as uint8) followed by the per-token norm scale.

Rotation and centroid table follow the published construction the reference uses: Q of the QR
decomposition of a seeded Gaussian matrix (CPU generator) with column signs fixed so R has a positive
diagonal; centroids +-sqrt(2 / (pi d)) at 1 bit, +-0.453 / sqrt(d) and +-1.51 / sqrt(d) at 2 bits,
and midpoints of 2^bits equal cells of [-3 / sqrt(d), 3 / sqrt(d)] above.  Quantization (one rotation
GEMM and a nearest-centroid search per coordinate) runs as cuBLAS / elementwise GPU work: it is not on
the SunShape decode path.
"""
from __future__ import annotations

import math
from typing import NamedTuple

import torch

from . import _lib


def generate_rotation(d: int, seed: int = 0, device: torch.device | None = None) -> torch.Tensor:
    gen = torch.Generator(device="cpu").manual_seed(int(seed))
    a = torch.randn(d, d, generator=gen)
    q, r = torch.linalg.qr(a)
    q = q * torch.sign(torch.diagonal(r)).unsqueeze(0)
    return q.float().to(device) if device is not None else q.float()


def scalar_centroids(d: int, bits: int) -> torch.Tensor:
    if bits == 1:
        c = math.sqrt(2.0 / (math.pi * d))
        return torch.tensor([-c, c])
    if bits == 2:
        s = 1.0 / math.sqrt(d)
        return torch.tensor([-1.51 * s, -0.453 * s, 0.453 * s, 1.51 * s])
    sigma = 1.0 / math.sqrt(d)
    edges = torch.linspace(-3.0 * sigma, 3.0 * sigma, 2 ** bits + 1)
    return (edges[:-1] + edges[1:]) / 2.0


class TurboQuantCompressed(NamedTuple):
    """Compressed keys: indices [n, d] (uint8, or bit-packed rows when ``bits`` <= 4) and norms [n]."""

    indices: torch.Tensor
    norms: torch.Tensor
    bits: int
    dim: int
    packed: bool


class TurboQuantMSE:
    def __init__(self, dim: int, bits: int = 1, seed: int = 0, device: torch.device | None = None):
        if not 1 <= bits <= 8:
            raise ValueError("bits must be in [1, 8]")
        self.dim, self.bits = int(dim), int(bits)
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda" if torch.cuda.is_available() else "cpu")
        self.rotation = generate_rotation(self.dim, seed, self.device)
        self.centroids = scalar_centroids(self.dim, self.bits).to(self.device)
        self._desc = None

    # ------------------------------------------------------------------ quantize / dequantize
    def quantize(self, x: torch.Tensor):
        """(indices [n, d] int64, norms [n]) as ``turbo_baseline.py:137-153``."""
        x = x.to(self.device).float()
        norms = x.norm(dim=-1, keepdim=True).clamp(min=1e-8)
        y = (x / norms) @ self.rotation.T
        idx = (y.unsqueeze(-1) - self.centroids).abs().argmin(dim=-1)
        return idx, norms.squeeze(-1)

    def dequantize(self, indices: torch.Tensor, norms: torch.Tensor) -> torch.Tensor:
        return (self.centroids[indices.long()] @ self.rotation) * norms.unsqueeze(-1)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        idx, norms = self.quantize(x)
        return self.dequantize(idx, norms)

    def compress(self, x: torch.Tensor) -> TurboQuantCompressed:
        """Storage form: uint8 indices, bit-packed at 1, 2 and 4 bits."""
        idx, norms = self.quantize(x)
        idx8 = idx.to(torch.uint8)
        if self.bits in (1, 2, 4):
            return TurboQuantCompressed(_lib.pack_indices(idx8, self.bits), norms, self.bits, self.dim, True)
        return TurboQuantCompressed(idx8.contiguous(), norms, self.bits, self.dim, False)

    # ------------------------------------------------------------------ scores
    def _score_desc(self):
        if self._desc is None:
            C = self.centroids.numel()
            cents = self.centroids.view(1, 1, C, 1).expand(1, self.dim, C, 1).contiguous()   # one table per block
            ident = torch.arange(self.dim, device=self.device, dtype=torch.int64)
            self._desc = (_lib.codec_desc(cents, ident, None, 0, self.dim, 1, None), (cents, ident))
        return self._desc

    def attention_scores(self, query: torch.Tensor, compressed) -> torch.Tensor:
        """``q R^T`` against the compressed keys (turbo_baseline.py:171-186), scores [n_q, n] fp32."""
        if isinstance(compressed, TurboQuantCompressed):
            idx, norms, packed = compressed.indices, compressed.norms, compressed.packed
        else:   # the reference's TurboQuantized: indices [n, d], norms in qjl_norms
            idx, norms, packed = compressed.indices.to(torch.uint8), compressed.qjl_norms, False
        if not idx.is_cuda:
            raise RuntimeError("sunshape_b200 runs only on CUDA tensors (B200, sm_100a); there is no CPU fallback.")
        q_rot = query.to(self.device).float() @ self.rotation.T
        desc, _keep = self._score_desc()
        bits = self.bits if packed else 8
        idx = idx.contiguous()
        n_q, n = q_rot.shape[0], idx.shape[0]
        out = torch.empty(n_q, n, device=self.device, dtype=torch.float32)
        for r0 in range(0, n_q, 16):
            rows = min(16, n_q - r0)
            _lib.attention_scores_packed(desc, idx, bits, n, n, q_rot[r0:r0 + rows].contiguous(), 1, 1, rows,
                                         out[r0:r0 + rows])
        if norms is not None:
            out.mul_(norms.to(out.device).float().unsqueeze(0))
        return out


__all__ = ["TurboQuantMSE", "TurboQuantCompressed", "generate_rotation", "scalar_centroids"]
