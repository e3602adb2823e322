"""Seeded synthetic decode workloads with the shapes of the SunShape decode configs.

The reference evaluates this path only on model traces that are not available
offline, so every benchmark and parity case runs on seeded synthetic data with
the configs' shapes and value distributions:

* keys: channel ``c`` ~ N(0, s_c^2) with ``s_c = exp(0.75 * N(0, 1))`` (an
  anisotropic, log-normal-scaled Gaussian), generator seed ``seed + 0``;
* ProfilePerm: a fixed random permutation of the ``head_dim`` channels, seed ``seed + 1``;
* codebooks: per KV head and per block, 256 rows sampled (without replacement)
  from that head's permuted synthetic keys, seed ``seed + 2``;
* values and queries ~ N(0, 1) in the config dtype, seeds ``seed + 3`` / ``seed + 4``;
* SunShape-Mixed: the ``n_heavy`` blocks with the largest sum of ``s_c^2``
  after permutation are kept dense; their key values are rounded to bf16 so the
  reference's fp32 passthrough equals the bf16 copy stored here.

The same generator feeds the golden-vector script, the parity tests and the
benchmark, so every consumer sees identical inputs for identical seeds.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch

__all__ = ["DecodeConfig", "CONFIGS", "make_case"]


@dataclass(frozen=True)
class DecodeConfig:
    name: str
    batch: int
    q_heads: int
    kv_heads: int
    head_dim: int
    seq_len: int
    block_dim: int
    n_centroids: int = 256
    dtype: str = "bf16"          # query / value dtype: "f32" | "bf16" | "f16"
    n_heavy: int = 0             # SunShape-Mixed dense blocks
    query_len: int = 1

    @property
    def n_blocks(self) -> int:
        return self.head_dim // self.block_dim

    @property
    def group(self) -> int:
        return self.q_heads // self.kv_heads

    @property
    def torch_dtype(self) -> torch.dtype:
        return {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[self.dtype]

    def kv_tokens(self) -> int:
        return self.batch * self.kv_heads * self.seq_len

    def bytes_per_kv_token(self) -> int:
        """Algorithmic HBM bytes per KV token for the decode path.

        The stored index row is ``n_blocks`` bytes (uint8, heavy blocks keep a zero
        index exactly like ``codec.py:365,379``), heavy blocks add ``block_dim`` bf16
        values each, and the value row adds ``head_dim * value_bytes``.
        """
        vbytes = {"f32": 4, "bf16": 2, "f16": 2}[self.dtype]
        return self.n_blocks + self.n_heavy * self.block_dim * 2 + self.head_dim * vbytes

    def with_(self, **kw) -> "DecodeConfig":
        return replace(self, **kw)


CONFIGS: dict[str, DecodeConfig] = {
    "c1": DecodeConfig("c1", 1, 14, 2, 64, 4096, 8, dtype="f32"),
    "c2": DecodeConfig("c2", 64, 32, 8, 128, 8192, 8),
    "c3": DecodeConfig("c3", 32, 32, 8, 128, 16384, 4),
    "c4": DecodeConfig("c4", 16, 32, 8, 128, 32768, 8, n_heavy=4),
    "c5": DecodeConfig("c5", 8, 64, 8, 128, 131072, 8),
}


def _gen(seed: int, device) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(int(seed))


def _bf16_exact(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


def make_case(cfg: DecodeConfig, *, device="cpu", seed: int = 0, with_keys: bool = True,
              key_batches: int | None = None) -> dict:
    """Build one seeded decode case.

    Returns a dict with ``keys`` [B,Hkv,T,D] fp32 (or None), ``perm`` int64 [D],
    ``inv_perm``, ``centroids`` [Hkv,nb,C,bd] fp32, ``heavy_mask`` bool [nb],
    ``channel_scale`` [D], ``query`` [B,Hq,L,D] and ``value`` [B,Hkv,T,D] in the
    config dtype.  ``key_batches`` limits how many sequences of keys are drawn for
    codebook sampling when ``with_keys`` is False (large benchmark configs).
    """
    device = torch.device(device)
    B, Hq, Hkv, D, T = cfg.batch, cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.seq_len
    bd, nb, C = cfg.block_dim, cfg.n_blocks, cfg.n_centroids
    g0 = _gen(seed + 0, device)
    s_c = torch.exp(0.75 * torch.randn(D, generator=g0, device=device, dtype=torch.float32))
    perm = torch.randperm(D, generator=_gen(seed + 1, "cpu")).to(device)
    inv_perm = torch.empty_like(perm)
    inv_perm[perm] = torch.arange(D, device=device)

    heavy = torch.zeros(nb, dtype=torch.bool, device=device)
    if cfg.n_heavy > 0:
        mass = (s_c[perm] ** 2).view(nb, bd).sum(1)
        heavy[torch.argsort(mass, descending=True, stable=True)[: cfg.n_heavy]] = True
    heavy_dims = heavy.repeat_interleave(bd)[inv_perm]   # heavy flag per ORIGINAL channel

    def draw_keys(nbatch: int) -> torch.Tensor:
        k = torch.randn(nbatch, Hkv, T, D, generator=g0, device=device, dtype=torch.float32) * s_c
        if cfg.n_heavy > 0:
            k[..., heavy_dims] = _bf16_exact(k[..., heavy_dims])
        return k

    nkb = B if with_keys else max(1, min(B, key_batches or 1))
    keys = draw_keys(nkb)

    # Codebooks: 256 sampled rows of each head's permuted keys, per block.
    g2 = _gen(seed + 2, "cpu")
    centroids = torch.zeros(Hkv, nb, C, bd, dtype=torch.float32, device=device)
    pool = nkb * T
    for h in range(Hkv):
        kp = keys[:, h].reshape(-1, D)[:, perm]
        for b in range(nb):
            if heavy[b]:
                continue
            sel = torch.randperm(pool, generator=g2)[:C].to(device)
            if pool < C:
                sel = torch.cat([sel, sel.new_zeros(C - pool)])
            centroids[h, b] = kp[sel, b * bd:(b + 1) * bd]

    dt = cfg.torch_dtype
    value = torch.randn(B, Hkv, T, D, generator=_gen(seed + 3, device), device=device,
                        dtype=torch.float32).to(dt)
    query = torch.randn(B, Hq, cfg.query_len, D, generator=_gen(seed + 4, device), device=device,
                        dtype=torch.float32).to(dt)
    return {
        "cfg": cfg,
        "keys": keys if with_keys else None,
        "key_sample": None if with_keys else keys,
        "perm": perm,
        "inv_perm": inv_perm,
        "centroids": centroids,
        "heavy_mask": heavy,
        "channel_scale": s_c,
        "query": query,
        "value": value,
        "scale": 1.0 / math.sqrt(D),
    }
