"""Shared test helpers: golden fixtures, codec construction and tolerance checks."""
from __future__ import annotations

import glob
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
# per-case decode fixtures; g7_bundle (reference bundle decode) and g8_cache (reference HF cache) have their own tests
GOLDEN_CASES = sorted(n for n in (os.path.splitext(os.path.basename(p))[0]
                                  for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))
                      if n not in ("g7_bundle", "g8_cache", "g11_turbo"))

# tolerances stated by the north star: fp32 accumulation rel 1e-5, bf16 outputs 2e-2
TOL_F32 = 1e-5
TOL_BF16 = 2e-2


def load_golden(name: str) -> dict:
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    g = {k: z[k] for k in z.files}
    for k in ("B", "Hq", "Hkv", "D", "T", "L", "block_dim", "n_centroids"):
        g[k] = int(g[k])
    g["dtype"] = str(g["dtype"])
    s = float(g["scale"])
    g["scale"] = None if np.isnan(s) else s
    g["mask"] = g["mask"] if g["mask"].size else None
    g["E"] = g.get("E")            # SunShape-Pro local metric (block-diagonal [D, D]) or None
    return g


def tie_space(keys_perm, centroids, E=None):
    """(keys, codebooks) in the space the reference measures distances in: as given, or transformed by
    the SunShape-Pro metric blocks (codec.py:375-377)."""
    if E is None:
        return keys_perm, centroids
    from oracle import sunshape_oracle as O

    return O.metric_transform(keys_perm, centroids, E)


def torch_dtype(name: str):
    return {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[name]


def make_codec(perm, centroids, heavy_mask, head_dim, block_dim, n_centroids, device, E=None):
    """SunShapeBlockCodec with per-KV-head codebooks written directly (no fitting); with ``E`` (a
    block-diagonal [D, D] metric) a SunShape-Pro codec."""
    from sunshape_b200.codec import SunShapeBlockCodec

    perm = torch.as_tensor(perm, dtype=torch.long).cpu()
    cents = torch.as_tensor(centroids, dtype=torch.float32).cpu()
    heavy = torch.as_tensor(heavy_mask, dtype=torch.bool).cpu()
    mode = "profileperm_mixed_precision" if bool(heavy.any()) else "profileperm_baseline"
    if E is not None:
        mode = "profileperm_localmetric_dsq"
    codec = SunShapeBlockCodec(head_dim=head_dim, block_dim=block_dim, n_centroids=n_centroids, mode=mode,
                               device=torch.device(device), kv_heads=cents.shape[0] if cents.ndim == 4 else None)
    codec.permutation.copy_(perm)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(len(perm), device=perm.device)
    codec.inv_permutation.copy_(inv)
    codec.centroids.copy_(cents)
    codec.mixed_high_precision_blocks.copy_(heavy)
    if E is not None:
        Et = torch.as_tensor(E, dtype=torch.float32)
        codec.E.copy_(Et)
        codec.E_inv.copy_(torch.linalg.pinv(Et))
    codec.invalidate()
    return codec


def assert_close_rowwise(actual, expected, rtol, what=""):
    """Per-row tolerance: for every row (the last axis: one output row of one query head, or one
    score row), max |actual - expected| <= rtol * max |expected| over that row.  NaN patterns
    (fully masked rows) must agree exactly."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, (a.shape, e.shape)
    nan_a, nan_e = np.isnan(a), np.isnan(e)
    assert (nan_a == nan_e).all(), f"{what}: NaN pattern differs ({nan_a.sum()} vs {nan_e.sum()})"
    if e.size == 0:
        return
    a2 = np.where(nan_e, 0.0, a).reshape(-1, e.shape[-1])
    e2 = np.where(nan_e, 0.0, e).reshape(-1, e.shape[-1])
    scale = np.maximum(np.abs(e2).max(axis=1), 1e-30)
    err = np.abs(a2 - e2).max(axis=1)
    bad = err > rtol * scale
    if bad.any():
        r = int(np.argmax(err / scale))
        raise AssertionError(f"{what}: {int(bad.sum())} of {len(bad)} rows out of tolerance; worst row {r}: "
                             f"max err {err[r]:.3e} > {rtol:.1e} * {scale[r]:.3e}")
