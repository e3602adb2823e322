"""CPU oracle for the SunShape quantized-key decode path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference's own CPU arithmetic for the hot
path so that the CUDA library can be checked against it.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it, and only as the checker or the timed CPU
baseline.  The product (``sunshape_b200``) never imports it and has no CPU
fallback.

Parity pinning: the reference ships no tests or golden vectors for this path.
The restatement is pinned against golden vectors produced by running the
reference code itself (``tests/golden/make_golden.py`` imports the reference
package and records its outputs on seeded inputs); ``tests/test_oracle_golden.py``
checks every function below against those vectors.

Citations are ``path:line`` inside the reference project (gauravsaini/sunshape).
The distance arithmetic of ``codec.quantize`` lives in torch 2.11.0
(``torch.cdist``'s matrix-multiply path, ``argmin`` first-index-on-ties); its
published algorithm is restated in :func:`cdist_mm_fp32`.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "compact_index_dtype", "invert_permutation", "cdist_mm_fp32", "exact_block_distances",
    "quantize", "dequantize", "attention_scores", "query_centroid_lut",
    "lut_scores", "apply_quantized_attention", "merge_partials", "bf16_round",
    "index_mismatches_are_ties", "metric_transform",
]


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even), returned as fp32."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32).copy()
    nan = np.isnan(a)
    out[nan] = np.float32("nan")
    return out


def f16_round(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16_round(x)
    if dtype == "f16":
        return f16_round(x)
    return np.asarray(x, dtype=np.float32)


def compact_index_dtype(n_centroids: int):
    """codec.py:78-83 -- uint8 up to 256 codewords, int16 up to 65535, else int32."""
    if n_centroids <= 256:
        return np.uint8
    if n_centroids <= 65535:
        return np.int16
    return np.int32


def invert_permutation(perm: np.ndarray) -> np.ndarray:
    """codec.py:86-89."""
    inv = np.empty_like(perm)
    inv[perm] = np.arange(len(perm), dtype=perm.dtype)
    return inv


def cdist_mm_fp32(x: np.ndarray, c: np.ndarray) -> np.ndarray:
    """Euclidean distances as torch.cdist computes them for >25 rows (codec.py:376).

    torch's matrix-multiply path augments both operands --
    ``[-2x, |x|^2, 1] @ [c, 1, |c|^2]^T`` -- clamps at zero and takes the square
    root, all in fp32.  BLAS summation order is not reproducible bit-for-bit,
    so near-ties may resolve differently; :func:`index_mismatches_are_ties`
    decides whether such a disagreement is a tie.
    """
    x = x.astype(np.float32)
    c = c.astype(np.float32)
    xn = (x * x).sum(-1, dtype=np.float32, keepdims=True)
    cn = (c * c).sum(-1, dtype=np.float32, keepdims=True)
    xa = np.concatenate([-2.0 * x, xn, np.ones_like(xn)], axis=-1).astype(np.float32)
    ca = np.concatenate([c, np.ones_like(cn), cn], axis=-1).astype(np.float32)
    d2 = xa @ ca.T
    return np.sqrt(np.maximum(d2, np.float32(0.0)))


def exact_block_distances(keys_perm_block: np.ndarray, cents_block: np.ndarray) -> np.ndarray:
    """Squared distances in fp64 by direct differences (the tie arbiter)."""
    diff = keys_perm_block.astype(np.float64)[:, None, :] - cents_block.astype(np.float64)[None, :, :]
    return (diff * diff).sum(-1)


def metric_transform(keys_perm: np.ndarray, centroids: np.ndarray, E: np.ndarray):
    """SunShape-Pro (profileperm_localmetric_dsq) distance space, codec.py:375-377: key block b and the
    block's codewords both multiplied by the metric block E[b*bd:(b+1)*bd, b*bd:(b+1)*bd] (transposed)
    in fp32.  Returns (transformed keys [T, D], transformed codebooks [nb, C, bd])."""
    nb, C, bd = centroids.shape
    kt = np.empty_like(keys_perm, dtype=np.float32)
    ct = np.empty_like(centroids, dtype=np.float32)
    for b in range(nb):
        sl = slice(b * bd, (b + 1) * bd)
        eb = np.asarray(E[sl, sl], dtype=np.float32)
        kt[:, sl] = keys_perm[:, sl].astype(np.float32) @ eb.T
        ct[b] = centroids[b].astype(np.float32) @ eb.T
    return kt, ct


def quantize(keys: np.ndarray, perm: np.ndarray, centroids: np.ndarray,
             heavy_mask: np.ndarray | None = None, E: np.ndarray | None = None):
    """SunShapeBlockCodec.quantize, codec.py:362-385 (E = I for the ProfilePerm modes; the
    SunShape-Pro metric E when given, compared in the transformed space, codec.py:375-377).

    keys [T, D] -> (indices [T, nb] compact dtype, passthrough [T, nb, bd] fp32 or None).
    Heavy (Mixed) blocks copy the permuted keys into the passthrough tensor and keep index 0.
    """
    if E is not None:
        kt, ct = metric_transform(np.asarray(keys, dtype=np.float32)[:, perm], centroids, E)
        return quantize(kt, np.arange(kt.shape[1]), ct, heavy_mask)
    keys = np.asarray(keys, dtype=np.float32)
    nb, C, bd = centroids.shape
    kp = keys[:, perm]                                        # codec.py:247-252
    idx = np.zeros((keys.shape[0], nb), dtype=np.int64)       # codec.py:365
    passthrough = None
    if heavy_mask is not None and heavy_mask.any():           # codec.py:367-368
        passthrough = np.zeros((keys.shape[0], nb, bd), dtype=np.float32)
    for b in range(nb):                                       # codec.py:369-377
        sl = slice(b * bd, (b + 1) * bd)
        if heavy_mask is not None and heavy_mask[b]:
            if passthrough is not None:
                passthrough[:, b, :] = kp[:, sl]
            continue
        d = cdist_mm_fp32(kp[:, sl], centroids[b])
        idx[:, b] = d.argmin(-1)
    return idx.astype(compact_index_dtype(C)), passthrough


def dequantize(indices: np.ndarray, centroids: np.ndarray, inv_perm: np.ndarray,
               heavy_mask: np.ndarray | None = None, passthrough: np.ndarray | None = None) -> np.ndarray:
    """SunShapeBlockCodec.dequantize, codec.py:387-398."""
    nb, C, bd = centroids.shape
    T = indices.shape[0]
    k_hat = np.zeros((T, nb * bd), dtype=np.float32)
    idx = indices.astype(np.int64)
    for b in range(nb):
        sl = slice(b * bd, (b + 1) * bd)
        if heavy_mask is not None and heavy_mask[b]:
            if passthrough is None:
                raise ValueError("Mixed-precision quantized keys are missing passthrough values.")
            k_hat[:, sl] = passthrough[:, b, :]
        else:
            k_hat[:, sl] = centroids[b][idx[:, b]]
    return k_hat[:, inv_perm]                                 # codec.py:254-256


def attention_scores(query: np.ndarray, indices, centroids, inv_perm, heavy_mask=None,
                     passthrough=None) -> np.ndarray:
    """_torch_attention_scores, triton_kernels.py:300-311: query @ dequantize(...)^T in fp32."""
    k_hat = dequantize(indices, centroids, inv_perm, heavy_mask, passthrough)
    return np.asarray(query, dtype=np.float32) @ k_hat.T


def query_centroid_lut(query_perm: np.ndarray, centroids: np.ndarray) -> np.ndarray:
    """_precompute_query_centroid_dots, triton_kernels.py:381-408: qdots[q,b,c]."""
    nb, C, bd = centroids.shape
    qb = np.asarray(query_perm, dtype=np.float32).reshape(query_perm.shape[0], nb, bd)
    return np.einsum("qbd,bcd->qbc", qb, centroids.astype(np.float32))


def lut_scores(query: np.ndarray, indices, centroids, perm, heavy_mask=None, passthrough=None):
    """_sunshape_precomputed_scores_kernel semantics, triton_kernels.py:134-204 (+ Mixed dense dot).

    score[q,t] = sum_b qdots[q,b,idx[t,b]] over light blocks + dense dot over heavy blocks.
    """
    nb, C, bd = centroids.shape
    qp = np.asarray(query, dtype=np.float32)[:, perm]
    lut = query_centroid_lut(qp, centroids)
    idx = indices.astype(np.int64)
    s = np.zeros((qp.shape[0], idx.shape[0]), dtype=np.float64)
    for b in range(nb):
        if heavy_mask is not None and heavy_mask[b]:
            s += qp[:, b * bd:(b + 1) * bd].astype(np.float64) @ passthrough[:, b, :].T.astype(np.float64)
        else:
            s += lut[:, b, :][:, idx[:, b]]
    return s.astype(np.float32)


def _mask_slice(attn_mask, b, q0, q1, batch):
    """_select_attn_mask_slice, vllm_attn_backend.py:197-213."""
    if attn_mask is None:
        return None
    if attn_mask.ndim == 2:
        return attn_mask[None]
    if attn_mask.ndim == 3:
        if attn_mask.shape[0] == batch:
            return attn_mask[b][None]
        return attn_mask[q0:q1]
    return attn_mask[b, q0:q1]


def apply_quantized_attention(query: np.ndarray, heads: list, value: np.ndarray, *,
                              centroids_for_head, inv_perm: np.ndarray, attn_mask=None,
                              scale=None, query_dtype: str = "f32", value_dtype: str = "f32"):
    """_apply_quantized_attention, vllm_attn_backend.py:216-253.

    query [B,Hq,L,D] and value [B,Hkv,T,Dv] hold values already representable in
    their dtype (given by ``query_dtype``/``value_dtype``); ``heads[b*Hkv+h]`` is
    ``(indices, heavy_mask, passthrough)``; ``centroids_for_head(h)`` returns the
    codebook of KV head ``h``.  Mirrors the reference's dtype steps: the query is
    scaled in its own dtype (``:235-236``), scores are fp32, softmax is fp32 and the
    probabilities are cast to the value dtype before ``P @ V`` (``:251-252``).
    """
    B, Hq, L, D = query.shape
    _, Hkv, T, Dv = value.shape
    G = Hq // Hkv
    out = np.empty((B, Hq, L, Dv), dtype=np.float32)
    for b in range(B):
        for h in range(Hkv):
            q0, q1 = h * G, (h + 1) * G
            qs = np.asarray(query[b, q0:q1], dtype=np.float32)
            if scale is not None:
                qs = round_to(qs * np.float32(scale), query_dtype)
            idx, hm, pt = heads[b * Hkv + h]
            scores = attention_scores(qs.reshape(-1, D), idx, centroids_for_head(h), inv_perm, hm, pt)
            scores = scores.reshape(G, L, T)
            ms = _mask_slice(attn_mask, b, q0, q1, B)
            if ms is not None:
                scores = scores + np.asarray(ms, dtype=np.float32)
            mx = scores.max(-1, keepdims=True)
            with np.errstate(invalid="ignore", over="ignore"):
                e = np.exp(scores - mx)
                probs = e / e.sum(-1, keepdims=True)
            probs = round_to(probs, value_dtype)
            out[b, q0:q1] = (probs.astype(np.float32) @ np.asarray(value[b, h], dtype=np.float32))
    return round_to(out, value_dtype)


def decode_partials(query, heads, value, *, centroids_for_head, inv_perm, scale=None, query_dtype="f32"):
    """Unnormalised (m, l, acc) of one KV shard: the quantities a KV-sequence split merges.

    m = max_t s, l = sum_t exp(s - m), acc = sum_t exp(s - m) v_t (fp64 accumulation).
    """
    B, Hq, L, D = query.shape
    _, Hkv, T, Dv = value.shape
    G = Hq // Hkv
    m = np.empty((B, Hq, L)); l = np.empty((B, Hq, L)); acc = np.empty((B, Hq, L, Dv))
    for b in range(B):
        for h in range(Hkv):
            qs = np.asarray(query[b, h * G:(h + 1) * G], dtype=np.float32)
            if scale is not None:
                qs = round_to(qs * np.float32(scale), query_dtype)
            idx, hm, pt = heads[b * Hkv + h]
            s = attention_scores(qs.reshape(-1, D), idx, centroids_for_head(h), inv_perm, hm, pt)
            s = s.reshape(G, L, T).astype(np.float64)
            mm = s.max(-1)
            e = np.exp(s - mm[..., None])
            m[b, h * G:(h + 1) * G] = mm
            l[b, h * G:(h + 1) * G] = e.sum(-1)
            acc[b, h * G:(h + 1) * G] = e @ np.asarray(value[b, h], dtype=np.float64)
    return m, l, acc


def merge_partials(ms, ls, accs):
    """Log-sum-exp merge of per-shard partials: M = max m_r, L = sum l_r e^(m_r-M), O = sum acc_r e^(m_r-M) / L."""
    M = np.max(np.stack(ms), axis=0)
    L = sum(l * np.exp(m - M) for m, l in zip(ms, ls))
    A = sum(a * np.exp(m - M)[..., None] for m, a in zip(ms, accs))
    return A / L[..., None]


def index_mismatches_are_ties(keys_perm: np.ndarray, centroids: np.ndarray, idx_a: np.ndarray,
                              idx_b: np.ndarray, heavy_mask=None, rtol: float = 1e-5):
    """Return (n_mismatch, n_non_tie) for two index tensors [T, nb].

    A mismatch is an exact-distance tie when the fp64 squared distances of the
    two chosen codewords differ by at most ``rtol`` relative to the key block's
    squared norm plus the distance itself -- the scale of fp32 rounding in the
    reference's ``|x|^2 + |c|^2 - 2 x.c`` distance (:func:`cdist_mm_fp32`).
    """
    nb, C, bd = centroids.shape
    a = idx_a.astype(np.int64); b_ = idx_b.astype(np.int64)
    n_mis = 0; n_bad = 0
    for blk in range(nb):
        if heavy_mask is not None and heavy_mask[blk]:
            continue
        rows = np.nonzero(a[:, blk] != b_[:, blk])[0]
        if rows.size == 0:
            continue
        n_mis += rows.size
        kb = keys_perm[rows, blk * bd:(blk + 1) * bd].astype(np.float64)
        ca = centroids[blk][a[rows, blk]].astype(np.float64)
        cb = centroids[blk][b_[rows, blk]].astype(np.float64)
        da = ((kb - ca) ** 2).sum(-1); db = ((kb - cb) ** 2).sum(-1)
        scale = (kb ** 2).sum(-1) + np.maximum(da, db)
        n_bad += int((np.abs(da - db) > rtol * scale).sum())
    return n_mis, n_bad
