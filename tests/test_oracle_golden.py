"""The CPU oracle reproduces the reference's own outputs recorded in tests/golden (no GPU)."""
import numpy as np
import pytest

from oracle import sunshape_oracle as O
from tests.helpers import GOLDEN_CASES, TOL_BF16, TOL_F32, assert_close_rowwise, load_golden, tie_space


def _heads(g, indices, passthrough):
    hm = g["heavy_mask"]
    heads = []
    for b in range(g["B"]):
        for h in range(g["Hkv"]):
            heads.append((indices[b, h], hm if hm.any() else None, passthrough[b, h] if hm.any() else None))
    return heads


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_oracle_quantize_matches_reference(name):
    g = load_golden(name)
    hm = g["heavy_mask"]
    for b in range(g["B"]):
        for h in range(g["Hkv"]):
            idx, pt = O.quantize(g["keys"][b, h], g["perm"], g["centroids"][h], hm, E=g["E"])
            assert idx.dtype == np.uint8
            kp, cents = tie_space(g["keys"][b, h][:, g["perm"]], g["centroids"][h], g["E"])
            n_mis, n_bad = O.index_mismatches_are_ties(kp, cents, idx, g["ref_indices"][b, h], hm)
            assert n_bad == 0, f"{n_mis} mismatches, {n_bad} not ties"
            if hm.any():
                np.testing.assert_array_equal(pt, g["ref_passthrough"][b, h])


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_oracle_scores_match_reference(name):
    g = load_golden(name)
    G, L, D = g["Hq"] // g["Hkv"], g["L"], g["D"]
    hm = g["heavy_mask"]
    for b in range(g["B"]):
        for h in range(g["Hkv"]):
            q = g["query"][b, h * G:(h + 1) * G].reshape(-1, D)
            if g["scale"] is not None:
                q = O.round_to(q * np.float32(g["scale"]), g["dtype"])
            s = O.attention_scores(q, g["ref_indices"][b, h], g["centroids"][h], g["inv_perm"],
                                   hm if hm.any() else None, g["ref_passthrough"][b, h] if hm.any() else None)
            assert_close_rowwise(s, g["ref_scores"][b, h], TOL_F32, f"{name} scores")
            s2 = O.lut_scores(q, g["ref_indices"][b, h], g["centroids"][h], g["perm"], hm if hm.any() else None,
                              g["ref_passthrough"][b, h] if hm.any() else None)
            assert_close_rowwise(s2, g["ref_scores"][b, h], TOL_F32, f"{name} lut scores")


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_oracle_attention_matches_reference(name):
    g = load_golden(name)
    out = O.apply_quantized_attention(
        g["query"], _heads(g, g["ref_indices"], g["ref_passthrough"]), g["value"],
        centroids_for_head=lambda h: g["centroids"][h], inv_perm=g["inv_perm"], attn_mask=g["mask"],
        scale=g["scale"], query_dtype=g["dtype"], value_dtype=g["dtype"])
    tol = TOL_F32 if g["dtype"] == "f32" else TOL_BF16
    assert_close_rowwise(out, g["ref_out"], tol, f"{name} out")


@pytest.mark.parametrize("name", ["g1_c1_fp32", "g2_bf16_mask4d"])
def test_oracle_shard_merge_equals_full(name):
    """Size-independent property of the KV split: merging per-shard partials gives the full softmax."""
    g = load_golden(name)
    if g["mask"] is not None:
        pytest.skip("partials helper has no mask")
    T = g["T"]
    heads = _heads(g, g["ref_indices"], g["ref_passthrough"])
    full = O.decode_partials(g["query"], heads, g["value"], centroids_for_head=lambda h: g["centroids"][h],
                             inv_perm=g["inv_perm"], scale=g["scale"], query_dtype=g["dtype"])
    ref = full[2] / full[1][..., None]
    ms, ls, accs = [], [], []
    bounds = [0, T // 3, T // 2 + 5, T]
    for a, b in zip(bounds[:-1], bounds[1:]):
        sh = [(i[a:b], hm, None if p is None else p[a:b]) for (i, hm, p) in heads]
        m, l, acc = O.decode_partials(g["query"], sh, g["value"][:, :, a:b],
                                      centroids_for_head=lambda h: g["centroids"][h], inv_perm=g["inv_perm"],
                                      scale=g["scale"], query_dtype=g["dtype"])
        ms.append(m); ls.append(l); accs.append(acc)
    merged = O.merge_partials(ms, ls, accs)
    np.testing.assert_allclose(merged, ref, rtol=1e-10, atol=1e-12)


def test_bf16_round_ties_to_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, np.inf], dtype=np.float32)
    r = O.bf16_round(x)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == 1.015625 and r[3] == -2.5 and np.isinf(r[4])
