"""Fixtures written by the reference itself (tests/golden/make_golden.py), checked on the CPU:

* ``bundle_ref.pt`` -- a bundle saved by the reference's ``SunShapeBundle.save`` (hf.py:273-303)
  loads through ``sunshape_b200.hf.SunShapeBundle.load`` with every buffer intact, and a bundle saved
  here has the same structure;
* ``g7_bundle.npz`` -- the reference's decode of that bundle's layers through its public backend
  (quantize_key_states -> SunShapeAttentionImpl.forward), reproduced by the oracle;
* ``g8_cache.npz`` -- the keys / values the reference's ``SunShapeCache.update`` stores over a
  prefill and two decode steps, reproduced by the oracle (quantize -> dequantize -> key dtype).
"""
import os

import numpy as np
import torch

from oracle import sunshape_oracle as O
from tests.helpers import GOLDEN_DIR, TOL_BF16, assert_close_rowwise

BUNDLE = os.path.join(GOLDEN_DIR, "bundle_ref.pt")


def _g7():
    z = np.load(os.path.join(GOLDEN_DIR, "g7_bundle.npz"))
    return {k: z[k] for k in z.files}


def test_reference_bundle_loads_with_every_buffer():
    from sunshape_b200.hf import SunShapeBundle

    raw = torch.load(BUNDLE, map_location="cpu", weights_only=False)
    b = SunShapeBundle.load(BUNDLE, device=torch.device("cpu"))
    assert b.layers == [3, 5] and sorted(b.codecs) == [3, 5]
    assert b.model_name == raw["model_name"] and b.block_dim == raw["block_dim"]
    assert b.codecs[3].mode == "profileperm_baseline"
    assert b.codecs[5].mode == "profileperm_mixed_precision"
    for layer, codec in b.codecs.items():
        ref_sd = raw["codecs"][str(layer)]["state_dict"]
        ours = codec.state_dict()
        assert set(ours) == set(ref_sd)
        for k, v in ref_sd.items():
            assert torch.equal(ours[k].cpu(), v), (layer, k)
        assert codec.n_codebooks == 1          # the reference layout: one codebook per layer
    # saving here gives the same structure the reference's loader reads
    again = b.state_dict()
    assert again.keys() == raw.keys()
    for layer in ("3", "5"):
        assert again["codecs"][layer].keys() == raw["codecs"][layer].keys()


def test_oracle_reproduces_reference_bundle_decode():
    raw = torch.load(BUNDLE, map_location="cpu", weights_only=False)
    z = _g7()
    for layer in z["layers"]:
        sd = raw["codecs"][str(layer)]["state_dict"]
        pre = f"l{layer}_"
        cents = sd["centroids"].numpy()
        perm, inv = sd["permutation"].numpy(), sd["inv_permutation"].numpy()
        hm = sd["mixed_high_precision_blocks"].numpy()
        mixed = raw["codecs"][str(layer)]["mode"] == "profileperm_mixed_precision"
        keys = z[pre + "keys"]
        B, H, T, _ = keys.shape
        heads = []
        for b in range(B):
            for h in range(H):
                idx, pt = O.quantize(keys[b, h], perm, cents, hm if mixed else None)
                n_mis, n_bad = O.index_mismatches_are_ties(keys[b, h][:, perm], cents, idx,
                                                           z[pre + "ref_indices"][b, h], hm if mixed else None)
                assert n_bad == 0, f"layer {layer}: {n_mis} mismatches, {n_bad} not ties"
                heads.append((idx, hm if mixed else None, pt if mixed else None))
        dt = str(z[pre + "dtype"])
        out = O.apply_quantized_attention(z[pre + "query"], heads, z[pre + "value"], centroids_for_head=lambda h: cents,
                                          inv_perm=inv, scale=float(z[pre + "scale"]), query_dtype=dt, value_dtype=dt)
        assert_close_rowwise(out, z[pre + "ref_out"], TOL_BF16, f"layer {layer}")


def test_oracle_reproduces_reference_cache_keys():
    z = np.load(os.path.join(GOLDEN_DIR, "g8_cache.npz"))
    keys, perm, inv, cents = z["keys"], z["perm"], z["inv_perm"], z["centroids"]
    B, H, _, D = keys.shape
    a, b = z["steps"][-1]
    stored = z[f"step{len(z['steps']) - 1}_l1_keys"]
    assert stored.shape == (B, H, b, D)
    np.testing.assert_array_equal(z[f"step{len(z['steps']) - 1}_l0_keys"], keys[:, :, :b])
    for bb in range(B):
        for h in range(H):
            idx, _ = O.quantize(keys[bb, h, :b], perm, cents)
            k_hat = O.bf16_round(O.dequantize(idx, cents, inv))
            np.testing.assert_array_equal(k_hat, stored[bb, h])
