"""TurboQuant-MSE counterpart against the reference's own outputs (tests/golden/g11_turbo.npz):
rotation and centroid table on the CPU; indices, round trip and compressed-key attention scores on
the GPU (scores on the LUT-scores kernel, bit-packed at 1 and 2 bits)."""
import os

import numpy as np
import pytest
import torch

from tests.helpers import GOLDEN_DIR, TOL_F32, assert_close_rowwise

Z = os.path.join(GOLDEN_DIR, "g11_turbo.npz")


@pytest.mark.parametrize("bits", [1, 2, 3])
def test_rotation_and_centroids_match_reference(bits):
    from sunshape_b200.turbo import generate_rotation, scalar_centroids

    z = np.load(Z)
    np.testing.assert_array_equal(generate_rotation(128, 5 + bits).numpy(), z[f"b{bits}_rotation"])
    np.testing.assert_array_equal(scalar_centroids(128, bits).float().numpy(), z[f"b{bits}_centroids"])


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [1, 2, 3])
def test_turbo_scores_match_reference(bits):
    from sunshape_b200.turbo import TurboQuantMSE

    z = np.load(Z)
    tq = TurboQuantMSE(128, bits=bits, seed=5 + bits, device=torch.device("cuda"))
    x = torch.from_numpy(z["x"]).cuda()
    q = torch.from_numpy(z["q"]).cuda()
    idx, norms = tq.quantize(x)
    mism = (idx.cpu().numpy() != z[f"b{bits}_indices"]).mean()
    assert mism < 1e-3, mism                       # coordinates exactly between two centroids may differ
    comp = tq.compress(x)
    assert comp.packed == (bits in (1, 2))
    s = tq.attention_scores(q, comp)
    ref_idx_scores = tq.attention_scores(
        q, type(comp)(torch.from_numpy(z[f"b{bits}_indices"]).cuda(), norms, bits, 128, False))
    assert_close_rowwise(ref_idx_scores.cpu().numpy(), z[f"b{bits}_scores"], TOL_F32, f"scores b{bits}")
    if mism == 0:
        assert_close_rowwise(s.cpu().numpy(), z[f"b{bits}_scores"], TOL_F32, f"scores from packed b{bits}")
    assert_close_rowwise(tq(x).cpu().numpy(), z[f"b{bits}_roundtrip"], 1e-5, f"round trip b{bits}")


@pytest.mark.gpu
def test_turbo_cache_for_layers_round_trips_keys():
    from sunshape_b200.turbo_cache import TurboQuantCache, TurboQuantLayer

    cache = TurboQuantCache.for_layers(head_dims={1: 64}, layers=[1], num_layers=2, bits=2, device=torch.device("cuda"))
    assert isinstance(cache.layers[1], TurboQuantLayer)
    k = torch.randn(1, 2, 5, 64, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(1, 2, 5, 64, device="cuda", dtype=torch.bfloat16)
    ko, vo = cache.update(k, v, 1)
    assert ko.dtype == torch.bfloat16 and torch.equal(vo, v)
    ref = cache.layers[1].quantizer(k.reshape(-1, 64).float()).reshape(k.shape).to(torch.bfloat16)
    assert torch.equal(ko, ref)
