"""The reference-facing entry points on the GPU against outputs recorded from the reference itself:

* ``SunShapeAttentionImpl.forward`` (vllm_attn_backend.py:271-305), reached through the runtime
  registry (``register_runtime_state``), on every per-case golden;
* a bundle saved by the reference (``bundle_ref.pt``): load, ``quantize_key_states`` and ``forward``
  per layer, against the reference's own decode of that bundle (``g7_bundle.npz``), also through
  ``install_sunshape_hooks`` from the file;
* ``SunShapeCache.update`` (cache.py:32-46) over a prefill and two decode steps, against what the
  reference's cache stored (``g8_cache.npz``).
"""
import os

import numpy as np
import pytest
import torch

from sunshape_b200 import vllm_attn_backend as vab
from sunshape_b200.hf import SunShapeBundle
from sunshape_b200.integration.vllm import runtime_state_from_bundle
from tests.helpers import (GOLDEN_CASES, GOLDEN_DIR, TOL_BF16, TOL_F32, assert_close_rowwise, load_golden, make_codec,
                           torch_dtype)
from tests.test_gpu_parity import golden_codec, golden_keys

pytestmark = pytest.mark.gpu
DEV = "cuda"
BUNDLE = os.path.join(GOLDEN_DIR, "bundle_ref.pt")


@pytest.fixture
def registry():
    yield
    vab.clear_registered_runtime()
    vab.clear_registered_handle()


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_forward_through_registry_matches_reference(name, registry):
    g = load_golden(name)
    codec = golden_codec(g)
    bundle = SunShapeBundle("golden", [7], 1.0, g["block_dim"], "sunshape_base", 0, 0, 0, {7: codec})
    vab.register_runtime_state(runtime_state_from_bundle(bundle))
    dt = torch_dtype(g["dtype"])
    q = torch.from_numpy(g["query"]).to(DEV).to(dt)
    v = torch.from_numpy(g["value"]).to(DEV).to(dt)
    mask = None if g["mask"] is None else torch.from_numpy(g["mask"]).to(DEV)
    impl = vab.SunShapeAttentionBackend().make_impl(layer_idx=7)
    out = impl.forward(q, golden_keys(g), v, attn_mask=mask, scale=g["scale"])
    tol = TOL_F32 if g["dtype"] == "f32" else TOL_BF16
    assert out.dtype == dt
    assert_close_rowwise(out.float().cpu().numpy(), g["ref_out"], tol, f"{name} forward")


def _check_bundle_layers(z):
    for layer in z["layers"]:
        pre = f"l{layer}_"
        dt = torch_dtype(str(z[pre + "dtype"]))
        keys = torch.from_numpy(z[pre + "keys"]).to(DEV).to(dt)
        qk = vab.quantize_key_states(int(layer), keys)
        codec = vab.get_registered_runtime().codec_for_layer(int(layer))
        assert codec.n_codebooks == 1
        idx = qk.indices.cpu().numpy()
        ref_idx = z[pre + "ref_indices"]
        mism = int((idx != ref_idx).sum())
        assert mism <= max(1, ref_idx.size // 100000), f"layer {layer}: {mism} index mismatches"
        q = torch.from_numpy(z[pre + "query"]).to(DEV).to(dt)
        v = torch.from_numpy(z[pre + "value"]).to(DEV).to(dt)
        impl = vab.SunShapeAttentionImpl(layer_idx=int(layer))
        out = impl.forward(q, qk, v, scale=float(z[pre + "scale"]))
        assert_close_rowwise(out.float().cpu().numpy(), z[pre + "ref_out"], TOL_BF16, f"bundle layer {layer}")


def test_reference_bundle_decodes_like_the_reference(registry):
    z = np.load(os.path.join(GOLDEN_DIR, "g7_bundle.npz"))
    bundle = SunShapeBundle.load(BUNDLE, device=torch.device(DEV))
    vab.register_runtime_state(runtime_state_from_bundle(bundle, bundle_path=BUNDLE))
    _check_bundle_layers(z)


def test_install_hooks_from_reference_bundle_file(registry):
    z = np.load(os.path.join(GOLDEN_DIR, "g7_bundle.npz"))
    handle = vab.install_sunshape_hooks(bundle_path=BUNDLE, model_name="synthetic-ref", mode="sunshape_base",
                                        bits_per_dim=1.0, block_dim=8, layers=[3, 5])
    assert vab.get_registered_handle() is handle and vab.get_mode() == vab.MODE_ACTIVE
    assert vab.describe_backend()["runtime"]["layers"] == [3, 5]
    _check_bundle_layers(z)
    handle.deactivate()
    assert vab.get_registered_runtime() is None and vab.get_mode() == vab.MODE_OFF


def test_cache_update_matches_reference_cache():
    from sunshape_b200.cache import SunShapeCache

    z = np.load(os.path.join(GOLDEN_DIR, "g8_cache.npz"))
    keys = torch.from_numpy(z["keys"]).to(DEV).to(torch.bfloat16)
    vals = torch.from_numpy(z["value"]).to(DEV).to(torch.bfloat16)
    D = keys.shape[-1]
    codec = make_codec(z["perm"], z["centroids"], np.zeros(D // 8, bool), D, 8, 256, DEV)
    assert codec.n_codebooks == 1
    cache = SunShapeCache.from_codecs({1: codec}, num_layers=2)
    for i, (a, b) in enumerate(z["steps"]):
        for layer in (0, 1):
            k_out, v_out = cache.update(keys[:, :, a:b], vals[:, :, a:b], layer)
            assert k_out.dtype == torch.bfloat16
            np.testing.assert_array_equal(v_out.float().cpu().numpy(), z[f"step{i}_l{layer}_values"])
            ours = k_out.float().cpu().numpy()
            ref = z[f"step{i}_l{layer}_keys"]
            if layer == 0:
                np.testing.assert_array_equal(ours, ref)
                continue
            # block-wise in the permuted basis: every block equals the reference's codeword, or the two
            # codewords are exact-distance ties
            perm = z["perm"]
            xp = z["keys"][:, :, :b][..., perm].astype(np.float64)
            op, rp = ours[..., perm].astype(np.float64), ref[..., perm].astype(np.float64)
            shp = (*op.shape[:3], -1, 8)
            xb, ob, rb_ = xp.reshape(shp), op.reshape(shp), rp.reshape(shp)
            for bb, h, t, blk in np.argwhere((ob != rb_).any(-1)):
                x = xb[bb, h, t, blk]
                d1, d2 = ((x - ob[bb, h, t, blk]) ** 2).sum(), ((x - rb_[bb, h, t, blk]) ** 2).sum()
                assert abs(d1 - d2) <= 1e-5 * ((x ** 2).sum() + d1), (bb, h, t, blk, d1, d2)
    assert cache.get_seq_length(1) == int(z["steps"][-1][1])
