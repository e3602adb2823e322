"""Host-side logic of the drop-in layer: mask strides, KV layouts, shards, bundle format (no GPU)."""
import torch

from sunshape_b200 import vllm_attn_backend as vab
from sunshape_b200.distributed import kv_shard_bounds
from sunshape_b200.hf import SunShapeBundle, SunShapeConfig, default_block_dim, resolve_mode_alias
from sunshape_b200.workloads import CONFIGS


def test_mask_view_follows_reference_slicing():
    B, Hq, L, T = 2, 8, 1, 33
    m4 = torch.randn(B, Hq, L, T)
    t, s = vab._mask_view(m4, B, Hq, L, T)
    assert s == (Hq * L * T, L * T, 0)
    m3b = torch.randn(B, L, T)                  # leading dim == batch: per-batch mask
    assert vab._mask_view(m3b, B, Hq, L, T)[1] == (L * T, 0, 0)
    m3h = torch.randn(Hq, L, T)                 # per query head
    assert vab._mask_view(m3h, B, Hq, L, T)[1] == (0, L * T, 0)
    m2 = torch.randn(L, T)
    assert vab._mask_view(m2, B, Hq, L, T)[1] == (0, 0, 0)
    mb = torch.zeros(L, T, dtype=torch.bool)
    assert vab._mask_view(mb, B, Hq, L, T)[0].dtype == torch.float32   # bool adds as 0/1 like the reference


def test_kv_layout_shares_head_stride_of_cache_views():
    B, H, Tcap, T, D, nb = 2, 3, 50, 40, 64, 8
    v = torch.zeros(B, H, Tcap, D)[:, :, :T]
    i = torch.zeros(B, H, Tcap, nb, dtype=torch.uint8)[:, :, :T]
    v2, i2, h2, hs = vab._kv_layout(v, i, None, B, H, T)
    assert hs == Tcap and v2.data_ptr() == v.data_ptr() and i2.data_ptr() == i.data_ptr()
    i_c = torch.zeros(B, H, T, nb, dtype=torch.uint8)                    # disagreeing layout -> copies
    v3, i3, _, hs3 = vab._kv_layout(v, i_c, None, B, H, T)
    assert hs3 == T and v3.is_contiguous()


def test_kv_shard_bounds_cover_sequence():
    for T in (1, 7, 131072, 131075):
        for w in (1, 2, 4, 8):
            spans = [kv_shard_bounds(T, w, r) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == T
            assert all(a[1] == b[0] for a, b in zip(spans[:-1], spans[1:]))
            assert max(e - s for s, e in spans) - min(e - s for s, e in spans) <= 1


def test_config_and_aliases():
    assert resolve_mode_alias("sunshape_mixed") == "profileperm_mixed_precision"
    assert default_block_dim(1.0) == 8 and default_block_dim(2.0) == 2
    assert SunShapeConfig(bits_per_dim=1.0).resolved_block_dim == 8


def test_bundle_roundtrip_keeps_reference_format(tmp_path):
    from tests.helpers import make_codec

    perm = torch.randperm(64)
    c = make_codec(perm, torch.randn(8, 256, 8), torch.zeros(8, dtype=torch.bool), 64, 8, 256, "cpu")
    b = SunShapeBundle(model_name="m", layers=[3], bits_per_dim=1.0, block_dim=8, mode="profileperm_baseline",
                       cal_points=16, dsq_steps=0, seed=1, codecs={3: c}, trace_meta={"x": 1})
    sd = b.state_dict()
    assert sd["format_version"] == 1 and set(sd["codecs"]["3"]["state_dict"]) >= {
        "E", "E_inv", "centroids", "permutation", "inv_permutation", "mixed_high_precision_blocks", "rotation"}
    p = b.save(tmp_path / "b.pt")
    b2 = SunShapeBundle.load(p, device=torch.device("cpu"))
    assert torch.equal(b2.codecs[3].centroids, c.centroids) and torch.equal(b2.codecs[3].permutation, perm)


def test_config_byte_model():
    assert CONFIGS["c2"].bytes_per_kv_token() == 272
    assert CONFIGS["c3"].bytes_per_kv_token() == 288
    assert CONFIGS["c4"].bytes_per_kv_token() == 16 + 64 + 256
    assert CONFIGS["c5"].kv_tokens() == 8 * 8 * 131072
