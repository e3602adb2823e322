"""HF cache classes (reference ``sunshape/cache.py``): host-side plumbing on CPU.

The quantize -> dequantize step itself runs on the GPU (covered by the encode and dequantize
parity tests); here it is replaced by a marker function so the tests check what the cache does
around it: which layers route keys through the codec, with which shapes and dtypes, that values
are untouched and that sequences concatenate like ``DynamicLayer``.  Without the replacement, CPU
keys must raise (there is no CPU fallback).
"""
import pytest
import torch

from sunshape_b200 import cache as cache_mod
from sunshape_b200.cache import IdentityLayer, SunShapeCache, SunShapeLayer
from sunshape_b200.codec import SunShapeBlockCodec
from sunshape_b200.hf import SunShapeBundle
from sunshape_b200.turbo_cache import TurboQuantCache, TurboQuantLayer


def _codec():
    return SunShapeBlockCodec(64, 8, 16, device=torch.device("cpu"))


@pytest.fixture
def marked(monkeypatch):
    seen = []

    def fake_quantize_keys(codec, key_states):
        seen.append((codec, tuple(key_states.shape), key_states.dtype))
        return key_states * 2

    monkeypatch.setattr(cache_mod, "fake_quantize_keys", fake_quantize_keys)
    return seen


def test_codec_layers_quantize_keys_and_concatenate(marked):
    codec = _codec()
    cache = SunShapeCache(num_layers=3, layer_codecs={0: codec}, identity_layers={2})
    assert [type(layer) for layer in cache.layers] == [SunShapeLayer, cache_mod.DynamicLayer, IdentityLayer]
    k = torch.randn(2, 2, 5, 64, dtype=torch.bfloat16)
    v = torch.randn(2, 2, 5, 64, dtype=torch.bfloat16)
    k0, v0 = cache.update(k, v, 0)
    assert torch.equal(k0, k * 2) and torch.equal(v0, v)
    k0, v0 = cache.update(k[:, :, :1], v[:, :, :1], 0)      # one decode step appends
    assert k0.shape == (2, 2, 6, 64) and torch.equal(k0[:, :, 5:], k[:, :, :1] * 2)
    assert cache.get_seq_length(0) == 6
    assert marked == [(codec, (2, 2, 5, 64), torch.bfloat16), (codec, (2, 2, 1, 64), torch.bfloat16)]
    for layer_idx in (1, 2):                                 # plain and identity layers store keys as given
        kk, vv = cache.update(k, v, layer_idx)
        assert torch.equal(kk, k) and torch.equal(vv, v)
    assert len(marked) == 2


def test_bundle_cache_uses_bundle_codecs(marked):
    codecs = {1: _codec(), 3: _codec()}
    bundle = SunShapeBundle(model_name="m", layers=[1, 3], bits_per_dim=1.0, block_dim=8,
                            mode="profileperm_baseline", cal_points=16, dsq_steps=3, seed=0, codecs=codecs)
    cache = bundle.make_cache(num_layers=4)
    assert [isinstance(layer, SunShapeLayer) for layer in cache.layers] == [False, True, False, True]
    assert cache.layers[3].codec is codecs[3]


def test_cpu_keys_have_no_fallback():
    layer = SunShapeLayer(codec=_codec())
    with pytest.raises(RuntimeError):
        layer.update(torch.randn(1, 1, 3, 64), torch.randn(1, 1, 3, 64))


def test_turbo_cache_routes_flattened_fp32_keys_through_quantizer():
    seen = []

    def quantizer(flat):
        seen.append((tuple(flat.shape), flat.dtype))
        return -flat

    cache = TurboQuantCache.from_quantizers({1: quantizer}, num_layers=2)
    assert [type(layer) for layer in cache.layers] == [cache_mod.DynamicLayer, TurboQuantLayer]
    k = torch.randn(1, 2, 3, 64, dtype=torch.bfloat16)
    v = torch.randn(1, 2, 3, 64, dtype=torch.bfloat16)
    k1, v1 = cache.update(k, v, 1)
    assert seen == [((6, 64), torch.float32)]
    assert k1.dtype == torch.bfloat16 and torch.equal(k1, -k) and torch.equal(v1, v)
    assert cache.get_seq_length(1) == 3 and not cache.has_previous_state()   # layer 0 decides, as in the reference
    with pytest.raises(NotImplementedError):
        TurboQuantCache.for_layers(head_dims={0: 64}, layers=[0], num_layers=1, mode="turboquant_prod")
    built = TurboQuantCache.for_layers(head_dims={0: 64}, layers=[0], num_layers=1, device=torch.device("cpu"))
    assert isinstance(built.layers[0], TurboQuantLayer) and built.layers[0].quantizer.bits == 3
    with pytest.raises(ValueError):
        TurboQuantCache(num_layers=None)


def test_reference_names_without_calibration_raise_with_reason():
    from sunshape_b200.kernels import require_fast_path, require_triton_fast_path

    assert require_triton_fast_path is require_fast_path
    with pytest.raises(NotImplementedError, match="offline calibration"):
        SunShapeCache.from_traces({}, [0], num_layers=1)


def test_compressed_cache_builds_and_registers_attention():
    import torch
    from transformers import AttentionInterface

    from sunshape_b200.compressed_cache import ATTN_IMPLEMENTATION, SunShapeCompressedCache, SunShapeCompressedLayer
    from tests.helpers import make_codec

    codec = make_codec(torch.arange(64), torch.zeros(8, 256, 8), torch.zeros(8, dtype=torch.bool), 64, 8, 256, "cpu")
    cache = SunShapeCompressedCache.from_codecs({1: codec}, num_layers=3)
    assert isinstance(cache.layers[1], SunShapeCompressedLayer)
    assert not isinstance(cache.layers[0], SunShapeCompressedLayer)
    assert cache.get_seq_length(1) == 0
    assert ATTN_IMPLEMENTATION in AttentionInterface._global_mapping
