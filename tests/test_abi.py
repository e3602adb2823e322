"""The C-ABI library loads, exports every declared entry point and validates arguments on the host (no GPU)."""
import ctypes
import os
import re

import pytest

from sunshape_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "sunshape_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sunshape_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_python_binding_symbols():
    assert declared_functions() == sorted(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load_library()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.sunshape_abi_version() == 1


def test_struct_layouts_match_header():
    # pointer fields then int32 fields; the header order is mirrored by the ctypes structs
    assert ctypes.sizeof(_lib.CodecDesc) == 3 * 8 + 5 * 4 + 4 + 8  # padded to 8
    assert ctypes.sizeof(_lib.KVDesc) == 8 + 4 + 4 + 8 + 4 + 4 + 8 + 4 + 4 + 4 + 4 + 8


def _expect(rc, code, text):
    lib = _lib.load_library()
    assert rc == code
    assert text in lib.sunshape_last_error().decode()


def test_invalid_arguments_are_rejected_before_any_launch():
    lib = _lib.load_library()
    _expect(lib.sunshape_encode(None, None, 0, 1, 1, 1, 0, 0, None, 3, None, 1, 1, None), -1, "codec descriptor")
    cd = _lib.CodecDesc(16, 16, None, 1, 64, 7, 256, 0, None)       # head_dim not divisible by block_dim
    _expect(lib.sunshape_encode(ctypes.byref(cd), 16, 0, 1, 1, 1, 0, 0, 16, 3, None, 1, 1, None), -1,
            "divisible by block_dim")
    cd = _lib.CodecDesc(16, 16, None, 1, 64, 8, 300, 0, None)       # uint8 too narrow for 300 codewords
    _expect(lib.sunshape_encode(ctypes.byref(cd), 16, 0, 1, 1, 1, 0, 0, 16, 3, None, 1, 1, None), -1,
            "too narrow")
    cd = _lib.CodecDesc(16, 16, None, 1, 64, 8, 256, 0, None)
    kd = _lib.KVDesc(16, 3, None, 1, 16, 1, 64, 10, 10)
    # query heads not divisible by kv heads
    _expect(lib.sunshape_decode_attention(ctypes.byref(cd), ctypes.byref(kd), 16, 1, 1, 6, 4, 1, None, 0, 0, 0, 0,
                                          float("nan"), 16, 1, None, 16, 1 << 20, None), -1, "divisible by kv-head")
    # more than 64 blocks is outside the fused LUT kernel
    cd2 = _lib.CodecDesc(16, 16, None, 1, 256, 2, 256, 0, None)
    _expect(lib.sunshape_decode_attention(ctypes.byref(cd2), ctypes.byref(kd), 16, 1, 1, 4, 4, 1, None, 0, 0, 0, 0,
                                          float("nan"), 16, 1, None, 16, 1 << 20, None), -2, "n_blocks > 64")
    # misaligned value buffer
    kd_bad = _lib.KVDesc(16, 3, None, 1, 24, 1, 64, 10, 10)
    _expect(lib.sunshape_decode_attention(ctypes.byref(cd), ctypes.byref(kd_bad), 16, 1, 1, 4, 4, 1, None, 0, 0, 0,
                                          0, float("nan"), 16, 1, None, 16, 1 << 20, None), -1, "16-byte aligned")
    _expect(lib.sunshape_merge_partials(None, 1, 1, 64, None, 1, None), -1, "NULL")


def test_cpu_tensors_raise_no_fallback():
    import torch

    from tests.helpers import make_codec

    codec = make_codec(torch.arange(64), torch.zeros(1, 8, 256, 8), torch.zeros(8, dtype=torch.bool), 64, 8, 256,
                       "cpu")
    with pytest.raises(RuntimeError, match="CUDA"):
        codec.quantize(torch.randn(10, 64))


def test_per_head_codec_requires_kv_head():
    """The reference signatures carry no KV head; on a codec with one codebook per KV head they must
    raise instead of silently using codebook 0 for every head."""
    import torch

    from sunshape_b200.kernels import sunshape_attention_scores
    from tests.helpers import make_codec

    codec = make_codec(torch.arange(64), torch.zeros(2, 8, 256, 8), torch.zeros(8, dtype=torch.bool), 64, 8, 256,
                       "cpu")
    with pytest.raises(RuntimeError, match="kv_head"):
        codec.quantize(torch.randn(10, 64))
    with pytest.raises(RuntimeError, match="kv_head"):
        codec.dequantize(None)
    with pytest.raises(RuntimeError, match="out of range"):
        codec.quantize(torch.randn(10, 64), kv_head=2)

    class _QK:
        indices = torch.zeros(10, 8, dtype=torch.uint8)

    with pytest.raises(RuntimeError, match="kv_head|CUDA"):
        sunshape_attention_scores(codec, torch.randn(4, 64), _QK())
