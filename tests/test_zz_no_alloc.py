"""sunshape_decode_attention_noalloc: decode attention for callers that cannot allocate device memory.

Such callers (plugin hosts whose GPU memory belongs to another allocator, engines that reserve all
device memory up front, bindings without a CUDA allocator) cannot hand the library a workspace.
The no-allocation entry point keeps its scratch in an array built into the library.  This test
calls it through the C ABI twice in a row (the array keeps the previous call's contents, so the
second call checks that what must start at zero is cleared) and compares each result with the
regular entry point's, within the bf16 tolerance the other parity tests use.  It lives in its own
file, collected last, and needs nothing from the other tests.
"""
import ctypes
import math

import pytest
import torch

from sunshape_b200 import _lib
from sunshape_b200 import vllm_attn_backend as vab
from sunshape_b200.workloads import CONFIGS, make_case
from tests.helpers import TOL_BF16, assert_close_rowwise, make_codec

pytestmark = pytest.mark.gpu


def _call_noalloc(codec, keys, query, value, scale):
    lib = _lib.load_library()
    desc, keep, _ = codec.kernel_desc()
    B, Hq, L, _ = query.shape
    _, Hkv, T, Dv = value.shape
    kd = _lib.kv_desc(keys.indices, keys.heavy, value, T, T, Dv)
    out = torch.empty(B, Hq, L, Dv, device=query.device, dtype=value.dtype)
    with torch.cuda.device(query.device):
        rc = lib.sunshape_decode_attention_noalloc(
            ctypes.byref(desc), ctypes.byref(kd), query.data_ptr(), _lib.dtype_code(query), B, Hq, Hkv, L, None,
            _lib.F32, 0, 0, 0, math.nan if scale is None else float(scale), out.data_ptr(), _lib.dtype_code(out),
            None, _lib.stream_ptr(query.device))
    return rc, out


def _error_word():
    code = ctypes.c_int32(-1)
    rc = _lib.load_library().sunshape_decode_attention_noalloc_error(ctypes.byref(code))
    assert rc == 0, _lib.load_library().sunshape_last_error().decode()
    return code.value


@pytest.mark.parametrize("shape", ["c2_ragged", "c5_headline_heads"])
def test_noalloc_matches_regular_entry_point_twice(shape):
    dev = torch.device("cuda", 0)
    # several CTAs share each KV head, so the per-head tickets in the scratch are exercised;
    # the second shape has the headline config's 64 KV heads of 8 query rows (fp16 LUT entries),
    # whose per-head LUT area does not fit the built-in array, so each CTA builds its LUTs
    if shape == "c2_ragged":
        cfg = CONFIGS["c2"].with_(batch=2, kv_heads=2, q_heads=8, seq_len=20000 + 11)
    else:
        cfg = CONFIGS["c5"].with_(batch=8, kv_heads=8, q_heads=64, seq_len=2048 + 5)
    case = make_case(cfg, device=dev, seed=21)
    codec = make_codec(case["perm"], case["centroids"], case["heavy_mask"], cfg.head_dim, cfg.block_dim,
                       cfg.n_centroids, dev)
    keys = vab.quantize_codec_keys(codec, case["keys"])
    ref = vab._apply_quantized_attention(codec=codec, query=case["query"], key=keys, value=case["value"],
                                         attn_mask=None, scale=case["scale"])
    for call in range(2):
        rc, out = _call_noalloc(codec, keys, case["query"], case["value"], case["scale"])
        torch.cuda.synchronize()
        assert rc == 0, _lib.load_library().sunshape_last_error().decode()
        assert _error_word() == 0
        assert_close_rowwise(out.float().cpu().numpy(), ref.float().cpu().numpy(), TOL_BF16, f"noalloc call {call}")


def test_noalloc_rejects_workspace_beyond_builtin_scratch():
    dev = torch.device("cuda", 0)
    cfg = CONFIGS["c2"].with_(batch=1, kv_heads=1, q_heads=16, seq_len=64)
    case = make_case(cfg, device=dev, seed=3)
    codec = make_codec(case["perm"], case["centroids"], case["heavy_mask"], cfg.head_dim, cfg.block_dim,
                       cfg.n_centroids, dev)
    keys = vab.quantize_codec_keys(codec, case["keys"])
    lib = _lib.load_library()
    desc, keep, _ = codec.kernel_desc()
    value = case["value"]
    # pretend 200000 sequences share these buffers: only the size check runs, nothing launches
    kd = _lib.kv_desc(keys.indices, None, value, 64, 64, 128)
    with torch.cuda.device(dev):
        rc = lib.sunshape_decode_attention_noalloc(
            ctypes.byref(desc), ctypes.byref(kd), case["query"].data_ptr(), _lib.BF16, 200000, 16, 1, 1, None,
            _lib.F32, 0, 0, 0, math.nan, value.data_ptr(), _lib.BF16, None, _lib.stream_ptr(dev))
    assert rc == -4
    assert "built-in array" in lib.sunshape_last_error().decode()
    # an empty batch is accepted without touching the device, as by the regular entry point
    with torch.cuda.device(dev):
        rc = lib.sunshape_decode_attention_noalloc(
            ctypes.byref(desc), ctypes.byref(kd), case["query"].data_ptr(), _lib.BF16, 0, 16, 1, 1, None,
            _lib.F32, 0, 0, 0, math.nan, value.data_ptr(), _lib.BF16, None, _lib.stream_ptr(dev))
    assert rc == 0
