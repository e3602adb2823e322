"""Tensor-core (tcgen05) key encode: parity with the reference's indices and with the CUDA-core kernel.

fp32 and 16-bit keys with block_dim 2, 4 or 8 and n_centroids a multiple of 64 (<= 256) take the
tensor-core kernel;
``SUNSHAPE_ENCODE=cuda_cores`` forces the CUDA-core kernel and ``SUNSHAPE_ENCODE=tensor_cores``
makes an unsupported shape an error, so these tests know which kernel ran.  Indices must agree
exactly except where two codewords are at the same distance within fp32 rounding (the rule of
``index_mismatches_are_ties``, the one the fp32 reference itself needs).
"""
import os
from contextlib import contextmanager

import numpy as np
import pytest
import torch

from oracle import sunshape_oracle as O
from sunshape_b200 import vllm_attn_backend as vab
from sunshape_b200.workloads import CONFIGS, make_case
from tests.helpers import GOLDEN_CASES, load_golden, make_codec, tie_space

pytestmark = pytest.mark.gpu
DEV = "cuda"


@contextmanager
def encode_path(path):
    old = os.environ.get("SUNSHAPE_ENCODE")
    os.environ["SUNSHAPE_ENCODE"] = path
    try:
        yield
    finally:
        if old is None:
            del os.environ["SUNSHAPE_ENCODE"]
        else:
            os.environ["SUNSHAPE_ENCODE"] = old


def _check_ties(keys, perm, centroids, heavy_mask, idx_a, idx_b, what, E=None):
    B, H = idx_a.shape[:2]
    for b in range(B):
        for h in range(H):
            kp, cents = tie_space(keys[b, h][:, perm], centroids[h % centroids.shape[0]], E)
            n_mis, n_bad = O.index_mismatches_are_ties(kp, cents, idx_a[b, h], idx_b[b, h], heavy_mask)
            assert n_bad == 0, f"{what} (b={b}, h={h}): {n_mis} mismatches, {n_bad} not ties"


@pytest.mark.parametrize("name", [n for n in GOLDEN_CASES if load_golden(n)["dtype"] == "bf16"
                                  and load_golden(n)["block_dim"] == 8])
def test_tensor_core_encode_matches_oracle_on_golden_keys(name):
    """The golden keys rounded to bf16 (the dtype a model hands the encoder); the oracle, pinned by
    the same fixtures, gives the expected indices for those keys."""
    g = load_golden(name)
    codec = make_codec(g["perm"], g["centroids"], g["heavy_mask"], g["D"], g["block_dim"], g["n_centroids"], DEV,
                       E=g["E"])
    keys = torch.from_numpy(g["keys"]).to(DEV).to(torch.bfloat16)
    kb = keys.float().cpu().numpy()
    with encode_path("tensor_cores"):
        qk = vab.quantize_codec_keys(codec, keys)
    torch.cuda.synchronize()
    hm = g["heavy_mask"]
    ref = np.empty(qk.indices.shape, dtype=np.int64)
    for b in range(g["B"]):
        for h in range(g["Hkv"]):
            ref[b, h], pt = O.quantize(kb[b, h], g["perm"], g["centroids"][h], hm, E=g["E"])
            if hm.any():
                np.testing.assert_array_equal(qk.heavy[b, h].float().cpu().numpy(), pt[:, hm.astype(bool)])
    _check_ties(kb, g["perm"], g["centroids"], hm, qk.indices.cpu().numpy(), ref, name, E=g["E"])


@pytest.mark.parametrize("cfg_name,dtype,seq_len,n_centroids,batch", [
    ("c2", torch.bfloat16, 1000 + 37, 256, 1),    # ragged tail tile
    ("c3", torch.bfloat16, 4096, 256, 1),         # block_dim 4
    ("c4", torch.bfloat16, 777, 256, 1),          # SunShape-Mixed heavy blocks
    ("c5", torch.float16, 300, 64, 1),            # f16 keys, 64 codewords
    ("c2", torch.bfloat16, 1, 64, 1),             # one key
    ("c2b2", torch.bfloat16, 515, 64, 1),         # block_dim 2
    ("c2", torch.float32, 1000 + 37, 256, 1),     # fp32 keys (3xTF32), ragged tail
    ("c3", torch.float32, 3000, 256, 2),          # fp32, block_dim 4, 16 heads of per-KV-head codebooks
    ("c4", torch.float32, 700, 256, 1),           # fp32 SunShape-Mixed
    ("c2b2", torch.float32, 333, 128, 1),         # fp32, block_dim 2, 128 codewords
    ("c5", torch.float32, 2, 256, 1),             # fp32, two keys per head
])
def test_tensor_core_encode_matches_cuda_core_kernel(cfg_name, dtype, seq_len, n_centroids, batch):
    base = CONFIGS[cfg_name[:2]].with_(block_dim=2) if cfg_name == "c2b2" else CONFIGS[cfg_name]
    cfg = base.with_(batch=batch, seq_len=seq_len, n_centroids=n_centroids)
    case = make_case(cfg, device=DEV, seed=5)
    codec = make_codec(case["perm"], case["centroids"], case["heavy_mask"], cfg.head_dim, cfg.block_dim,
                       cfg.n_centroids, DEV)
    keys = case["keys"].to(dtype)
    with encode_path("tensor_cores"):
        tc = vab.quantize_codec_keys(codec, keys)
    with encode_path("cuda_cores"):
        cc = vab.quantize_codec_keys(codec, keys)
    torch.cuda.synchronize()
    kf = keys.float().cpu().numpy()
    cents = case["centroids"].cpu().numpy() if torch.is_tensor(case["centroids"]) else case["centroids"]
    perm = case["perm"].cpu().numpy() if torch.is_tensor(case["perm"]) else case["perm"]
    hm = case["heavy_mask"].cpu().numpy() if torch.is_tensor(case["heavy_mask"]) else case["heavy_mask"]
    _check_ties(kf, perm, cents, hm, tc.indices.cpu().numpy(), cc.indices.cpu().numpy(), cfg_name)
    agree = (tc.indices == cc.indices).float().mean().item()
    assert agree > 0.999, f"only {agree:.5f} of indices agree"
    if tc.heavy is not None:
        assert torch.equal(tc.heavy, cc.heavy)
    from sunshape_b200 import _lib
    assert _lib.encode_error_word(torch.device(DEV)) == 0


def test_tensor_core_encode_rejects_unsupported_shape_when_forced():
    cfg = CONFIGS["c2"].with_(batch=1, seq_len=64, n_centroids=48)
    case = make_case(cfg, device=DEV, seed=1)
    codec = make_codec(case["perm"], case["centroids"], case["heavy_mask"], cfg.head_dim, cfg.block_dim,
                       cfg.n_centroids, DEV)
    with encode_path("tensor_cores"), pytest.raises(RuntimeError, match="tensor_cores"):
        vab.quantize_codec_keys(codec, case["keys"].float())
