"""Bit-packed (1, 2, 4 bits per block) and int16 codeword indices on the GPU, against the oracle.

The packed layout is the reference's packed-index format (triton_kernels.py:213-292): block b of a
row sits in byte b // (8 // bits) at bit offset (b % (8 // bits)) * bits.  Codebooks above 256
codewords store int16 indices (codec.py:78-83)."""
import numpy as np
import pytest
import torch

from oracle import sunshape_oracle as O
from sunshape_b200 import vllm_attn_backend as vab
from sunshape_b200.kernels import pack_indices, sunshape_attention_scores, sunshape_attention_scores_packed
from sunshape_b200.workloads import CONFIGS, make_case
from tests.helpers import TOL_F32, assert_close_rowwise, make_codec

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _unpack(packed: np.ndarray, nb: int, bits: int) -> np.ndarray:
    per = 8 // bits
    b = np.arange(nb)
    return (packed[..., b // per] >> ((b % per) * bits)) & ((1 << bits) - 1)


@pytest.mark.parametrize("bits,block_dim", [(4, 4), (2, 2), (1, 8), (4, 8)])
def test_packed_scores_match_oracle(bits, block_dim):
    C = 1 << bits
    cfg = CONFIGS["c2"].with_(batch=1, kv_heads=2, q_heads=8, seq_len=3001, block_dim=block_dim, n_centroids=C)
    case = make_case(cfg, device=DEV, seed=31)
    codec = make_codec(case["perm"], case["centroids"], case["heavy_mask"], cfg.head_dim, block_dim, C, DEV)
    qk = vab.quantize_codec_keys(codec, case["keys"])
    idx = qk.indices                                                  # [1, 2, T, nb] uint8
    packed = pack_indices(idx, bits)
    assert packed.shape[-1] == (cfg.n_blocks * bits + 7) // 8
    np.testing.assert_array_equal(_unpack(packed.cpu().numpy(), cfg.n_blocks, bits), idx.cpu().numpy())
    G = cfg.group
    for h in range(cfg.kv_heads):
        q = case["query"][0, h * G:(h + 1) * G, 0].float()
        s = sunshape_attention_scores_packed(codec, q, packed[0, h], bits, kv_head=h)
        ref = O.lut_scores(q.cpu().numpy(), idx[0, h].cpu().numpy(), case["centroids"][h].cpu().numpy(),
                           case["perm"].cpu().numpy())
        assert_close_rowwise(s.cpu().numpy(), ref, TOL_F32, f"packed bits {bits} head {h}")


def test_int16_indices_above_256_codewords():
    cfg = CONFIGS["c2"].with_(batch=1, kv_heads=1, q_heads=4, seq_len=2000, n_centroids=512)
    case = make_case(cfg, device=DEV, seed=37)
    codec = make_codec(case["perm"], case["centroids"], case["heavy_mask"], cfg.head_dim, cfg.block_dim, 512, DEV)
    qk = vab.quantize_codec_keys(codec, case["keys"])
    assert qk.indices.dtype == torch.int16
    idx = qk.indices[0, 0]
    kp = case["keys"][0, 0].cpu().numpy()
    ref_idx, _ = O.quantize(kp, case["perm"].cpu().numpy(), case["centroids"][0].cpu().numpy())
    n_mis, n_bad = O.index_mismatches_are_ties(kp[:, case["perm"].cpu().numpy()], case["centroids"][0].cpu().numpy(),
                                               idx.cpu().numpy(), ref_idx)
    assert n_bad == 0, (n_mis, n_bad)
    q = case["query"][0, :, 0].float()
    s = sunshape_attention_scores(codec, q, qk.head(0, 0), kv_head=0)
    ref = O.lut_scores(q.cpu().numpy(), idx.cpu().numpy().astype(np.int64), case["centroids"][0].cpu().numpy(),
                       case["perm"].cpu().numpy())
    assert_close_rowwise(s.cpu().numpy(), ref, TOL_F32, "int16 scores")
