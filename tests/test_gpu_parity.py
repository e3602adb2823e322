"""Parity of the CUDA path (through the C ABI) with the reference's recorded outputs and the CPU oracle."""
import numpy as np
import pytest
import torch

from oracle import sunshape_oracle as O
from sunshape_b200 import vllm_attn_backend as vab
from sunshape_b200.kernels import _torch_attention_scores, sunshape_attention_scores
from sunshape_b200.workloads import CONFIGS, make_case
from tests.helpers import GOLDEN_CASES, TOL_BF16, TOL_F32, assert_close_rowwise, load_golden, make_codec, tie_space, torch_dtype

pytestmark = pytest.mark.gpu
DEV = "cuda"


def golden_codec(g):
    return make_codec(g["perm"], g["centroids"], g["heavy_mask"], g["D"], g["block_dim"], g["n_centroids"], DEV,
                      E=g["E"])


def golden_keys(g):
    """Packed payload from the reference's own indices / passthrough values."""
    hm = g["heavy_mask"]
    idx = torch.from_numpy(g["ref_indices"]).to(DEV)
    heavy = None
    if hm.any():
        hv = g["ref_passthrough"][:, :, :, hm.astype(bool)]
        heavy = torch.from_numpy(np.ascontiguousarray(hv)).to(DEV).to(torch_dtype(g["dtype"]) if g["dtype"] == "bf16"
                                                                       else torch.float32)
    return vab.SunShapeQuantizedKeys(quantized_heads=(), batch_size=g["B"], num_kv_heads=g["Hkv"], seq_len=g["T"],
                                     indices=idx, heavy=heavy,
                                     passthrough_blocks=torch.from_numpy(hm).to(DEV) if hm.any() else None,
                                     head_dim=g["D"], block_dim=g["block_dim"])


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_encode_matches_reference_indices(name):
    g = load_golden(name)
    codec = golden_codec(g)
    keys = torch.from_numpy(g["keys"]).to(DEV)
    qk = vab.quantize_codec_keys(codec, keys)
    idx = qk.indices.cpu().numpy()
    hm = g["heavy_mask"]
    for b in range(g["B"]):
        for h in range(g["Hkv"]):
            kp, cents = tie_space(g["keys"][b, h][:, g["perm"]], g["centroids"][h], g["E"])
            n_mis, n_bad = O.index_mismatches_are_ties(kp, cents, idx[b, h], g["ref_indices"][b, h], hm)
            assert n_bad == 0, f"{name}: {n_mis} index mismatches, {n_bad} not exact-distance ties"
    if hm.any():
        ref_h = g["ref_passthrough"][:, :, :, hm.astype(bool)]
        np.testing.assert_array_equal(qk.heavy.float().cpu().numpy(), ref_h)


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_decode_matches_reference_output(name):
    g = load_golden(name)
    codec = golden_codec(g)
    dt = torch_dtype(g["dtype"])
    q = torch.from_numpy(g["query"]).to(DEV).to(dt)
    v = torch.from_numpy(g["value"]).to(DEV).to(dt)
    mask = None if g["mask"] is None else torch.from_numpy(g["mask"]).to(DEV)
    out = vab._apply_quantized_attention(codec=codec, query=q, key=golden_keys(g), value=v, attn_mask=mask,
                                         scale=g["scale"])
    torch.cuda.synchronize()
    assert out.dtype == dt and out.shape == (g["B"], g["Hq"], g["L"], g["D"])
    tol = TOL_F32 if g["dtype"] == "f32" else TOL_BF16
    assert_close_rowwise(out.float().cpu().numpy(), g["ref_out"], tol, f"{name} decode")


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_scores_match_reference(name):
    g = load_golden(name)
    codec = golden_codec(g)
    dt = torch_dtype(g["dtype"])
    G = g["Hq"] // g["Hkv"]
    keys = golden_keys(g)
    for b in range(g["B"]):
        for h in range(g["Hkv"]):
            q = torch.from_numpy(g["query"][b, h * G:(h + 1) * G]).to(DEV).to(dt)
            if g["scale"] is not None:
                q = q * float(g["scale"])
            qh, kh = q.reshape(-1, g["D"]), keys.head(b, h)
            ref = g["ref_scores"][b, h]
            s = sunshape_attention_scores(codec, qh, kh, kv_head=h)
            assert_close_rowwise(s.cpu().numpy(), ref, TOL_F32, f"{name} scores b{b}h{h}")
            # the codec method (codec.py:403-422) upcasts the query to fp32 first, as the reference does
            s2 = codec.attention_scores(qh, kh, kv_head=h)
            assert_close_rowwise(s2.cpu().numpy(), ref, TOL_F32, f"{name} codec.attention_scores b{b}h{h}")
            # dequantize + cuBLAS matmul (triton_kernels.py:300-311)
            s3 = _torch_attention_scores(codec, qh, kh, kv_head=h)
            assert_close_rowwise(s3.cpu().numpy(), ref, TOL_F32, f"{name} _torch_attention_scores b{b}h{h}")
    if g["Hkv"] > 1:
        with pytest.raises(RuntimeError, match="kv_head"):
            sunshape_attention_scores(codec, torch.zeros(1, g["D"], device=DEV), keys.head(0, 0))


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_dequantize_is_exact_gather(name):
    g = load_golden(name)
    codec = golden_codec(g)
    k = vab.dequantize_keys(codec, golden_keys(g)).cpu().numpy()
    hm = g["heavy_mask"]
    for b in range(g["B"]):
        for h in range(g["Hkv"]):
            ref = O.dequantize(g["ref_indices"][b, h], g["centroids"][h], g["inv_perm"], hm if hm.any() else None,
                               g["ref_passthrough"][b, h] if hm.any() else None)
            if g["dtype"] == "bf16" and hm.any():
                ref = ref  # heavy values are bf16-exact by construction
            np.testing.assert_array_equal(k[b, h], ref)


# ---------------------------------------------------------------------------------------------
# Seeded cases beyond the goldens, checked against the oracle: ragged tails, cache views, GQA
# widths that need row chunking, masks, query_len > 1.
# ---------------------------------------------------------------------------------------------
def _oracle_out(case, idx, heavy, mask, scale):
    cfg = case["cfg"]
    hm = case["heavy_mask"].cpu().numpy()
    cents = case["centroids"].cpu().numpy()
    idx_n = idx.cpu().numpy()
    heavy_n = None if heavy is None else heavy.float().cpu().numpy()
    nb, bd = cfg.n_blocks, cfg.block_dim
    heads = []
    for b in range(cfg.batch):
        for h in range(cfg.kv_heads):
            pt = None
            if hm.any():
                pt = np.zeros((cfg.seq_len, nb, bd), np.float32)
                pt[:, hm] = heavy_n[b, h]
            heads.append((idx_n[b, h], hm if hm.any() else None, pt))
    return O.apply_quantized_attention(
        case["query"].float().cpu().numpy(), heads, case["value"].float().cpu().numpy(),
        centroids_for_head=lambda h: cents[h], inv_perm=case["inv_perm"].cpu().numpy(),
        attn_mask=None if mask is None else mask.float().cpu().numpy(), scale=scale, query_dtype=cfg.dtype,
        value_dtype=cfg.dtype)


SEEDED = {
    "c2_ragged": CONFIGS["c2"].with_(batch=2, kv_heads=2, q_heads=8, seq_len=8192 + 37),
    "c3_bd4": CONFIGS["c3"].with_(batch=1, kv_heads=2, q_heads=8, seq_len=3000),
    "c4_mixed": CONFIGS["c4"].with_(batch=2, kv_heads=2, q_heads=8, seq_len=2049),
    "c5_g8": CONFIGS["c5"].with_(batch=1, kv_heads=2, q_heads=16, seq_len=20000),
    "g16_chunked": CONFIGS["c2"].with_(batch=1, kv_heads=1, q_heads=16, seq_len=777),
    "g7_fp32": CONFIGS["c1"].with_(seq_len=4096),
    "g12_f16": CONFIGS["c2"].with_(batch=1, kv_heads=2, q_heads=24, seq_len=100, dtype="f16"),
    "t_short": CONFIGS["c2"].with_(batch=3, kv_heads=2, q_heads=4, seq_len=5),
    "qlen3": CONFIGS["c2"].with_(batch=1, kv_heads=2, q_heads=4, seq_len=300, query_len=3),
    "dv64_g1": CONFIGS["c1"].with_(q_heads=2, kv_heads=2, seq_len=1000, dtype="bf16"),
    # block_dim 2 (64 blocks per head, the reference's default 4 bits/dim): fp16-entry LUTs, 4 rows per launch
    "bd2_g8": CONFIGS["c5"].with_(batch=2, kv_heads=2, q_heads=16, seq_len=5000 + 3, block_dim=2),
    "bd2_mixed": CONFIGS["c4"].with_(batch=1, kv_heads=2, q_heads=8, seq_len=3000, block_dim=2, n_heavy=2),
    "bd2_fp32": CONFIGS["c1"].with_(head_dim=128, seq_len=2000, block_dim=2),
}


@pytest.mark.parametrize("name", list(SEEDED))
def test_decode_matches_oracle_seeded(name):
    cfg = SEEDED[name]
    case = make_case(cfg, device=DEV, seed=11)
    codec = make_codec(case["perm"], case["centroids"], case["heavy_mask"], cfg.head_dim, cfg.block_dim,
                       cfg.n_centroids, DEV)
    qk = vab.quantize_codec_keys(codec, case["keys"])
    mask = None
    if name in ("c2_ragged", "qlen3", "bd2_fp32"):
        gen = torch.Generator(device=DEV).manual_seed(3)
        mask = torch.randn(cfg.batch, cfg.q_heads, cfg.query_len, cfg.seq_len, device=DEV, generator=gen)
        mask[..., ::5] = float("-inf")
    scale = None if name == "g7_fp32" else case["scale"]
    out = vab._apply_quantized_attention(codec=codec, query=case["query"], key=qk, value=case["value"],
                                         attn_mask=mask, scale=scale)
    ref = _oracle_out(case, qk.indices, qk.heavy, mask, scale)
    if cfg.dtype == "f32" and mask is None:
        # fp32 at logits of ~80 (no scale): the reference's own fp32 arithmetic is ~1e-5 per row away
        # from exact arithmetic, so the bound is 1e-5 plus that measured error of the reference
        exact = _exact_out(case, qk.indices, scale)
        ref_err = (np.abs(ref - exact).reshape(-1, cfg.head_dim).max(1) /
                   np.abs(exact).reshape(-1, cfg.head_dim).max(1))
        ours = out.float().cpu().numpy()
        err = np.abs(ours - ref).reshape(-1, cfg.head_dim).max(1) / np.abs(ref).reshape(-1, cfg.head_dim).max(1)
        assert (err <= TOL_F32 + ref_err).all(), (err.max(), ref_err.max())
        return
    tol = TOL_F32 if cfg.dtype == "f32" else TOL_BF16
    assert_close_rowwise(out.float().cpu().numpy(), ref, tol, name)


def _exact_out(case, idx, scale):
    """fp64 softmax(q k_hat^T) V of an unmasked case (the error-free value of the same quantities)."""
    cfg = case["cfg"]
    cents = case["centroids"].cpu().numpy()
    inv = case["inv_perm"].cpu().numpy()
    q = case["query"].double().cpu().numpy()
    v = case["value"].double().cpu().numpy()
    idx_n = idx.cpu().numpy()
    G, L = cfg.group, cfg.query_len
    out = np.zeros((cfg.batch, cfg.q_heads, L, cfg.head_dim))
    for b in range(cfg.batch):
        for h in range(cfg.kv_heads):
            kh = O.dequantize(idx_n[b, h], cents[h], inv).astype(np.float64)
            qq = q[b, h * G:(h + 1) * G].reshape(-1, cfg.head_dim) * (1.0 if scale is None else scale)
            s = qq @ kh.T
            p = np.exp(s - s.max(1, keepdims=True))
            p /= p.sum(1, keepdims=True)
            out[b, h * G:(h + 1) * G] = (p @ v[b, h]).reshape(G, L, -1)
    return out


# The in-CTA LUT branch: with the smallest accepted workspace (no room for the per-head LUT area),
# every CTA builds its heads' LUTs in shared memory instead of the separate LUT kernel.
MIN_WS = {
    "c5_g8_fp16lut": CONFIGS["c5"].with_(batch=2, kv_heads=2, q_heads=16, seq_len=20000),
    "c3_nb32": CONFIGS["c3"].with_(batch=1, kv_heads=2, q_heads=8, seq_len=9000),
    "c2_g4": CONFIGS["c2"].with_(batch=3, kv_heads=2, q_heads=8, seq_len=7000 + 3),
    "c4_mixed": CONFIGS["c4"].with_(batch=1, kv_heads=2, q_heads=8, seq_len=5000),
}


@pytest.mark.parametrize("name", list(MIN_WS))
def test_decode_in_cta_lut_with_minimum_workspace(name):
    from sunshape_b200 import _lib

    cfg = MIN_WS[name]
    case = make_case(cfg, device=DEV, seed=23)
    codec = make_codec(case["perm"], case["centroids"], case["heavy_mask"], cfg.head_dim, cfg.block_dim,
                       cfg.n_centroids, DEV)
    qk = vab.quantize_codec_keys(codec, case["keys"])
    n_heads, rows = cfg.batch * cfg.kv_heads, cfg.group * cfg.query_len
    need_min = _lib.decode_workspace_min_bytes(n_heads, cfg.seq_len, rows, cfg.head_dim)
    need_full = int(_lib.load_library().sunshape_decode_workspace_bytes(n_heads, cfg.seq_len, rows, cfg.head_dim,
                                                                        cfg.n_blocks))
    assert need_min < need_full
    ws = torch.zeros(need_min, dtype=torch.uint8, device=DEV)
    desc, keep, _ = codec.kernel_desc()
    kd = _lib.kv_desc(qk.indices, qk.heavy, case["value"], cfg.seq_len, cfg.seq_len, cfg.head_dim)
    ref = _oracle_out(case, qk.indices, qk.heavy, None, case["scale"])
    for call in range(2):     # the workspace's tickets must be left at zero for the next call
        out = torch.empty(cfg.batch, cfg.q_heads, 1, cfg.head_dim, device=DEV, dtype=case["value"].dtype)
        _lib.decode_attention(desc, kd, case["query"], cfg.batch, cfg.q_heads, cfg.kv_heads, 1, None, (0, 0, 0),
                              case["scale"], out, None, workspace=ws)
        torch.cuda.synchronize()
        assert int(ws[:4].view(torch.int32).item()) == 0
        assert_close_rowwise(out.float().cpu().numpy(), ref, TOL_BF16, f"{name} in-CTA LUT call {call}")
    # and the LUT-kernel path on the same inputs agrees with it
    full = vab._apply_quantized_attention(codec=codec, query=case["query"], key=qk, value=case["value"],
                                          attn_mask=None, scale=case["scale"])
    assert_close_rowwise(full.float().cpu().numpy(), ref, TOL_BF16, f"{name} LUT kernel")


def test_cache_view_head_stride_and_fully_masked_row():
    cfg = CONFIGS["c2"].with_(batch=2, kv_heads=2, q_heads=8, seq_len=300)
    case = make_case(cfg, device=DEV, seed=5)
    codec = make_codec(case["perm"], case["centroids"], case["heavy_mask"], 128, 8, 256, DEV)
    qk = vab.quantize_codec_keys(codec, case["keys"])
    T, cap = cfg.seq_len, 512
    idx_cap = torch.zeros(2, 2, cap, 16, dtype=torch.uint8, device=DEV)
    v_cap = torch.zeros(2, 2, cap, 128, dtype=torch.bfloat16, device=DEV)
    idx_cap[:, :, :T] = qk.indices
    v_cap[:, :, :T] = case["value"]
    view = vab.SunShapeQuantizedKeys((), 2, 2, T, indices=idx_cap[:, :, :T])
    mask = torch.zeros(2, 8, 1, T, device=DEV)
    mask[1, 3] = float("-inf")                          # one fully masked row -> NaN like torch.softmax
    out = vab._apply_quantized_attention(codec=codec, query=case["query"], key=view, value=v_cap[:, :, :T],
                                         attn_mask=mask, scale=case["scale"])
    ref = _oracle_out(case, qk.indices, None, mask, case["scale"])
    assert torch.isnan(out[1, 3]).all()
    assert_close_rowwise(out.float().cpu().numpy(), ref, TOL_BF16, "cache view")


def test_split_kv_partials_merge_equals_full():
    """Size-independent property: merging per-shard partials reproduces the single-shot output."""
    from sunshape_b200 import _lib
    from sunshape_b200.distributed import kv_shard_bounds

    cfg = CONFIGS["c5"].with_(batch=2, kv_heads=2, q_heads=16, seq_len=50000)
    case = make_case(cfg, device=DEV, seed=7)
    codec = make_codec(case["perm"], case["centroids"], case["heavy_mask"], 128, 8, 256, DEV)
    qk = vab.quantize_codec_keys(codec, case["keys"])
    full = vab._apply_quantized_attention(codec=codec, query=case["query"], key=qk, value=case["value"],
                                          attn_mask=None, scale=case["scale"])
    parts = []
    for r in range(3):
        a, b = kv_shard_bounds(cfg.seq_len, 3, r)
        sh = vab.SunShapeQuantizedKeys((), 2, 2, b - a, indices=qk.indices[:, :, a:b])
        parts.append(vab.decode_partials(codec=codec, query=case["query"], key=sh, value=case["value"][:, :, a:b],
                                         scale=case["scale"]))
    merged = torch.empty(full.numel() // 128, 128, device=DEV, dtype=torch.bfloat16)
    _lib.merge_partials(torch.stack(parts), merged)
    assert_close_rowwise(merged.view_as(full).float().cpu().numpy(), full.float().cpu().numpy(), 1e-2, "merge")


def test_unsupported_inputs_raise_with_reason():
    codec = make_codec(torch.randperm(256), torch.randn(1, 128, 256, 2), torch.zeros(128, dtype=torch.bool), 256, 2,
                       256, DEV)
    q = torch.randn(1, 4, 1, 256, device=DEV, dtype=torch.bfloat16)
    v = torch.randn(1, 1, 10, 256, device=DEV, dtype=torch.bfloat16)
    keys = vab.SunShapeQuantizedKeys((), 1, 1, 10, indices=torch.zeros(1, 1, 10, 128, dtype=torch.uint8, device=DEV))
    with pytest.raises(RuntimeError, match="n_blocks > 64"):
        vab._apply_quantized_attention(codec=codec, query=q, key=keys, value=v, attn_mask=None, scale=None)


def test_no_device_errors_recorded():
    from sunshape_b200 import _lib

    torch.cuda.synchronize()
    assert _lib.decode_error_word() == 0
    assert _lib.encode_error_word(torch.device(DEV)) == 0
