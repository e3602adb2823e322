"""Generate golden vectors by running the REFERENCE SunShape code on seeded inputs.

Run in a container that has the reference checkout (it is not needed anywhere else):

    PYTHONPATH=<reference checkout> python tests/golden/make_golden.py

For every case this imports the reference package unmodified, builds one codec
per KV head by writing its buffers directly (the configs use per-KV-head
codebooks; the reference keeps one codec per layer, so the oracle loops over
heads), and records the reference's own outputs:

* ``codec.quantize`` indices / passthrough      (codec.py:362-385)
* ``_torch_attention_scores`` per head           (triton_kernels.py:300-311)
* ``_apply_quantized_attention`` output          (vllm_attn_backend.py:216-253)
* a bundle saved by ``SunShapeBundle.save`` and the decode of its layers through
  ``SunShapeAttentionImpl.forward`` (``bundle_ref.pt``, ``g7_bundle.npz``)
* the keys and values ``SunShapeCache.update`` stores over prefill + decode (``g8_cache.npz``)

The results are written to ``tests/golden/<case>.npz`` together with the inputs,
so tests never need the reference at run time.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from sunshape_b200.workloads import CONFIGS, make_case  # noqa: E402

CASES = {
    # c1-shaped (fp32, GQA 7:1, D64, bd8) at T=1024
    "g1_c1_fp32": dict(cfg=CONFIGS["c1"].with_(seq_len=1024), scale=None, mask=None),
    # bf16 GQA 4:1, ragged T, 4-D additive mask with -inf holes, scale given
    "g2_bf16_mask4d": dict(cfg=CONFIGS["c2"].with_(batch=2, q_heads=8, kv_heads=2, seq_len=333),
                           scale="default", mask="4d"),
    # SunShape-Mixed, 4 heavy blocks of 16
    "g3_mixed": dict(cfg=CONFIGS["c4"].with_(batch=1, q_heads=8, kv_heads=2, seq_len=500),
                     scale="default", mask=None),
    # bd=4 (2 bits/dim, 32 blocks)
    "g4_bd4": dict(cfg=CONFIGS["c3"].with_(batch=1, q_heads=4, kv_heads=1, seq_len=256),
                   scale="default", mask="2d"),
    # smallest: one token, MHA (G=1)
    "g5_t1_g1": dict(cfg=CONFIGS["c1"].with_(q_heads=2, kv_heads=2, seq_len=1, dtype="bf16"),
                     scale="default", mask=None),
    # query_len 2 (non-causal) and a 3-D per-head mask, G=8
    # block_dim 2 (the reference's default 4 bits/dim): 64 blocks per head at head_dim 128
    "g9_bd2": dict(cfg=CONFIGS["c2"].with_(batch=1, q_heads=8, kv_heads=2, seq_len=300, block_dim=2),
                   scale="default", mask="2d"),
    # SunShape-Pro: block-diagonal local metric E (codec.py:375-377), per-KV-head codebooks
    "g10_pro_metric": dict(cfg=CONFIGS["c2"].with_(batch=1, q_heads=8, kv_heads=2, seq_len=400),
                           scale="default", mask=None, metric=True),
    "g6_qlen2_mask3d": dict(cfg=CONFIGS["c5"].with_(batch=1, q_heads=16, kv_heads=2, seq_len=129,
                                                    head_dim=64, query_len=2),
                            scale="default", mask="3d"),
}


def _mask(kind, cfg, gen):
    B, Hq, L, T = cfg.batch, cfg.q_heads, cfg.query_len, cfg.seq_len
    if kind is None:
        return None
    if kind == "4d":
        m = torch.randn(B, Hq, L, T, generator=gen) * 0.5
        m[..., ::7] = float("-inf")
        return m
    if kind == "3d":
        m = torch.randn(Hq, L, T, generator=gen)
        m[:, :, -5:] = float("-inf")
        return m
    if kind == "2d":
        m = torch.zeros(L, T)
        m[:, : T // 3] = float("-inf")
        return m
    raise ValueError(kind)


def run_case(name, spec):
    from sunshape.codec import SunShapeBlockCodec
    from sunshape.triton_kernels import _torch_attention_scores
    from sunshape.vllm_attn_backend import SunShapeQuantizedKeys, _apply_quantized_attention

    cfg = spec["cfg"]
    case = make_case(cfg, device="cpu", seed=0)
    scale = None if spec["scale"] is None else case["scale"]
    mask = _mask(spec["mask"], cfg, torch.Generator().manual_seed(5))
    B, Hq, Hkv, D, T = cfg.batch, cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.seq_len
    G = cfg.group
    mode = "profileperm_mixed_precision" if cfg.n_heavy else "profileperm_baseline"
    E = None
    if spec.get("metric"):
        mode = "profileperm_localmetric_dsq"
        gm = torch.Generator().manual_seed(9)
        bd = cfg.block_dim
        E = torch.zeros(D, D)
        for b in range(cfg.n_blocks):
            a = torch.randn(bd, bd, generator=gm) * 0.3
            E[b * bd:(b + 1) * bd, b * bd:(b + 1) * bd] = torch.eye(bd) + 0.5 * (a + a.T)

    codecs = []
    for h in range(Hkv):
        codec = SunShapeBlockCodec(head_dim=D, block_dim=cfg.block_dim, n_centroids=cfg.n_centroids,
                                   mode=mode, device=torch.device("cpu"))
        codec.permutation.copy_(case["perm"])
        codec.inv_permutation.copy_(case["inv_perm"])
        codec.centroids.copy_(case["centroids"][h])
        codec.mixed_high_precision_blocks.copy_(case["heavy_mask"])
        if E is not None:
            codec.E.copy_(E)
            codec.E_inv.copy_(torch.linalg.pinv(E))
        codecs.append(codec)

    nb, bd = cfg.n_blocks, cfg.block_dim
    indices = np.zeros((B, Hkv, T, nb), dtype=np.uint8)
    passthrough = np.zeros((B, Hkv, T, nb, bd), dtype=np.float32)
    scores = np.zeros((B, Hkv, G * cfg.query_len, T), dtype=np.float32)
    out = torch.empty(B, Hq, cfg.query_len, D, dtype=cfg.torch_dtype)
    for b in range(B):
        for h in range(Hkv):
            qk = codecs[h].quantize(case["keys"][b, h])
            indices[b, h] = qk.indices.numpy()
            if qk.passthrough_values is not None:
                passthrough[b, h] = qk.passthrough_values.numpy()
            qs = case["query"][b, h * G:(h + 1) * G]
            if scale is not None:
                qs = qs * float(scale)
            scores[b, h] = _torch_attention_scores(codecs[h], qs.reshape(-1, D), qk).numpy()
            keys_obj = SunShapeQuantizedKeys(quantized_heads=(qk,), batch_size=1, num_kv_heads=1, seq_len=T)
            m = None
            if mask is not None:
                if mask.ndim == 4:
                    m = mask[b:b + 1, h * G:(h + 1) * G]
                elif mask.ndim == 3:
                    m = mask[h * G:(h + 1) * G]
                else:
                    m = mask
            out[b:b + 1, h * G:(h + 1) * G] = _apply_quantized_attention(
                codec=codecs[h], query=case["query"][b:b + 1, h * G:(h + 1) * G], key=keys_obj,
                value=case["value"][b:b + 1, h:h + 1], attn_mask=m, scale=scale)

    def f32(t):
        return t.float().numpy()

    payload = dict(
        B=B, Hq=Hq, Hkv=Hkv, D=D, T=T, L=cfg.query_len, block_dim=bd, n_centroids=cfg.n_centroids,
        dtype=cfg.dtype, scale=np.float64("nan") if scale is None else np.float64(scale),
        keys=f32(case["keys"]), perm=case["perm"].numpy(), inv_perm=case["inv_perm"].numpy(),
        centroids=f32(case["centroids"]), heavy_mask=case["heavy_mask"].numpy(),
        query=f32(case["query"]), value=f32(case["value"]),
        mask=np.zeros(0, np.float32) if mask is None else f32(mask),
        ref_indices=indices, ref_passthrough=passthrough, ref_scores=scores, ref_out=f32(out),
        **({"E": E.numpy()} if E is not None else {}),
    )
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **payload)
    print(f"{name}: wrote {os.path.getsize(path) / 1024:.0f} KiB")


def _ref_codec(cfg, case, mode):
    """A reference codec (one codebook shared by all KV heads, the reference's layout) with its
    buffers written from the seeded case: codebook of KV head 0."""
    from sunshape.codec import SunShapeBlockCodec

    codec = SunShapeBlockCodec(head_dim=cfg.head_dim, block_dim=cfg.block_dim, n_centroids=cfg.n_centroids,
                               mode=mode, device=torch.device("cpu"))
    codec.permutation.copy_(case["perm"])
    codec.inv_permutation.copy_(case["inv_perm"])
    codec.centroids.copy_(case["centroids"][0])
    codec.mixed_high_precision_blocks.copy_(case["heavy_mask"])
    return codec


def run_bundle():
    """A bundle written by the reference's SunShapeBundle.save (hf.py:273-303) with two layers -- one
    SunShape-base, one SunShape-Mixed -- plus, per layer, the reference's decode through its public
    backend: runtime registry -> SunShapeAttentionImpl.forward (vllm_attn_backend.py:271-305) on keys
    quantized by quantize_key_states (:101-123)."""
    from sunshape import vllm_attn_backend as rb
    from sunshape.hf import SunShapeBundle
    from sunshape.integration.vllm import SunShapeVLLMRuntimeState

    layer_cfgs = {3: (CONFIGS["c2"].with_(batch=2, q_heads=8, kv_heads=2, seq_len=300), "profileperm_baseline"),
                  5: (CONFIGS["c4"].with_(batch=1, q_heads=8, kv_heads=2, seq_len=200), "profileperm_mixed_precision")}
    codecs, cases = {}, {}
    for layer, (cfg, mode) in layer_cfgs.items():
        case = make_case(cfg, device="cpu", seed=40 + layer)
        codecs[layer] = _ref_codec(cfg, case, mode)
        cases[layer] = (cfg, case)
    bundle = SunShapeBundle(model_name="synthetic-ref", layers=sorted(codecs), bits_per_dim=1.0, block_dim=8,
                            mode="sunshape_base", cal_points=256, dsq_steps=0, seed=0, codecs=codecs,
                            trace_meta={"source": "make_golden.py"})
    bpath = os.path.join(HERE, "bundle_ref.pt")
    bundle.save(bpath)
    state = SunShapeVLLMRuntimeState(bundle_path=bpath, model_name="synthetic-ref", mode="sunshape_base",
                                     bits_per_dim=1.0, block_dim=8, layers=sorted(codecs), bundle=bundle,
                                     device="cpu")
    rb.register_runtime_state(state)
    payload = {}
    for layer, (cfg, case) in cases.items():
        keys = case["keys"]
        if cfg.dtype != "f32":
            keys = keys.to(cfg.torch_dtype)        # a model hands 16-bit keys to the backend
        qk = rb.quantize_key_states(layer, keys)
        impl = rb.SunShapeAttentionImpl(layer_idx=layer, runtime_state=state)
        out = impl.forward(case["query"], qk, case["value"], scale=case["scale"])
        idx = np.stack([h.indices.numpy() for h in qk.quantized_heads]).reshape(cfg.batch, cfg.kv_heads,
                                                                                cfg.seq_len, -1)
        pre = f"l{layer}_"
        payload.update({pre + "keys": keys.float().numpy(), pre + "query": case["query"].float().numpy(),
                        pre + "value": case["value"].float().numpy(), pre + "scale": np.float64(case["scale"]),
                        pre + "dtype": cfg.dtype, pre + "ref_indices": idx.astype(np.uint8),
                        pre + "ref_out": out.float().numpy()})
    rb.clear_registered_runtime()
    path = os.path.join(HERE, "g7_bundle.npz")
    np.savez_compressed(path, layers=np.array(sorted(cases)), **payload)
    print(f"bundle_ref.pt: {os.path.getsize(bpath) / 1024:.0f} KiB; g7_bundle: {os.path.getsize(path) / 1024:.0f} KiB")


def run_cache():
    """The reference's HF cache (cache.py:32-46, 55-104): a prefill of 37 bf16 keys then two decode
    steps through SunShapeCache.update on layer 1 (layer 0 unquantized); records what the cache
    stores (the fake-quantized keys and the values) after every update."""
    from sunshape.cache import SunShapeCache

    cfg = CONFIGS["c2"].with_(batch=2, q_heads=8, kv_heads=2, head_dim=64, seq_len=39)
    case = make_case(cfg, device="cpu", seed=61)
    codec = _ref_codec(cfg, case, "profileperm_baseline")
    cache = SunShapeCache.from_codecs({1: codec}, num_layers=2)
    keys = case["keys"].to(torch.bfloat16)
    vals = case["value"]
    steps = [(0, 37), (37, 38), (38, 39)]
    payload = {"keys": keys.float().numpy(), "value": vals.float().numpy(), "perm": case["perm"].numpy(),
               "inv_perm": case["inv_perm"].numpy(), "centroids": case["centroids"][0].numpy(),
               "steps": np.array(steps)}
    for i, (a, b) in enumerate(steps):
        for layer in (0, 1):
            k_out, v_out = cache.update(keys[:, :, a:b], vals[:, :, a:b], layer)
            payload[f"step{i}_l{layer}_keys"] = k_out.float().numpy()
            payload[f"step{i}_l{layer}_values"] = v_out.float().numpy()
    path = os.path.join(HERE, "g8_cache.npz")
    np.savez_compressed(path, **payload)
    print(f"g8_cache: wrote {os.path.getsize(path) / 1024:.0f} KiB")


def run_turbo():
    """The reference's TurboQuant-MSE (turbo_baseline.py:117-186) at 1, 2 and 3 bits: rotation,
    indices, norms and compressed-key attention scores for seeded keys and queries."""
    from sunshape.turbo_baseline import TurboQuantMSE

    g = torch.Generator().manual_seed(71)
    d = 128
    x = torch.randn(300, d, generator=g) * 0.7
    q = torch.randn(8, d, generator=g)
    payload = {"x": x.numpy(), "q": q.numpy()}
    for bits in (1, 2, 3):
        tq = TurboQuantMSE(d, bits=bits, seed=5 + bits, device=torch.device("cpu"))
        comp = tq.compress(x)
        payload[f"b{bits}_rotation"] = tq.rotation.numpy()
        payload[f"b{bits}_centroids"] = tq.centroids.numpy()
        payload[f"b{bits}_indices"] = comp.indices.numpy().astype(np.uint8)
        payload[f"b{bits}_norms"] = comp.qjl_norms.numpy()
        payload[f"b{bits}_scores"] = tq.attention_scores(q, comp).numpy()
        payload[f"b{bits}_roundtrip"] = tq(x).numpy()
    path = os.path.join(HERE, "g11_turbo.npz")
    np.savez_compressed(path, **payload)
    print(f"g11_turbo: wrote {os.path.getsize(path) / 1024:.0f} KiB")


if __name__ == "__main__":
    import sunshape  # noqa: F401  (must resolve to the reference checkout)
    which = set(sys.argv[1:])
    torch.manual_seed(0)
    for n, s in CASES.items():
        if not which or n in which:
            run_case(n, s)
    if not which or "bundle" in which:
        run_bundle()
    if not which or "cache" in which:
        run_cache()
    if not which or "turbo" in which:
        run_turbo()
