"""KV-sequence split across 2 GPUs (skipped with fewer): the fused peer-memory exchange and the
NCCL all-gather path both reproduce the single-GPU decode output, over several consecutive calls
(the exchange buffers alternate halves between calls)."""
import os
import socket
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        import numpy as np
        import torch.distributed as dist

        from sunshape_b200 import vllm_attn_backend as vab
        from sunshape_b200.distributed import KVShardedDecode, kv_shard_bounds
        from sunshape_b200.workloads import CONFIGS, make_case
        from tests.helpers import make_codec

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        cfg = CONFIGS["c5"].with_(batch=2, kv_heads=2, q_heads=16, seq_len=30000 + 7)
        case = make_case(cfg, device=dev, seed=17)
        codec = make_codec(case["perm"], case["centroids"], case["heavy_mask"], 128, 8, 256, dev)
        qk = vab.quantize_codec_keys(codec, case["keys"])
        full = vab._apply_quantized_attention(codec=codec, query=case["query"], key=qk, value=case["value"],
                                              attn_mask=None, scale=case["scale"]).float().cpu().numpy()
        a, b = kv_shard_bounds(cfg.seq_len, world, rank)
        shard = vab.SunShapeQuantizedKeys((), cfg.batch, cfg.kv_heads, b - a,
                                          indices=qk.indices[:, :, a:b].contiguous())
        v = case["value"][:, :, a:b].contiguous()
        errs = {}
        for mode in ("p2p", "peer", "nccl"):
            dec = KVShardedDecode(codec, exchange=mode)
            worst = 0.0
            for call in range(3):
                qry = case["query"] * (1.0 + 0.25 * call)      # different queries each call
                ref = full if call == 0 else vab._apply_quantized_attention(
                    codec=codec, query=qry, key=qk, value=case["value"], attn_mask=None,
                    scale=case["scale"]).float().cpu().numpy()
                out = dec(qry, shard, v, scale=case["scale"]).float().cpu().numpy()
                rows_err = np.abs(out - ref).reshape(-1, ref.shape[-1]).max(1) / np.abs(ref).reshape(-1, ref.shape[-1]).max(1)
                worst = max(worst, float(rows_err.max()))
            errs[mode] = worst
        torch.cuda.synchronize()
        q.put((rank, "ok", errs))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_kv_split_two_gpus_peer_and_nccl_match_single_gpu():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, status, val in res:
        assert status == "ok", val
        for mode, err in val.items():
            assert err <= 2e-2, f"rank {rank} {mode}: worst per-row error {err:.3e}"
