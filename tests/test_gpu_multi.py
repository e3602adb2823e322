"""KV-sequence split across 2 GPUs (skipped with fewer): the fused peer-memory exchange and the
NCCL all-gather path both reproduce the single-GPU decode output, over several consecutive calls
(the exchange buffers alternate halves between calls)."""
import ctypes
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


def test_peer_exchange_poisoned_buffer_reports_error():
    """A merge that gave up on a peer poisons the exchange buffer: later calls must record error 106 and
    write NaN rows instead of merging stale arrivals, until a new buffer is set up.  Driven on one GPU:
    a two-rank group whose two buffer entries are the same buffer, with rank 1's rows pre-set to an
    empty shard (m = -inf), so both arrival bumps land here and the merge equals the single-GPU
    decode.  The poison word is set by hand, so no wait ever times out."""
    import math

    from sunshape_b200 import _lib
    from sunshape_b200 import vllm_attn_backend as vab
    from sunshape_b200.workloads import CONFIGS, make_case
    from tests.helpers import TOL_BF16, assert_close_rowwise, make_codec

    dev = torch.device("cuda", 0)
    cfg = CONFIGS["c5"].with_(batch=2, kv_heads=2, q_heads=16, seq_len=3000)
    case = make_case(cfg, device=dev, seed=5)
    codec = make_codec(case["perm"], case["centroids"], case["heavy_mask"], 128, 8, 256, dev)
    qk = vab.quantize_codec_keys(codec, case["keys"])
    ref = vab._apply_quantized_attention(codec=codec, query=case["query"], key=qk, value=case["value"],
                                         attn_mask=None, scale=case["scale"]).float()
    lib = _lib.load_library()
    rows, n_heads, dv = cfg.batch * cfg.q_heads, cfg.batch * cfg.kv_heads, cfg.head_dim
    nbytes = int(lib.sunshape_peer_buffer_bytes(2, rows, dv, n_heads))
    desc, keep, _ = codec.kernel_desc()
    kd = _lib.kv_desc(qk.indices, None, case["value"], cfg.seq_len, cfg.seq_len, cfg.head_dim)
    ws = _lib.decode_workspace(dev, n_heads, cfg.seq_len, cfg.group, dv, cfg.n_blocks)
    up = lambda x: (x + 255) // 256 * 256
    poison_off = up(2 * 2 * rows * (dv + 2) * 4) + up(2 * n_heads * 4) + 8

    def new_buffer():
        buf = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        recv = buf[:2 * 2 * rows * (dv + 2) * 4].view(torch.float32).view(2, 2, rows, dv + 2)
        recv[:, 1, :, 0] = float("-inf")      # rank 1 holds no tokens: its rows drop out of the merge
        return buf

    def run(buf):
        p = buf.data_ptr()
        grp = _lib.PeerGroupDesc(0, 2, (ctypes.c_void_p * 8)(p, p, *([None] * 6)))
        out = torch.empty(cfg.batch, cfg.q_heads, 1, dv, device=dev, dtype=case["value"].dtype)
        _lib.decode_attention_peers(desc, kd, case["query"], cfg.batch, cfg.q_heads, cfg.kv_heads, 1, None,
                                    (0, 0, 0), case["scale"], out, grp)
        torch.cuda.synchronize()
        return out.float(), int(ws[:4].view(torch.int32).item())

    try:
        buf = new_buffer()
        for _ in range(3):   # healthy buffer: the merged output is the single-GPU output
            out, err = run(buf)
            assert err == 0
            assert_close_rowwise(out.cpu().numpy(), ref.cpu().numpy(), TOL_BF16, "peer exchange, self group")
        buf[poison_off:poison_off + 4].view(torch.int32).fill_(1)
        for _ in range(2):
            out, err = run(buf)
            assert err == 106
            assert torch.isnan(out).all()
            ws[:4].zero_()
        fresh = new_buffer()
        out, err = run(fresh)
        assert err == 0 and not math.isnan(float(out.sum()))
        assert_close_rowwise(out.cpu().numpy(), ref.cpu().numpy(), TOL_BF16, "fresh exchange buffer")
    finally:
        ws[:4].zero_()
