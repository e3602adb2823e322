"""KV-sequence split across ranks, on CPU gloo ranks (world size 2): sharding, the partial
all-gather and the merge reproduce the single-rank softmax; a rank that fails before the
collective makes the other rank's collective fail with an error instead of hanging."""
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import sunshape_oracle as O
from sunshape_b200.distributed import gather_partials, kv_shard_bounds
from tests.helpers import load_golden


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _worker_merge(rank, world, port, q):
    try:
        _init(rank, world, port)
        g = load_golden("g1_c1_fp32")
        T = g["T"]
        a, b = kv_shard_bounds(T, world, rank)
        hm = g["heavy_mask"]
        heads = [(g["ref_indices"][bb, h][a:b], None, None) for bb in range(g["B"]) for h in range(g["Hkv"])]
        m, l, acc = O.decode_partials(g["query"], heads, g["value"][:, :, a:b],
                                      centroids_for_head=lambda h: g["centroids"][h], inv_perm=g["inv_perm"],
                                      scale=g["scale"], query_dtype=g["dtype"])
        rows = m.size
        part = torch.from_numpy(np.concatenate([m.reshape(rows, 1), l.reshape(rows, 1),
                                                acc.reshape(rows, -1)], axis=1))
        gathered = gather_partials(part).numpy()          # [world, rows, 2 + Dv]
        merged = O.merge_partials([gathered[r][:, 0] for r in range(world)],
                                  [gathered[r][:, 1] for r in range(world)],
                                  [gathered[r][:, 2:] for r in range(world)])
        out = merged.reshape(g["ref_out"].shape)
        err = float(np.abs(out - g["ref_out"]).max() / np.abs(g["ref_out"]).max())
        q.put((rank, "ok", err))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def test_kv_split_merge_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_merge, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, status, val in res:
        assert status == "ok", val
        assert val <= 1e-5, f"rank {rank}: merged output differs from the reference by {val:.2e}"


def _worker_fail(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            q.put((rank, "raised", ""))
            raise SystemExit(1)      # this rank dies between steps, before its collective
        part = torch.zeros(4, 10)
        try:
            gather_partials(part)
            q.put((rank, "no-error", ""))
        except Exception as exc:     # the survivor learns of it through the collective's error
            q.put((rank, "error-seen", type(exc).__name__))
    except SystemExit:
        pass
    except Exception:
        q.put((rank, "setup-error", traceback.format_exc()))


def test_failed_rank_surfaces_as_collective_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_fail, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (s, v)) for r, s, v in (q.get(timeout=240) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1][0] == "raised"
    assert res[0][0] == "error-seen", res[0]
