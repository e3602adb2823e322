"""Benchmark of the SunShape quantized-key decode path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c5]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU, NCCL)

A step is one decode-attention pass over the whole synthetic KV cache of the
workload (default ``c5``: batch 8, 64 query / 8 KV heads, head_dim 128, 128K
context, block_dim 8, uint8 indices, bf16 values -- the 1/2/4/8-GPU config).
With N GPUs the KV sequence is split evenly (strong scaling: total work fixed);
each rank runs the fused kernel on its shard, the (max, sum, acc) partials are
all-gathered over NCCL and merged.  Inputs (2.28 GB at N=1) are larger than the
126 MB L2, so no flush is needed between steps.

Prints ONE JSON line (rank 0).  ``value`` is whole-job KV tokens/s with inputs
resident in HBM; ``e2e`` is the same metric through the public API
(``SunShapeAttentionImpl.forward`` / ``KVShardedDecode``) with the step's query
copied from pinned host memory and the output copied back inside the timed
region.  ``--impl reference`` times the unmodified reference package
(installed into ``baseline/_ref``, which travels with the repository) through its
own ``_apply_quantized_attention`` on the host cores, one sequence of the workload
per step, with every host thread.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from sunshape_b200.workloads import CONFIGS, DecodeConfig, make_case  # noqa: E402

METRIC = "KV tokens scored/s and HBM GB/s (% of peak), VQ decode attn, 1/2/4/8 B200"
UNIT = "KV tokens/s"
FALLBACK_HBM_GBS = 6650.0


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ----------------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            import tempfile
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": float(rows[0][2]),
                "reasons": sorted(reasons), "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


# ----------------------------------------------------------------------------------- setup
def build_shard(cfg: DecodeConfig, rank: int, world: int, dev: torch.device, seed: int = 0):
    """Codec, encoded indices (+heavy) and values of this rank's KV shard; full queries."""
    from sunshape_b200.codec import SunShapeBlockCodec
    from sunshape_b200.distributed import kv_shard_bounds

    case = make_case(cfg.with_(seq_len=min(cfg.seq_len, 8192)), device=dev, seed=seed)   # codebooks + perm
    mode = "profileperm_mixed_precision" if cfg.n_heavy else "profileperm_baseline"
    codec = SunShapeBlockCodec(cfg.head_dim, cfg.block_dim, cfg.n_centroids, mode=mode, device=dev,
                               kv_heads=cfg.kv_heads)
    codec.permutation.copy_(case["perm"])
    codec.inv_permutation.copy_(case["inv_perm"])
    codec.centroids.copy_(case["centroids"])
    codec.mixed_high_precision_blocks.copy_(case["heavy_mask"])
    codec.invalidate()
    a, b = kv_shard_bounds(cfg.seq_len, world, rank)
    Tl = b - a
    B, H, D = cfg.batch, cfg.kv_heads, cfg.head_dim
    s_c = case["channel_scale"]
    gk = torch.Generator(device=dev).manual_seed(seed + 100)
    gv = torch.Generator(device=dev).manual_seed(seed + 103)
    idx = torch.empty(B, H, Tl, cfg.n_blocks, dtype=torch.uint8, device=dev)
    heavy = None
    if cfg.n_heavy:
        heavy = torch.empty(B, H, Tl, cfg.n_heavy, cfg.block_dim, dtype=torch.bfloat16, device=dev)
    value = torch.empty(B, H, Tl, D, dtype=cfg.torch_dtype, device=dev)
    heavy_dims = case["heavy_mask"].repeat_interleave(cfg.block_dim)[case["inv_perm"]]
    for bb in range(B):
        keys = torch.randn(H, cfg.seq_len, D, generator=gk, device=dev)[:, a:b] * s_c
        if cfg.n_heavy:
            keys[..., heavy_dims] = keys[..., heavy_dims].to(torch.bfloat16).float()
        i, hv = codec.quantize_packed(keys.to(cfg.torch_dtype if cfg.n_heavy else torch.float32), kv_heads=H)
        idx[bb] = i
        if heavy is not None:
            heavy[bb] = hv
        value[bb] = torch.randn(H, cfg.seq_len, D, generator=gv, device=dev)[:, a:b].to(cfg.torch_dtype)
    query = case["query"].new_empty(B, cfg.q_heads, 1, D).copy_(
        torch.randn(B, cfg.q_heads, 1, D, generator=torch.Generator(device=dev).manual_seed(seed + 4),
                    device=dev).to(cfg.torch_dtype))
    return codec, idx, heavy, value, query, case["scale"], Tl


def algorithmic_bytes(cfg: DecodeConfig, local_tokens: int) -> int:
    """Bytes one decode launch must move: per-token rows + codebooks + queries + outputs."""
    vb = {"f32": 4, "bf16": 2, "f16": 2}[cfg.dtype]
    per_token = cfg.bytes_per_kv_token()
    consts = cfg.kv_heads * cfg.n_blocks * cfg.n_centroids * cfg.block_dim * 4 \
        + 2 * cfg.batch * cfg.q_heads * cfg.head_dim * vb
    return cfg.batch * cfg.kv_heads * local_tokens * per_token + consts


# ----------------------------------------------------------------------------------- CPU baseline
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def use_all_host_threads() -> int:
    """torchrun exports OMP_NUM_THREADS=1; the CPU baseline gets every host core explicitly."""
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


class ReferenceSample:
    """The UNMODIFIED reference package (installed into baseline/_ref) timed on the host cores.

    One sample = one sequence of the workload with all its KV heads: the reference's own
    ``_apply_quantized_attention`` (vllm_attn_backend.py:216-253, the per-(b, h) loop over
    ``sunshape_attention_scores`` -> on CPU ``_torch_attention_scores`` (dequantize + matmul), torch
    softmax and P @ V) on a ``SunShapeQuantizedKeys`` of per-head ``SunShapeQuantized`` payloads.
    The indices are seeded uniform codewords (decode time does not depend on their values) and the
    codec is the reference's one-codebook-per-layer layout.  Falls back to the numpy restatement
    of the same algorithm (``oracle/``) only if the reference cannot be imported.
    """

    def __init__(self, cfg: DecodeConfig, seed: int = 0):
        self.cfg = cfg
        self.kind = "reference"
        g = torch.Generator().manual_seed(seed)
        T, H, G, D = cfg.seq_len, cfg.kv_heads, cfg.group, cfg.head_dim
        dt = cfg.torch_dtype
        try:
            if REF_DIR not in sys.path:
                sys.path.insert(0, REF_DIR)
            from sunshape.codec import SunShapeBlockCodec, SunShapeQuantized
            from sunshape import vllm_attn_backend as rb
        except Exception as exc:   # pragma: no cover - depends on the install
            self.kind = "port"
            self.why = f"reference not importable from baseline/_ref ({exc!r})"
            return
        mode = "profileperm_mixed_precision" if cfg.n_heavy else "profileperm_baseline"
        codec = SunShapeBlockCodec(head_dim=D, block_dim=cfg.block_dim, n_centroids=cfg.n_centroids, mode=mode,
                                   device=torch.device("cpu"))
        perm = torch.randperm(D, generator=g)
        codec.permutation.copy_(perm)
        codec.inv_permutation[perm] = torch.arange(D)
        codec.centroids.copy_(torch.randn(codec.centroids.shape, generator=g))
        heavy = torch.zeros(cfg.n_blocks, dtype=torch.bool)
        heavy[:cfg.n_heavy] = True
        codec.mixed_high_precision_blocks.copy_(heavy)
        heads = []
        for _ in range(H):
            idx = torch.randint(0, cfg.n_centroids, (T, cfg.n_blocks), generator=g).to(torch.uint8)
            pv = torch.randn(T, cfg.n_blocks, cfg.block_dim, generator=g) if cfg.n_heavy else None
            heads.append(SunShapeQuantized(indices=idx, head_dim=D, block_dim=cfg.block_dim, n_blocks=cfg.n_blocks,
                                           passthrough_blocks=heavy.clone() if cfg.n_heavy else None,
                                           passthrough_values=pv))
        self.keys = rb.SunShapeQuantizedKeys(quantized_heads=tuple(heads), batch_size=1, num_kv_heads=H, seq_len=T)
        self.query = torch.randn(1, H * G, 1, D, generator=g).to(dt)
        self.value = torch.randn(1, H, T, D, generator=g).to(dt)
        self.codec, self.rb = codec, rb
        self.scale = 1.0 / (D ** 0.5)

    def limit_heads(self, n: int) -> None:
        """Shrink the per-step sample to the first n KV heads (keeps long --steps runs bounded)."""
        if self.kind != "reference" or n >= self.keys.num_kv_heads:
            return
        G = self.cfg.group
        self.keys = self.rb.SunShapeQuantizedKeys(quantized_heads=self.keys.quantized_heads[:n], batch_size=1,
                                                  num_kv_heads=n, seq_len=self.cfg.seq_len)
        self.query = self.query[:, :n * G].contiguous()
        self.value = self.value[:, :n].contiguous()

    @property
    def tokens(self) -> int:
        return (self.keys.num_kv_heads if self.kind == "reference" else 1) * self.cfg.seq_len

    @property
    def desc(self) -> str:
        c = self.cfg
        if self.kind == "reference":
            return (f"one sequence of {c.name} per step: {self.keys.num_kv_heads} KV heads x {c.seq_len} tokens, "
                    f"G={c.group}, "
                    "reference _apply_quantized_attention (baseline/_ref, torch CPU)")
        return f"one (sequence, KV head) of {c.seq_len} tokens per step, oracle port (numpy); {self.why}"

    def step(self) -> float:
        """Run one sample; return its KV tokens/s."""
        if self.kind != "reference":
            tps, _ = cpu_port_sample(self.cfg, budget_s=0.0)
            return tps
        t0 = time.perf_counter()
        self.rb._apply_quantized_attention(codec=self.codec, query=self.query, key=self.keys, value=self.value,
                                           attn_mask=None, scale=self.scale)
        return self.tokens / (time.perf_counter() - t0)


def cpu_port_sample(cfg: DecodeConfig, budget_s: float = 12.0, seed: int = 0):
    """The oracle port (numpy restatement of the reference's algorithm) on one (sequence, KV head):
    the fallback when the reference cannot be imported.  Returns (KV tokens/s, description)."""
    from oracle import sunshape_oracle as O

    T = cfg.seq_len
    rng = np.random.default_rng(seed)
    G, D, nb, bd, C = cfg.group, cfg.head_dim, cfg.n_blocks, cfg.block_dim, cfg.n_centroids
    idx = rng.integers(0, C, size=(T, nb), dtype=np.uint8)
    cents = rng.standard_normal((nb, C, bd), dtype=np.float32)
    perm = rng.permutation(D)
    inv = O.invert_permutation(perm)
    hm = np.zeros(nb, dtype=bool)
    pt = None
    if cfg.n_heavy:
        hm[:cfg.n_heavy] = True
        pt = rng.standard_normal((T, nb, bd), dtype=np.float32)
    q = O.bf16_round(rng.standard_normal((1, G, 1, D), dtype=np.float32))
    v = O.bf16_round(rng.standard_normal((1, 1, T, D), dtype=np.float32))
    heads = [(idx, hm if cfg.n_heavy else None, pt)]
    reps = 0
    t0 = time.perf_counter()
    while True:
        O.apply_quantized_attention(q, heads, v, centroids_for_head=lambda h: cents, inv_perm=inv,
                                    scale=1.0 / np.sqrt(D), query_dtype=cfg.dtype, value_dtype=cfg.dtype)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 10000:
            break
    return reps * T / el, f"{reps} x one (sequence, KV head) of {T} tokens, G={G} (oracle port, numpy)"


def cpu_baseline(cfg: DecodeConfig, budget_s: float = 12.0) -> dict:
    """cpu_baseline object for our arm's line: the reference on the host cores, bounded sample."""
    cores = use_all_host_threads()
    ref = ReferenceSample(cfg)
    ref.step()                                 # warm-up
    vals, t0 = [], time.perf_counter()
    while time.perf_counter() - t0 < budget_s or not vals:
        vals.append(ref.step())
    return {"value": statistics.median(vals), "unit": UNIT, "cores": cores, "kind": ref.kind,
            "sample": f"{len(vals)} steps of {ref.desc}"}


# ----------------------------------------------------------------------------------- timing
def time_steps(fn, steps: int, warmup: int, stream: torch.cuda.Stream, extra_events=False):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end)


class GraphStep:
    """A step captured as a CUDA graph of `per_graph` consecutive steps (every launch of every step is
    replayed: nothing is cached between steps).  Removes the host launch overhead from the device-side
    timing; falls back to eager calls if capture is not possible."""

    def __init__(self, fn, per_graph: int = 10):
        self.fn, self.per_graph, self.graph = fn, per_graph, None
        try:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for _ in range(3):
                    fn()
            torch.cuda.current_stream().wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(per_graph):
                    fn()
            torch.cuda.synchronize()
            self.graph = g
        except Exception as exc:   # pragma: no cover - depends on the runtime
            print(f"[bench] CUDA graph capture unavailable ({exc!r}); timing eager calls", file=sys.stderr)
            torch.cuda.synchronize()

    def run(self, steps: int):
        if self.graph is None:
            for _ in range(steps):
                self.fn()
            return steps
        for _ in range(max(1, steps // self.per_graph)):
            self.graph.replay()
        return max(1, steps // self.per_graph) * self.per_graph


def run_ours(args, cfg: DecodeConfig):
    from sunshape_b200 import vllm_attn_backend as vab
    from sunshape_b200.distributed import KVShardedDecode

    world, rank, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import torch.distributed as dist
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"      # keep stdout to the one JSON line
        dist.init_process_group("nccl", device_id=dev)
    codec, idx, heavy, value, query, scale, Tl = build_shard(cfg, rank, world, dev)
    keys = vab.SunShapeQuantizedKeys((), cfg.batch, cfg.kv_heads, Tl, indices=idx, heavy=heavy,
                                     passthrough_blocks=codec.mixed_high_precision_blocks if cfg.n_heavy else None,
                                     head_dim=cfg.head_dim, block_dim=cfg.block_dim)
    stream = torch.cuda.current_stream(dev)
    sharded = KVShardedDecode(codec, exchange=args.exchange) if world > 1 else None
    out = torch.empty(cfg.batch, cfg.q_heads, 1, cfg.head_dim, device=dev, dtype=value.dtype)

    if world == 1:
        def step():
            vab._apply_quantized_attention(codec=codec, query=query, key=keys, value=value, attn_mask=None,
                                           scale=scale, out=out)
        launches_per_step = 2   # lut_kernel + decode_mma_kernel
    else:
        def step():
            sharded(query, keys, value, scale=scale)
        launches_per_step = 3   # lut_kernel + decode_mma_kernel + merge / exchange kernel; NCCL not counted

    # decode kernel alone (events around the launch on its stream) for the roofline
    def kernel_only():
        if world == 1:
            vab._apply_quantized_attention(codec=codec, query=query, key=keys, value=value, attn_mask=None,
                                           scale=scale, out=out)
        else:
            sharded.partials(query, keys, value, scale=scale)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):
        step()
    g_kernel = GraphStep(kernel_only)
    g_step = GraphStep(step)
    for _ in range(max(3, args.warmup)):
        g_step.run(g_step.per_graph)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    nk = g_kernel.run(max(20, args.steps // 4))
    e1.record(stream)
    torch.cuda.synchronize()
    kernel_ms = e0.elapsed_time(e1) / nk

    sampler = ClockSampler(local)
    barrier()
    sampler.start()
    time.sleep(0.3)           # let the sampler attach before the timed region
    barrier()
    e0.record(stream)
    n_steps = g_step.run(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    t_ms = e0.elapsed_time(e1) * args.steps / n_steps
    barrier()
    # e2e through the public API: pinned host query in, host output out, every step
    from sunshape_b200.integration.vllm import runtime_state_from_bundle
    from sunshape_b200.hf import SunShapeBundle
    bundle = SunShapeBundle("synthetic", [0], 1.0, cfg.block_dim, "sunshape_base", 0, 0, 0, {0: codec}, {})
    state = runtime_state_from_bundle(bundle, device=str(dev))
    impl = vab.SunShapeAttentionImpl(layer_idx=0, runtime_state=state)
    q_host = query.cpu().pin_memory()
    o_host = torch.empty(out.shape, dtype=out.dtype).pin_memory()

    def e2e_step():
        q = q_host.to(dev, non_blocking=True)
        if world == 1:
            o = impl.forward(q, keys, value, scale=scale)
        else:
            o = sharded(q, keys, value, scale=scale)
        o_host.copy_(o, non_blocking=True)

    for _ in range(3):
        e2e_step()
    barrier()
    e2e_ms = time_steps(e2e_step, args.steps, 0, stream)
    barrier()
    clocks = sampler.stop()

    parity = None
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([t_ms, e2e_ms, kernel_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_ms, e2e_ms, kernel_ms = t.tolist()
        parity = multi_gpu_parity(args, rank, world, dev)

    total_tokens = cfg.kv_tokens()
    ms_per_step = t_ms / args.steps
    value_tps = total_tokens / (ms_per_step * 1e-3)
    e2e_tps = total_tokens / (e2e_ms / args.steps * 1e-3)
    peak, peak_kind = measured_peaks()
    alg = algorithmic_bytes(cfg, Tl)
    achieved = alg / (kernel_ms * 1e-3) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", f"decode_mma_kernel_{cfg.name}_traffic.json")
    if os.path.exists(tp):
        # DRAM bytes per algorithmic byte from one ncu capture, applied to this launch's bytes
        with open(tp) as f:
            traffic = round(alg * json.load(f)["traffic_over_algorithmic"])
    res = {
        "metric": METRIC, "value": value_tps, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded anisotropic log-normal keys, N(0,1) bf16 "
                                                       "values/queries; no dataset)",
        "config": {"workload": f"{cfg.name}: batch {cfg.batch}, {cfg.q_heads}/{cfg.kv_heads} heads, head_dim "
                               f"{cfg.head_dim}, context {cfg.seq_len}, block_dim {cfg.block_dim}, "
                               f"{cfg.n_centroids} codewords, {cfg.n_heavy} heavy blocks",
                   "global_batch": cfg.batch, "seq_len": cfg.seq_len, "parallelism": f"kv-seq-split{world}", "exchange": args.exchange if world > 1 else None,
                   "kv_tokens_per_step": total_tokens, "bytes_per_kv_token": cfg.bytes_per_kv_token(),
                   "l2": "inputs larger than L2 (no flush needed)"},
        "hbm_gbs": achieved, "query_scores_per_s": value_tps * cfg.group,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                     "kernel": "decode_mma_kernel (with its lut_kernel, overlapped by programmatic dependent launch; events around CUDA-graph replays)", "kernel_ms": kernel_ms, "algorithmic_bytes_per_launch": alg,
                     "frac_of_nominal_8tbs": achieved / 8000.0},
        "e2e": {"value": e2e_tps, "unit": UNIT, "h2d_bytes_per_step": query.numel() * query.element_size(),
                "d2h_bytes_per_step": out.numel() * out.element_size()},
        "clocks": clocks,
        "gpu_launches": args.steps * launches_per_step,
        **({"decode_ms": kernel_ms, "exchange_ms": max(0.0, ms_per_step - kernel_ms), "parity": parity}
           if world > 1 else {}),
        "timing": "device-side: CUDA-graph replay of whole steps (all launches of every step); e2e: eager public-API calls",
    }
    return res, rank, world


def multi_gpu_parity(args, rank: int, world: int, dev: torch.device) -> dict:
    """Before trusting the scaling numbers: a seeded c5-shaped case (2 sequences, 16/2 heads, ragged
    4099-token context) decoded through KVShardedDecode with this run's exchange, three calls with
    different queries, against the single-GPU fused decode of the unsharded cache on the same rank
    (the path the -m gpu tests check against the reference).  Worst per-row relative error, max over
    ranks; ok = within the bf16 output tolerance 2e-2."""
    import torch.distributed as dist
    from sunshape_b200 import vllm_attn_backend as vab
    from sunshape_b200.codec import SunShapeBlockCodec
    from sunshape_b200.distributed import KVShardedDecode, kv_shard_bounds

    cfg = CONFIGS["c5"].with_(batch=2, kv_heads=2, q_heads=16, seq_len=4099)
    case = make_case(cfg, device=dev, seed=17)
    codec = SunShapeBlockCodec(cfg.head_dim, cfg.block_dim, cfg.n_centroids, device=dev, kv_heads=cfg.kv_heads)
    codec.permutation.copy_(case["perm"])
    codec.inv_permutation.copy_(case["inv_perm"])
    codec.centroids.copy_(case["centroids"])
    codec.invalidate()
    qk = vab.quantize_codec_keys(codec, case["keys"])
    a, b = kv_shard_bounds(cfg.seq_len, world, rank)
    shard = vab.SunShapeQuantizedKeys((), cfg.batch, cfg.kv_heads, b - a, indices=qk.indices[:, :, a:b].contiguous())
    v = case["value"][:, :, a:b].contiguous()
    dec = KVShardedDecode(codec, exchange=args.exchange)
    worst = 0.0
    for call in range(3):
        q = case["query"] * (1.0 + 0.25 * call)
        ref = vab._apply_quantized_attention(codec=codec, query=q, key=qk, value=case["value"], attn_mask=None,
                                             scale=case["scale"]).float()
        out = dec(q, shard, v, scale=case["scale"]).float()
        err = ((out - ref).abs().amax(-1) / ref.abs().amax(-1).clamp_min(1e-30)).max().item()
        worst = max(worst, err if err == err else float("inf"))
    torch.cuda.synchronize()
    dist.barrier()
    dec.close()
    t = torch.tensor([worst], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    worst = float(t.item())
    return {"max_rel_err_per_row": worst, "ok": worst <= 2e-2, "calls": 3,
            "against": "single-GPU fused decode of the unsharded cache", "case": "c5-shaped B2 16/2 heads T4099"}


def run_extra_configs(args):
    """N=1 figures for the other decode configs and the c3 encode path (parity configs; informational)."""
    from sunshape_b200 import vllm_attn_backend as vab

    dev = torch.device("cuda", 0)
    peak, _ = measured_peaks()
    extra = {}
    for name in ("c2", "c3", "c4", "c5_fp32_lut", "c2_bd2"):
        if name == "c5_fp32_lut":      # the headline shape with fp32 LUT entries (fewer pipeline stages)
            cfg = CONFIGS["c5"]
            os.environ["SUNSHAPE_LUT_FP32"] = "1"
        elif name == "c2_bd2":         # block_dim 2: the reference's default 4 bits/dim, 64 blocks per head
            cfg = CONFIGS["c2"].with_(block_dim=2)
        else:
            cfg = CONFIGS[name]
        codec, idx, heavy, value, query, scale, Tl = build_shard(cfg, 0, 1, dev)
        keys = vab.SunShapeQuantizedKeys((), cfg.batch, cfg.kv_heads, Tl, indices=idx, heavy=heavy,
                                         passthrough_blocks=codec.mixed_high_precision_blocks if cfg.n_heavy else None)
        out = torch.empty(cfg.batch, cfg.q_heads, 1, cfg.head_dim, device=dev, dtype=value.dtype)

        def step():
            vab._apply_quantized_attention(codec=codec, query=query, key=keys, value=value, attn_mask=None,
                                           scale=scale, out=out)
        n = 100
        ms = time_steps(step, n, 5, torch.cuda.current_stream(dev)) / n
        alg = algorithmic_bytes(cfg, Tl)
        os.environ.pop("SUNSHAPE_LUT_FP32", None)
        extra[name] = {"kv_tokens_per_s": cfg.kv_tokens() / (ms * 1e-3), "ms_per_step": ms,
                       "hbm_gbs": alg / (ms * 1e-3) / 1e9, "frac": alg / (ms * 1e-3) / 1e9 / peak}
        if name == "c3":
            # encode: append 16384 fp32 keys per (sequence, KV head)
            kk = torch.randn(cfg.batch, cfg.kv_heads, cfg.seq_len, cfg.head_dim, device=dev)
            ms_e = time_steps(lambda: codec.quantize_packed(kk, kv_heads=cfg.kv_heads), 5, 2,
                              torch.cuda.current_stream(dev)) / 5
            nkeys = kk.shape[0] * kk.shape[1] * kk.shape[2]
            byt = nkeys * (cfg.head_dim * 4 + cfg.n_blocks)
            extra["c3_encode"] = {"keys_per_s": nkeys / (ms_e * 1e-3), "ms": ms_e, "hbm_gbs": byt / (ms_e * 1e-3) / 1e9,
                                  "argmin_compares_per_s": nkeys * cfg.n_blocks * cfg.n_centroids / (ms_e * 1e-3),
                                  "kernel": "encode_tc_kernel (fp32 keys, 3xTF32 on tcgen05, TMA key tiles)"}
            # bf16 keys (what a model hands the encoder): the tcgen05 kernel, 3 tf32 MMAs per block
            kb = kk.to(torch.bfloat16)
            del kk
            ms_b = time_steps(lambda: codec.quantize_packed(kb, kv_heads=cfg.kv_heads), 5, 2,
                              torch.cuda.current_stream(dev)) / 5
            kw = 16 if 2 * cfg.block_dim + 3 <= 16 else 32     # MMA K per block (tf32 words)
            flops = 2.0 * nkeys * cfg.n_blocks * cfg.n_centroids * kw
            extra["c3_encode_bf16"] = {"keys_per_s": nkeys / (ms_b * 1e-3), "ms": ms_b,
                                       "hbm_gbs": nkeys * (cfg.head_dim * 2 + cfg.n_blocks) / (ms_b * 1e-3) / 1e9,
                                       "argmin_compares_per_s": nkeys * cfg.n_blocks * cfg.n_centroids / (ms_b * 1e-3),
                                       "tf32_tflops": flops / (ms_b * 1e-3) / 1e12,
                                       "kernel": "encode_tc_kernel (bf16 keys on tcgen05, TMA key tiles)"}
            del kb
        del codec, idx, heavy, value, query, keys, out
        torch.cuda.empty_cache()
    return extra


def run_reference(args, cfg: DecodeConfig):
    """--impl reference: the unmodified reference's CPU decode path on the host cores (rank 0 only)."""
    world, rank, _ = dist_env()
    if rank != 0:
        return None
    cores = use_all_host_threads()
    ref = ReferenceSample(cfg)
    t_full = ref.tokens / ref.step()           # seconds per full sample
    per_head = t_full / max(1, cfg.kv_heads)
    budget = 150.0                             # whole --steps + --warmup run within a few minutes
    ref.limit_heads(max(1, min(cfg.kv_heads, int(budget / max(args.steps + args.warmup, 1) / per_head))))
    for _ in range(args.warmup):
        ref.step()
    t0 = time.perf_counter()
    per_step = [ref.step() for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    v = args.steps * ref.tokens / wall if ref.kind == "reference" else statistics.median(per_step)
    return {
        "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": wall / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": cfg.dtype, "data": "synthetic", "impl": "reference",
        "config": {"workload": cfg.name, "global_batch": cfg.batch, "seq_len": cfg.seq_len,
                   "parallelism": f"cpu, {cores} threads",
                   "sample_kv_tokens_per_step": ref.tokens if ref.kind == "reference" else cfg.seq_len,
                   "note": "each step is a bounded sample (one sequence) of the workload; value = KV tokens/s"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": ref.kind, "sample": ref.desc},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="c5", choices=sorted(CONFIGS))
    ap.add_argument("--no-extra", action="store_true", help="skip the N=1 figures for the other configs")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--seq-len", type=int, default=0,
                    help="override the workload's context length (small cases for profiler captures)")
    ap.add_argument("--exchange", choices=["nccl", "peer", "p2p"], default="nccl",
                    help="N>1 merge: NCCL all-gather + merge kernel; peer-memory stores from the decode kernel; or "
                         "one exchange kernel pushing partials over NVLink and merging (p2p)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    cfg = CONFIGS[args.workload]
    if args.seq_len:
        cfg = cfg.with_(seq_len=args.seq_len)

    if args.impl == "reference":
        res = run_reference(args, cfg)
        if res is not None:
            print(json.dumps(res))
        return

    res, rank, world = run_ours(args, cfg)
    if world == 1:
        if not args.no_cpu:
            res["cpu_baseline"] = cpu_baseline(cfg, budget_s=12.0)
        if not args.no_extra:
            res["other_configs_n1"] = run_extra_configs(args)
    if rank == 0:
        print(json.dumps(res))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
