"""KV-sequence split of SunShape decode attention across GPUs (one process per GPU).

The reference keeps the whole KV cache on one device and has no distributed code;
long contexts here are sharded along the sequence: rank r owns tokens
``[start_r, end_r)`` of every (sequence, KV head) -- indices, heavy blocks and
values -- while codebooks, the permutation and the queries are replicated.  Each
rank runs the fused decode kernel over its shard and emits unnormalised softmax
partials ``(m, l, acc)`` per query row; ONE collective (an all-gather of the
packed fp32 partials over NCCL / NVLink) brings every rank's partials to every
rank, and a merge kernel combines them in a fixed rank order, so all ranks hold
the identical final output:

    M = max_r m_r,   L = sum_r l_r e^(m_r - M),   O = sum_r acc_r e^(m_r - M) / L.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .vllm_attn_backend import SunShapeQuantizedKeys, _apply_quantized_attention, decode_partials


def kv_shard_bounds(seq_len: int, world_size: int, rank: int) -> tuple[int, int]:
    """Even contiguous split of ``seq_len`` tokens; the first ``seq_len % world_size`` ranks get one extra."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("bad world_size / rank")
    base, rem = divmod(int(seq_len), int(world_size))
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def shard_mask(attn_mask: torch.Tensor | None, start: int, end: int) -> torch.Tensor | None:
    return None if attn_mask is None else attn_mask[..., start:end]


def gather_partials(partials: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather [rows, 2 + Dv] fp32 partials into [world, rows, 2 + Dv] (the only collective)."""
    world = dist.get_world_size(group)
    out = torch.empty((world * partials.shape[0], *partials.shape[1:]), dtype=partials.dtype,
                      device=partials.device)
    dist.all_gather_into_tensor(out, partials.contiguous(), group=group)   # concatenated form (NCCL and gloo)
    return out.view(world, *partials.shape)


def merge_gathered(gathered: torch.Tensor, out_shape, out_dtype) -> torch.Tensor:
    """Merge [world, rows, 2 + Dv] partials on the GPU (fixed rank order)."""
    Dv = gathered.shape[-1] - 2
    out = torch.empty(gathered.shape[1], Dv, device=gathered.device, dtype=out_dtype)
    _lib.merge_partials(gathered.contiguous(), out)
    return out.view(*out_shape)


class PeerGroup:
    """One exchange buffer per rank, mapped into every rank's process (CUDA IPC), for the fused
    cross-GPU merge: the decode kernel stores its rank-local results straight into the peers'
    buffers over NVLink (see ``sunshape_decode_attention_peers``)."""

    def __init__(self, nbytes: int, device: torch.device, group=None):
        lib = _lib.load_library()
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world > 8:
            raise RuntimeError("the peer exchange supports at most 8 ranks")
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        with torch.cuda.device(device):
            _lib._check(lib.sunshape_peer_alloc(int(nbytes), ctypes.byref(own), handle))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._own, self._opened = own.value, []
        bufs = []
        with torch.cuda.device(device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    bufs.append(own.value)
                    continue
                hb = (ctypes.c_char * 64).from_buffer_copy(h)
                pp = ctypes.c_void_p()
                _lib._check(lib.sunshape_peer_open(hb, ctypes.byref(pp)))
                bufs.append(pp.value)
                self._opened.append(pp.value)
        self.desc = _lib.PeerGroupDesc(self.rank, self.world, (ctypes.c_void_p * 8)(*(bufs + [None] * (8 - len(bufs)))))
        self.device = device

    def close(self):
        lib = _lib.load_library()
        with torch.cuda.device(self.device):
            for pp in self._opened:
                lib.sunshape_peer_close(ctypes.c_void_p(pp))
            if self._own:
                lib.sunshape_peer_free(ctypes.c_void_p(self._own))
        self._opened, self._own = [], None


class KVShardedDecode:
    """Decode attention over a KV cache whose sequence is split across the ranks of ``group``.

    ``exchange="nccl"`` (default): partials, one NCCL all-gather, merge kernel.
    ``exchange="p2p"`` (CUDA, at most 8 ranks): partials, then ONE exchange kernel per rank that pushes
    them into every rank's exchange buffer over NVLink (16-byte peer stores, per-slice flags) and merges
    all ranks' rows as soon as they land (``sunshape_exchange_merge``); no library collective.
    ``exchange="peer"`` (CUDA, 16-bit values, at most 8 ranks): ranks write their per-head results
    straight into every peer's exchange buffer from inside the decode kernel (CUDA IPC mappings,
    NVLink stores, system-scope arrival counters), then one merge kernel per rank combines them; no
    library collective.  On 8 B200s at the c5 shape it measured 131 us per step against 120 us for
    the NCCL path, so it is opt-in.
    """

    def __init__(self, codec, group=None, exchange: str = "nccl"):
        self.codec = codec
        self.group = group
        self.exchange = exchange
        self._partials = None
        self._peers: dict = {}

    def partials(self, query, key: SunShapeQuantizedKeys, value, attn_mask=None, scale=None) -> torch.Tensor:
        B, Hq, L, _ = query.shape
        Dv = value.shape[-1]
        shape = (B * Hq * L, 2 + Dv)
        if self._partials is None or self._partials.shape != shape or self._partials.device != query.device:
            self._partials = torch.empty(shape, device=query.device, dtype=torch.float32)
        return decode_partials(codec=self.codec, query=query, key=key, value=value, attn_mask=attn_mask,
                               scale=scale, partials=self._partials)

    def _p2p_group(self, query, value) -> "PeerGroup | None":
        if self.exchange != "p2p" or not query.is_cuda or dist.get_world_size(self.group) > 8:
            return None
        B, Hq, L, _ = query.shape
        Dv = value.shape[-1]
        key = ("p2p", B * Hq * L, Dv, query.device)
        pg = self._peers.get(key)
        if pg is None:
            nbytes = _lib.load_library().sunshape_exchange_buffer_bytes(dist.get_world_size(self.group),
                                                                        B * Hq * L, Dv)
            pg = self._peers[key] = PeerGroup(nbytes, query.device, self.group)
        return pg

    def _peer_group(self, query, value) -> "PeerGroup | None":
        if self.exchange != "peer" or not query.is_cuda or value.dtype == torch.float32:
            return None
        B, Hq, L, _ = query.shape
        Hkv, Dv = value.shape[1], value.shape[-1]
        if (Hq // Hkv) * L > 16 or dist.get_world_size(self.group) > 8:
            return None
        key = (B * Hq * L, Dv, B * Hkv, query.device)
        pg = self._peers.get(key)
        if pg is None:
            nbytes = _lib.load_library().sunshape_peer_buffer_bytes(dist.get_world_size(self.group), B * Hq * L, Dv,
                                                                    B * Hkv)
            pg = self._peers[key] = PeerGroup(nbytes, query.device, self.group)
        return pg

    def forward(self, query, key: SunShapeQuantizedKeys, value, attn_mask=None, scale=None) -> torch.Tensor:
        """Rank-local shard in, full merged output [B, Hq, L, Dv] (value dtype) out, on every rank."""
        pg = self._peer_group(query, value)
        if pg is not None:
            return _apply_quantized_attention(codec=self.codec, query=query, key=key, value=value,
                                              attn_mask=attn_mask, scale=scale, peer_group=pg.desc)
        part = self.partials(query, key, value, attn_mask, scale)
        B, Hq, L, _ = query.shape
        x = self._p2p_group(query, value)
        if x is not None:
            out = torch.empty(B, Hq, L, value.shape[-1], device=query.device, dtype=value.dtype)
            _lib.exchange_merge(part, out.view(B * Hq * L, -1), x.desc)
            return out
        gathered = gather_partials(part, self.group)
        return merge_gathered(gathered, (B, Hq, L, value.shape[-1]), value.dtype)

    __call__ = forward

    def close(self) -> None:
        """Unmap the peers' exchange buffers and free this rank's.  Every rank must have finished its
        last decode first (a barrier), since peers store into this rank's buffer during a decode."""
        for pg in self._peers.values():
            pg.close()
        self._peers.clear()
