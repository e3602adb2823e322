"""ctypes binding of ``libsunshape_b200.so`` (the C ABI in ``include/sunshape_b200.h``).

Tensors cross the boundary as raw device pointers plus sizes; every call runs on
the current torch CUDA stream of the tensors' device.  There is no CPU path:
CPU tensors, a missing library or an unsupported shape raise ``RuntimeError``
with the reason, in the style of the reference's fast-path gate
(``sunshape/triton_kernels.py:327-373``).
"""
from __future__ import annotations

import ctypes
import math
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsunshape_b200.so")

F32, BF16, F16, U8, I16, I32 = 0, 1, 2, 3, 4, 5
_DTYPE_CODE = {
    torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16,
    torch.uint8: U8, torch.int16: I16, torch.int32: I32,
}

EXPORTED_SYMBOLS = (
    "sunshape_abi_version", "sunshape_last_error", "sunshape_encode", "sunshape_dequantize",
    "sunshape_attention_scores", "sunshape_decode_workspace_bytes", "sunshape_decode_attention",
    "sunshape_merge_partials", "sunshape_decode_attention_noalloc", "sunshape_peer_buffer_bytes",
    "sunshape_peer_alloc", "sunshape_peer_open", "sunshape_peer_close", "sunshape_peer_free",
    "sunshape_decode_attention_peers", "sunshape_decode_workspace_min_bytes", "sunshape_encode_error",
    "sunshape_decode_attention_noalloc_error", "sunshape_exchange_buffer_bytes", "sunshape_exchange_merge",
    "sunshape_exchange_error", "sunshape_index_row_bytes", "sunshape_pack_indices",
    "sunshape_attention_scores_packed",
)


class CodecDesc(ctypes.Structure):
    _fields_ = [
        ("centroids", ctypes.c_void_p),
        ("permutation", ctypes.c_void_p),
        ("heavy_mask", ctypes.c_void_p),
        ("n_cb", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("block_dim", ctypes.c_int32),
        ("n_centroids", ctypes.c_int32),
        ("n_heavy", ctypes.c_int32),
        ("centroid_norm_max", ctypes.c_void_p),
    ]


class KVDesc(ctypes.Structure):
    _fields_ = [
        ("indices", ctypes.c_void_p),
        ("index_dtype", ctypes.c_int32),
        ("heavy", ctypes.c_void_p),
        ("heavy_dtype", ctypes.c_int32),
        ("value", ctypes.c_void_p),
        ("value_dtype", ctypes.c_int32),
        ("value_dim", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("head_stride", ctypes.c_int64),
    ]


class PeerGroupDesc(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int32), ("world", ctypes.c_int32), ("buffers", ctypes.c_void_p * 8)]


_lib = None
_lock = threading.Lock()


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and type the C ABI.  Raises if the library was not built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"sunshape_b200 CUDA library not found at {path}; build it with `python -m sunshape_b200.build`."
            )
        lib = ctypes.CDLL(path)
        vp, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
        pc, pk = ctypes.POINTER(CodecDesc), ctypes.POINTER(KVDesc)
        lib.sunshape_abi_version.restype = ctypes.c_int
        lib.sunshape_last_error.restype = ctypes.c_char_p
        lib.sunshape_encode.argtypes = [pc, vp, i32, i32, i32, i32, i64, i64, vp, i32, vp, i32, i64, vp]
        lib.sunshape_dequantize.argtypes = [pc, pk, i32, i32, vp, vp]
        lib.sunshape_attention_scores.argtypes = [pc, pk, vp, i32, i32, i32, i32, f32, vp, vp]
        lib.sunshape_decode_workspace_bytes.argtypes = [i32, i32, i32, i32, i32]
        lib.sunshape_decode_workspace_bytes.restype = ctypes.c_int64
        lib.sunshape_decode_attention.argtypes = [pc, pk, vp, i32, i32, i32, i32, i32, vp, i32, i64, i64, i64,
                                                  f32, vp, i32, vp, vp, i64, vp]
        lib.sunshape_decode_workspace_min_bytes.argtypes = [i32, i32, i32, i32]
        lib.sunshape_decode_workspace_min_bytes.restype = ctypes.c_int64
        lib.sunshape_encode_error.argtypes = [ctypes.POINTER(ctypes.c_int32), i32]
        lib.sunshape_encode_error.restype = ctypes.c_int
        lib.sunshape_decode_attention_noalloc_error.argtypes = [ctypes.POINTER(ctypes.c_int32)]
        lib.sunshape_decode_attention_noalloc_error.restype = ctypes.c_int
        lib.sunshape_exchange_buffer_bytes.argtypes = [i32, i64, i32]
        lib.sunshape_exchange_buffer_bytes.restype = ctypes.c_int64
        lib.sunshape_exchange_merge.argtypes = [vp, i64, i32, ctypes.POINTER(PeerGroupDesc), vp, i32, vp]
        lib.sunshape_exchange_merge.restype = ctypes.c_int
        lib.sunshape_exchange_error.argtypes = [vp, i32, i64, i32, ctypes.POINTER(ctypes.c_int32)]
        lib.sunshape_exchange_error.restype = ctypes.c_int
        lib.sunshape_index_row_bytes.argtypes = [i32, i32]
        lib.sunshape_index_row_bytes.restype = ctypes.c_int64
        lib.sunshape_pack_indices.argtypes = [vp, i64, i32, i32, vp, vp]
        lib.sunshape_pack_indices.restype = ctypes.c_int
        lib.sunshape_attention_scores_packed.argtypes = [pc, vp, i32, i32, i64, vp, i32, i32, i32, i32, vp, vp]
        lib.sunshape_attention_scores_packed.restype = ctypes.c_int
        lib.sunshape_merge_partials.argtypes = [vp, i32, i64, i32, vp, i32, vp]
        lib.sunshape_decode_attention_noalloc.argtypes = [pc, pk, vp, i32, i32, i32, i32, i32, vp, i32, i64, i64,
                                                          i64, f32, vp, i32, vp, vp]
        lib.sunshape_decode_attention_noalloc.restype = ctypes.c_int
        lib.sunshape_peer_buffer_bytes.argtypes = [i32, i64, i32, i32]
        lib.sunshape_peer_buffer_bytes.restype = ctypes.c_int64
        lib.sunshape_peer_alloc.argtypes = [i64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
        lib.sunshape_peer_open.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
        lib.sunshape_peer_close.argtypes = [vp]
        lib.sunshape_peer_free.argtypes = [vp]
        for name in ("sunshape_peer_alloc", "sunshape_peer_open", "sunshape_peer_close", "sunshape_peer_free",
                     "sunshape_decode_attention_peers"):
            getattr(lib, name).restype = ctypes.c_int
        lib.sunshape_decode_attention_peers.argtypes = [pc, pk, vp, i32, i32, i32, i32, i32, vp, i32, i64, i64, i64,
                                                        f32, vp, i32, ctypes.POINTER(PeerGroupDesc), vp, i64, vp]
        for name in ("sunshape_encode", "sunshape_dequantize", "sunshape_attention_scores",
                     "sunshape_decode_attention", "sunshape_merge_partials"):
            getattr(lib, name).restype = ctypes.c_int
        if lib.sunshape_abi_version() != 1:
            raise RuntimeError("sunshape_b200 library ABI version mismatch; rebuild it.")
        _lib = lib
        return lib


def _check(rc: int) -> None:
    if rc != 0:
        msg = load_library().sunshape_last_error().decode(errors="replace")
        raise RuntimeError(msg or f"sunshape_b200 call failed with status {rc}")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {t.dtype} at the sunshape_b200 boundary") from None


def require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "sunshape_b200 runs only on CUDA tensors (B200, sm_100a); there is no CPU fallback."
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError("all sunshape_b200 inputs must live on the same CUDA device.")
    if dev is None:
        raise RuntimeError("sunshape_b200 call without any CUDA tensor.")
    return dev


def aligned16(t: torch.Tensor | None) -> torch.Tensor | None:
    """Return t, or a fresh (16-byte aligned) contiguous copy if its data pointer is not 16-byte aligned."""
    if t is None or t.data_ptr() % 16 == 0:
        return t
    return t.clone(memory_format=torch.contiguous_format)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def codec_desc(centroids: torch.Tensor, perm: torch.Tensor, heavy_mask: torch.Tensor | None,
               n_heavy: int, head_dim: int, block_dim: int, norm_max: torch.Tensor | None = None) -> CodecDesc:
    """centroids [n_cb, nb, C, bd] fp32 contiguous, perm int64 [D], heavy_mask uint8 [nb] or None,
    norm_max [n_cb] fp32 (max centroid norm per codebook) or None."""
    return CodecDesc(ptr(centroids), ptr(perm), ptr(heavy_mask), int(centroids.shape[0]), int(head_dim),
                     int(block_dim), int(centroids.shape[2]), int(n_heavy), ptr(norm_max))


def kv_desc(indices: torch.Tensor, heavy: torch.Tensor | None, value: torch.Tensor | None, seq_len: int,
            head_stride: int, value_dim: int = 0) -> KVDesc:
    return KVDesc(ptr(indices), dtype_code(indices), ptr(heavy), dtype_code(heavy) if heavy is not None else BF16,
                  ptr(value), dtype_code(value) if value is not None else F32, int(value_dim), int(seq_len),
                  int(head_stride))


def encode(cd: CodecDesc, keys: torch.Tensor, n_heads: int, kv_heads: int, n_tokens: int, key_head_stride: int,
           key_token_stride: int, indices_out: torch.Tensor, heavy_out: torch.Tensor | None,
           out_head_stride: int) -> None:
    dev = require_cuda(keys, indices_out, heavy_out)
    lib = load_library()
    with torch.cuda.device(dev):
        _check(lib.sunshape_encode(
            ctypes.byref(cd), ptr(keys), dtype_code(keys), n_heads, kv_heads, n_tokens, key_head_stride,
            key_token_stride, ptr(indices_out), dtype_code(indices_out), ptr(heavy_out),
            dtype_code(heavy_out) if heavy_out is not None else BF16, out_head_stride, stream_ptr(dev)))


def dequantize(cd: CodecDesc, kd: KVDesc, n_heads: int, kv_heads: int, out: torch.Tensor) -> None:
    dev = require_cuda(out)
    with torch.cuda.device(dev):
        _check(load_library().sunshape_dequantize(ctypes.byref(cd), ctypes.byref(kd), n_heads, kv_heads, ptr(out),
                                                  stream_ptr(dev)))


def attention_scores(cd: CodecDesc, kd: KVDesc, query: torch.Tensor, n_heads: int, kv_heads: int, rows: int,
                     scale: float | None, out: torch.Tensor) -> None:
    dev = require_cuda(query, out)
    with torch.cuda.device(dev):
        _check(load_library().sunshape_attention_scores(
            ctypes.byref(cd), ctypes.byref(kd), ptr(query), dtype_code(query), n_heads, kv_heads, rows,
            math.nan if scale is None else float(scale), ptr(out), stream_ptr(dev)))


_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def decode_workspace(dev: torch.device, n_heads: int, seq_len: int, rows: int, value_dim: int,
                     n_blocks: int) -> torch.Tensor:
    """Zero-initialised workspace cached per (device, stream); the kernels leave the tickets zeroed."""
    if os.environ.get("SUNSHAPE_DECODE_LUT") == "cta":     # per-head LUTs built in each CTA (minimum workspace)
        need = int(load_library().sunshape_decode_workspace_min_bytes(n_heads, seq_len, rows, value_dim))
    else:
        need = int(load_library().sunshape_decode_workspace_bytes(n_heads, seq_len, rows, value_dim, n_blocks))
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), stream_ptr(dev))
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(need, dtype=torch.uint8, device=dev)
        _workspaces[key] = ws
    return ws[:need]


def decode_error_word(dev: torch.device | None = None) -> int:
    """First device-side error code recorded by decode kernels on this device (0 = none)."""
    codes = [int(ws[:4].view(torch.int32).item()) for (d, _), ws in _workspaces.items()
             if dev is None or d == (dev.index or 0)]
    return next((c for c in codes if c), 0)


def encode_error_word(dev: torch.device, clear: bool = True) -> int:
    """Device error code recorded by the encode kernels on ``dev`` (0 = none); waits for the device."""
    code = ctypes.c_int32(0)
    with torch.cuda.device(dev):
        _check(load_library().sunshape_encode_error(ctypes.byref(code), 1 if clear else 0))
    return int(code.value)


def decode_workspace_min_bytes(n_heads: int, seq_len: int, rows: int, value_dim: int) -> int:
    """Smallest workspace the decode accepts (per-head LUTs built inside each CTA)."""
    return int(load_library().sunshape_decode_workspace_min_bytes(n_heads, seq_len, rows, value_dim))


def decode_attention(cd: CodecDesc, kd: KVDesc, query: torch.Tensor, batch: int, q_heads: int, kv_heads: int,
                     query_len: int, mask: torch.Tensor | None, mask_strides: tuple[int, int, int],
                     scale: float | None, out: torch.Tensor | None, partials: torch.Tensor | None,
                     workspace: torch.Tensor | None = None) -> None:
    dev = require_cuda(query, out, partials, mask)
    lib = load_library()
    with torch.cuda.device(dev):
        if workspace is None:
            workspace = decode_workspace(dev, batch * kv_heads, kd.seq_len, (q_heads // kv_heads) * query_len,
                                         kd.value_dim, cd.head_dim // cd.block_dim)
        _check(lib.sunshape_decode_attention(
            ctypes.byref(cd), ctypes.byref(kd), ptr(query), dtype_code(query), batch, q_heads, kv_heads, query_len,
            ptr(mask), dtype_code(mask) if mask is not None else F32, *mask_strides,
            math.nan if scale is None else float(scale), ptr(out), dtype_code(out) if out is not None else F32,
            ptr(partials), ptr(workspace), workspace.numel(), stream_ptr(dev)))


def merge_partials(parts: torch.Tensor, out: torch.Tensor) -> None:
    """parts [n_parts, rows, 2 + Dv] fp32 -> out [rows, Dv]."""
    dev = require_cuda(parts, out)
    with torch.cuda.device(dev):
        _check(load_library().sunshape_merge_partials(
            ptr(parts), int(parts.shape[0]), int(parts.shape[1]), int(parts.shape[2] - 2), ptr(out),
            dtype_code(out), stream_ptr(dev)))


def decode_attention_peers(cd: CodecDesc, kd: KVDesc, query: torch.Tensor, batch: int, q_heads: int, kv_heads: int,
                           query_len: int, mask: torch.Tensor | None, mask_strides: tuple[int, int, int],
                           scale: float | None, out: torch.Tensor, group: PeerGroupDesc) -> None:
    dev = require_cuda(query, out, mask)
    lib = load_library()
    with torch.cuda.device(dev):
        ws = decode_workspace(dev, batch * kv_heads, kd.seq_len, (q_heads // kv_heads) * query_len, kd.value_dim,
                              cd.head_dim // cd.block_dim)
        _check(lib.sunshape_decode_attention_peers(
            ctypes.byref(cd), ctypes.byref(kd), ptr(query), dtype_code(query), batch, q_heads, kv_heads, query_len,
            ptr(mask), dtype_code(mask) if mask is not None else F32, *mask_strides,
            math.nan if scale is None else float(scale), ptr(out), dtype_code(out), ctypes.byref(group), ptr(ws),
            ws.numel(), stream_ptr(dev)))


def exchange_merge(parts: torch.Tensor, out: torch.Tensor, group: PeerGroupDesc) -> None:
    """parts [rows, 2 + Dv] fp32 (this rank's) -> out [rows, Dv] merged over every rank of ``group``."""
    dev = require_cuda(parts, out)
    with torch.cuda.device(dev):
        _check(load_library().sunshape_exchange_merge(ptr(parts), int(parts.shape[0]), int(parts.shape[1] - 2),
                                                      ctypes.byref(group), ptr(out), dtype_code(out),
                                                      stream_ptr(dev)))


def pack_indices(indices: torch.Tensor, bits: int) -> torch.Tensor:
    """uint8 indices [..., n_blocks] -> packed uint8 rows [..., ceil(n_blocks * bits / 8)]."""
    dev = require_cuda(indices)
    nb = int(indices.shape[-1])
    lib = load_library()
    rb = int(lib.sunshape_index_row_bytes(bits, nb))
    idx = indices.contiguous()
    out = torch.empty(*idx.shape[:-1], rb, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _check(lib.sunshape_pack_indices(ptr(idx), idx.numel() // nb, nb, bits, ptr(out), stream_ptr(dev)))
    return out


def attention_scores_packed(cd: CodecDesc, indices: torch.Tensor, index_bits: int, seq_len: int, head_stride: int,
                            query: torch.Tensor, n_heads: int, kv_heads: int, rows: int, out: torch.Tensor) -> None:
    dev = require_cuda(indices, query, out)
    with torch.cuda.device(dev):
        _check(load_library().sunshape_attention_scores_packed(
            ctypes.byref(cd), ptr(indices), index_bits, seq_len, head_stride, ptr(query), dtype_code(query), n_heads,
            kv_heads, rows, ptr(out), stream_ptr(dev)))
