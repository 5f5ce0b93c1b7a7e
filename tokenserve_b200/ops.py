"""ctypes bindings of the C ABI (``include/tokenserve_b200.h``) with torch-tensor wrappers.

The wrappers only translate tensors into pointers, sizes and the current CUDA stream; all
compute happens in the CUDA kernels of ``libtokenserve_b200.so``. There is no fallback: if the
library is missing or a call fails, a :class:`KernelError` is raised.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtokenserve_b200.so"
ABI_VERSION = 1

TS_FLOAT32, TS_FLOAT16, TS_BFLOAT16 = 0, 1, 2
TS_ERR_INVALID_ARGUMENT, TS_ERR_UNSUPPORTED, TS_ERR_WORKSPACE, TS_ERR_MISALIGNED = -1, -2, -3, -4
DTYPE_CODES = {torch.float32: TS_FLOAT32, torch.float16: TS_FLOAT16, torch.bfloat16: TS_BFLOAT16}

_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ts_version": (ctypes.c_int, []),
    "ts_last_error": (ctypes.c_char_p, []),
    "ts_reshape_and_cache": (
        ctypes.c_int,
        [_p, _p, _i64, _i64, _p, _p, _p, _i64, _i32, _i32, _i32, _i64, _i32, _p, _p, _p, _p],
    ),
    "ts_paged_decode_workspace_size": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32, _i32]),
    "ts_paged_decode": (
        ctypes.c_int,
        [_p, _p, _i64, _p, _p, _p, _i32, _p, _i32, _i32, _i32, _i32, _i32, _i64, _f32, _i32,
         _p, _sz, _p],
    ),
    "ts_paged_decode_planned": (
        ctypes.c_int,
        [_p, _p, _i64, _p, _p, _p, _i32, _p, _i32, _i32, _i32, _i32, _i32, _i64, _f32, _i32,
         _p, _sz, _p],
    ),
    "ts_paged_prefill": (
        ctypes.c_int,
        [_p, _p, _i64, _p, _p, _p, _i32, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
         _i64, _f32, _i32, _p],
    ),
    "ts_copy_blocks": (ctypes.c_int, [_p, _i64, _i64, _i64, _i64, _p, _i64, _p, _p]),
    "ts_verify_tags": (ctypes.c_int, [_p, _p, _i32, _p, _p, _p, _i32, _i32, _i64, _p, _p]),
    "ts_swap_blocks": (
        ctypes.c_int, [_p, _i64, _i64, _p, _i64, _i64, _i64, _i64, _p, _i64, _p, _p]
    ),
    "ts_paged_decode_peer": (
        ctypes.c_int,
        [_p, _i32, _i32, _p, ctypes.c_uint32, _p, _i64, _p, _p, _p, _i32, _p, _i32, _i32, _i32,
         _i32, _i32, _i64, _f32, _i32, _p, ctypes.c_size_t, _i32, _p],
    ),
    "ts_paged_decode_publish": (
        ctypes.c_int,
        [_p, _i32, _i32, _p, ctypes.c_uint32, _p, _i64, _p, _p, _p, _i32, _p, _i32, _i32, _i32,
         _i32, _i32, _i64, _f32, _i32, _p, ctypes.c_size_t, _i32, _p],
    ),
    "ts_gather_peers": (
        ctypes.c_int, [_p, _i32, _i32, _p, ctypes.c_uint32, _i32, _i32, _i32, _i32, _p, _p]
    ),
    "ts_wait_peers": (ctypes.c_int, [_p, _i32, ctypes.c_uint32, _p, _p]),
    "ts_peer_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "ts_peer_free": (ctypes.c_int, [_p]),
    "ts_ipc_get_handle": (ctypes.c_int, [_p, _p]),
    "ts_ipc_open": (ctypes.c_int, [_p, ctypes.POINTER(ctypes.c_void_p)]),
    "ts_ipc_close": (ctypes.c_int, [_p]),
    "ts_add_rmsnorm": (ctypes.c_int, [_p, _p, _p, _p, _i64, _i32, _f32, _i32, _p]),
    "ts_rope_and_cache": (
        ctypes.c_int,
        [_p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i32, _i32, _i32, _i32, _i64, _i32, _p, _p],
    ),
    "ts_silu_mul": (ctypes.c_int, [_p, _p, _i64, _i32, _i32, _p]),
}

_lib: ctypes.CDLL | None = None
_lock = threading.Lock()


class KernelError(RuntimeError):
    """A tokenserve_b200 kernel call was rejected or failed to launch."""


def load_library() -> ctypes.CDLL:
    """Loads (once) and returns the kernel library; raises if it was not built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise KernelError(
                f"{LIB_PATH} is missing; build it with `python -m tokenserve_b200._build` "
                "(there is no CPU fallback)"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.ts_version() != ABI_VERSION:
            raise KernelError(f"ABI version {lib.ts_version()} != {ABI_VERSION}")
        _lib = lib
        return lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def _check(code: int, what: str) -> None:
    if code != 0:
        msg = load_library().ts_last_error().decode(errors="replace")
        raise KernelError(f"{what} failed (status {code}): {msg}")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dtype(t: torch.Tensor) -> int:
    try:
        return DTYPE_CODES[t.dtype]
    except KeyError:
        raise KernelError(f"unsupported dtype {t.dtype}") from None


def _rows(t: torch.Tensor, heads: int, head_dim: int, what: str) -> int:
    """Token stride (elements) of a [tokens, heads, head_dim] view with contiguous rows."""
    if t.dim() != 3 or t.shape[1] != heads or t.shape[2] != head_dim:
        raise KernelError(f"{what}: expected [tokens, {heads}, {head_dim}], got {tuple(t.shape)}")
    if t.stride(2) != 1 or t.stride(1) != head_dim:
        raise KernelError(f"{what}: heads and head_dim must be contiguous")
    return t.stride(0)


def _pool_dims(pool: torch.Tensor) -> tuple[int, int, int, int]:
    if pool.dim() != 4 or not pool.is_contiguous():
        raise KernelError("KV pool must be a contiguous [num_blocks, kv_heads, block_size, head_dim]")
    nb, h, bs, d = pool.shape
    return nb, h, bs, d


def reshape_and_cache(
    key: torch.Tensor,
    value: torch.Tensor,
    key_pool: torch.Tensor,
    value_pool: torch.Tensor,
    slot_mapping: torch.Tensor,
    *,
    token_tags: torch.Tensor | None = None,
    tag_pool: torch.Tensor | None = None,
    error_flag: torch.Tensor | None = None,
) -> None:
    """K1: ``key/value [T, Hkv, D]`` -> pools at ``slot_mapping [T]`` (int64)."""
    nb, h, bs, d = _pool_dims(key_pool)
    if value_pool.shape != key_pool.shape or value_pool.dtype != key_pool.dtype:
        raise KernelError("key and value pools differ")
    if key.dtype != key_pool.dtype or value.dtype != key_pool.dtype:
        raise KernelError("K/V rows must have the pool's dtype")
    ks = _rows(key, h, d, "key")
    vs = _rows(value, h, d, "value")
    if slot_mapping.dtype != torch.int64 or slot_mapping.numel() != key.shape[0]:
        raise KernelError("slot_mapping must be int64 with one entry per token")
    code = load_library().ts_reshape_and_cache(
        _ptr(key), _ptr(value), ks, vs, _ptr(key_pool), _ptr(value_pool),
        _ptr(slot_mapping), key.shape[0], h, d, bs, nb, _dtype(key_pool),
        _ptr(token_tags), _ptr(tag_pool), _ptr(error_flag), _stream(),
    )  # fmt: skip
    _check(code, "reshape_and_cache")


def decode_workspace_size(
    batch: int, num_q_heads: int, num_kv_heads: int, head_dim: int, max_blocks: int,
    block_size: int, dtype: torch.dtype,
) -> int:  # fmt: skip
    return int(
        load_library().ts_paged_decode_workspace_size(
            batch, num_q_heads, num_kv_heads, head_dim, max_blocks, block_size, DTYPE_CODES[dtype]
        )
    )


def paged_decode(
    out: torch.Tensor,
    query: torch.Tensor,
    key_pool: torch.Tensor,
    value_pool: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    scale: float,
    workspace: torch.Tensor | None,
    reuse_plan: bool = False,
) -> None:
    """K2: ``query [B, Hq, D]`` over each sequence's context -> ``out [B, Hq, D]``.

    ``reuse_plan=True`` runs the work plan an earlier call left in ``workspace`` (same block
    tables, context lengths, batch, KV heads and table width: the later layers of one decode
    step) and skips the prep kernel (``ts_paged_decode_planned``).
    """
    nb, hkv, bs, d = _pool_dims(key_pool)
    hq = query.shape[1]
    qs = _rows(query, hq, d, "query")
    if not out.is_contiguous() or out.shape != (query.shape[0], hq, d):
        raise KernelError("out must be a contiguous [B, Hq, D]")
    if block_tables.dtype != torch.int32 or not block_tables.is_contiguous():
        raise KernelError("block_tables must be contiguous int32 [B, max_blocks]")
    if context_lens.dtype != torch.int32:
        raise KernelError("context_lens must be int32")
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    lib = load_library()
    fn = lib.ts_paged_decode_planned if reuse_plan else lib.ts_paged_decode
    code = fn(
        _ptr(out), _ptr(query), qs, _ptr(key_pool), _ptr(value_pool), _ptr(block_tables),
        block_tables.shape[1], _ptr(context_lens), query.shape[0], hq, hkv, d, bs, nb,
        float(scale), _dtype(key_pool), _ptr(workspace), ws_bytes, _stream(),
    )  # fmt: skip
    _check(code, "paged_decode")


def paged_prefill(
    out: torch.Tensor,
    query: torch.Tensor,
    key_pool: torch.Tensor,
    value_pool: torch.Tensor,
    block_tables: torch.Tensor,
    query_start_loc: torch.Tensor,
    context_lens: torch.Tensor,
    max_query_len: int,
    scale: float,
) -> None:
    """K3: causal chunk attention, ``query [T, Hq, D]`` -> ``out [T, Hq, D]``."""
    nb, hkv, bs, d = _pool_dims(key_pool)
    hq = query.shape[1]
    qs = _rows(query, hq, d, "query")
    if not out.is_contiguous() or out.shape != (query.shape[0], hq, d):
        raise KernelError("out must be a contiguous [T, Hq, D]")
    if block_tables.dtype != torch.int32 or not block_tables.is_contiguous():
        raise KernelError("block_tables must be contiguous int32")
    if query_start_loc.dtype != torch.int32 or context_lens.dtype != torch.int32:
        raise KernelError("query_start_loc and context_lens must be int32")
    code = load_library().ts_paged_prefill(
        _ptr(out), _ptr(query), qs, _ptr(key_pool), _ptr(value_pool), _ptr(block_tables),
        block_tables.shape[1], _ptr(query_start_loc), _ptr(context_lens),
        context_lens.shape[0], query.shape[0], int(max_query_len), hq, hkv, d, bs, nb,
        float(scale), _dtype(key_pool), _stream(),
    )  # fmt: skip
    _check(code, "paged_prefill")


def copy_blocks(
    planes: torch.Tensor, src_dst: torch.Tensor, error_flag: torch.Tensor | None = None
) -> None:
    """K4: ``planes [P, num_blocks, ...]`` (contiguous); copy each (src, dst) block in every plane."""
    if not planes.is_contiguous() or planes.dim() < 2:
        raise KernelError("planes must be a contiguous [P, num_blocks, ...] tensor")
    if src_dst.dtype != torch.int64 or not src_dst.is_contiguous():
        raise KernelError("src_dst must be contiguous int64 [n, 2]")
    if not planes.is_cuda or src_dst.device != planes.device:
        raise KernelError("planes and src_dst must be on the same CUDA device")
    es = planes.element_size()
    block_bytes = planes[0, 0].numel() * es
    code = load_library().ts_copy_blocks(
        _ptr(planes), planes.shape[0], planes.stride(0) * es, block_bytes, planes.shape[1],
        _ptr(src_dst), src_dst.numel() // 2, _ptr(error_flag), _stream(),
    )  # fmt: skip
    _check(code, "copy_blocks")


def swap_blocks(dst: torch.Tensor, src: torch.Tensor, src_dst: torch.Tensor,
                error_flag: torch.Tensor | None = None) -> None:  # fmt: skip
    """K4 between two arenas ``[P, blocks, ...]`` of one plane layout: ``dst[p, d] = src[p, s]``
    for each pair ``(s, d)``. One side may be pinned host memory (swap-out / swap-in)."""
    for t in (dst, src):
        if not t.is_contiguous() or t.dim() < 2:
            raise KernelError("swap_blocks: arenas must be contiguous [P, blocks, ...] tensors")
        if not t.is_cuda and not t.is_pinned():
            raise KernelError("swap_blocks: a host arena must be pinned memory")
    if dst.shape[0] != src.shape[0] or dst[0, 0].numel() * dst.element_size() != (
            src[0, 0].numel() * src.element_size()):  # fmt: skip
        raise KernelError("swap_blocks: arenas differ in planes or block size")
    if src_dst.dtype != torch.int64 or not src_dst.is_contiguous() or not src_dst.is_cuda:
        raise KernelError("swap_blocks: src_dst must be contiguous int64 [n, 2] on the device")
    bb = dst[0, 0].numel() * dst.element_size()
    code = load_library().ts_swap_blocks(
        _ptr(dst), dst.stride(0) * dst.element_size(), dst.shape[1],
        _ptr(src), src.stride(0) * src.element_size(), src.shape[1],
        dst.shape[0], bb, _ptr(src_dst), src_dst.numel() // 2, _ptr(error_flag), _stream(),
    )  # fmt: skip
    _check(code, "swap_blocks")


def verify_tags(
    tag_pool: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    expected_offsets: torch.Tensor,
    expected_tokens: torch.Tensor,
    block_size: int,
    mismatch_pos: torch.Tensor,
) -> None:
    """Device shadow-KV read-back check; ``mismatch_pos[b]`` = first bad position or -1."""
    num_blocks = tag_pool.numel() // block_size
    code = load_library().ts_verify_tags(
        _ptr(tag_pool), _ptr(block_tables), block_tables.shape[1], _ptr(context_lens),
        _ptr(expected_offsets), _ptr(expected_tokens), context_lens.shape[0], block_size,
        num_blocks, _ptr(mismatch_pos), _stream(),
    )  # fmt: skip
    _check(code, "verify_tags")


def add_rmsnorm(out: torch.Tensor, residual: torch.Tensor, x: torch.Tensor | None,
                weight: torch.Tensor, eps: float) -> None:  # fmt: skip
    """``residual += x`` (skipped when ``x`` is None), then ``out = RMSNorm(residual) * weight``."""
    rows, hidden = residual.shape
    for t in (out, residual, weight) + (() if x is None else (x,)):
        if not t.is_contiguous() or t.dtype != residual.dtype:
            raise KernelError("add_rmsnorm: tensors must be contiguous and of one dtype")
    code = load_library().ts_add_rmsnorm(_ptr(out), _ptr(residual), _ptr(x), _ptr(weight), rows,
                                         hidden, float(eps), _dtype(residual), _stream())  # fmt: skip
    _check(code, "add_rmsnorm")


def rope_and_cache(qkv: torch.Tensor, q_out: torch.Tensor, key_pool: torch.Tensor,
                   value_pool: torch.Tensor, slot_mapping: torch.Tensor, positions: torch.Tensor,
                   inv_freq: torch.Tensor, num_q_heads: int, num_kv_heads: int,
                   error_flag: torch.Tensor | None = None) -> None:  # fmt: skip
    """RoPE on q and k of fused ``qkv [T, (Hq + 2 Hkv) * D]``; q -> ``q_out``, k/v -> the pool."""
    nb, hkv, bs, d = _pool_dims(key_pool)
    if hkv != num_kv_heads or qkv.stride(1) != 1 or not q_out.is_contiguous():
        raise KernelError("rope_and_cache: bad layout")
    if slot_mapping.dtype != torch.int64 or positions.dtype != torch.int64:
        raise KernelError("rope_and_cache: slot_mapping and positions must be int64")
    code = load_library().ts_rope_and_cache(
        _ptr(qkv), qkv.stride(0), _ptr(q_out), _ptr(key_pool), _ptr(value_pool),
        _ptr(slot_mapping), _ptr(positions), _ptr(inv_freq), qkv.shape[0], num_q_heads,
        num_kv_heads, d, bs, nb, _dtype(key_pool), _ptr(error_flag), _stream(),
    )  # fmt: skip
    _check(code, "rope_and_cache")


def silu_mul(out: torch.Tensor, gate_up: torch.Tensor) -> None:
    """``out = silu(gate) * up`` for ``gate_up = [gate | up]`` of shape ``[T, 2 I]``."""
    rows, two_i = gate_up.shape
    if not gate_up.is_contiguous() or not out.is_contiguous() or out.shape != (rows, two_i // 2):
        raise KernelError("silu_mul: bad layout")
    code = load_library().ts_silu_mul(_ptr(out), _ptr(gate_up), rows, two_i // 2,
                                      _dtype(gate_up), _stream())  # fmt: skip
    _check(code, "silu_mul")
