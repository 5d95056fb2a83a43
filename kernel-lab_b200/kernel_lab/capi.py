"""ctypes binding of the C ABI in ``include/kernel_lab_b200.h`` (libkernel_lab_b200.so).

This is the boundary a non-PyTorch host (or kernel-lab's own C++ launcher callers)
binds. Tensors are passed as raw device pointers; PyTorch is used here only to
allocate device memory and to name the current stream.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

import torch

LIB_PATH = Path(__file__).with_name("libkernel_lab_b200.so")

KL_FLOAT32, KL_FLOAT16, KL_BFLOAT16 = 0, 1, 2
KL_STATUS_BAD_PAGE, KL_STATUS_LEN_CLAMPED, KL_STATUS_WAIT_TIMEOUT = 1, 2, 4
DTYPE_CODES = {torch.float32: KL_FLOAT32, torch.float16: KL_FLOAT16, torch.bfloat16: KL_BFLOAT16}

_c_int, _c_i64, _c_float, _c_vp, _c_sz = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t
_c_i32p = ctypes.POINTER(ctypes.c_int32)
_c_szp = ctypes.POINTER(ctypes.c_size_t)
_c_u32p = ctypes.POINTER(ctypes.c_uint32)

# Exported symbol -> (restype, argtypes); the same list as the header declares.
SIGNATURES = {
    "kl_version": (ctypes.c_char_p, []),
    "kl_status_string": (ctypes.c_char_p, [_c_int]),
    "kl_rms_norm": (_c_int, [_c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_i64, _c_float, _c_vp]),
    "kl_paged_decode_workspace_size": (
        _c_int,
        [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_szp, _c_szp],
    ),
    "kl_paged_decode": (
        _c_int,
        [_c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_i64, _c_int,
         _c_i64, _c_float, _c_int, _c_vp, _c_sz, _c_vp, _c_sz, _c_vp],
    ),
    "kl_paged_decode_attention": (
        _c_int,
        [_c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_i64, _c_float,
         _c_vp],
    ),
    "kl_paged_decode_read_status": (_c_int, [_c_vp, _c_u32p, _c_int, _c_vp]),
    "kl_paged_kv_append": (
        _c_int,
        [_c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_i64, _c_int, _c_i64,
         _c_i64, _c_vp, _c_vp],
    ),
    "kl_paged_decode_fp8": (
        _c_int,
        [_c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_int,
         _c_i64, _c_int, _c_i64, _c_float, _c_int, _c_vp, _c_sz, _c_vp, _c_sz, _c_vp],
    ),
    "kl_paged_kv_append_fp8": (
        _c_int,
        [_c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_i64,
         _c_int, _c_i64, _c_i64, _c_vp, _c_vp],
    ),
    "kl_paged_decode_cascade_workspace_size": (
        _c_int,
        [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_szp, _c_szp],
    ),
    "kl_paged_decode_cascade": (
        _c_int,
        [_c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_i64, _c_int, _c_vp, _c_vp,
         _c_int, _c_int, _c_int, _c_int, _c_int, _c_i64, _c_int, _c_i64, _c_float, _c_vp, _c_sz, _c_vp, _c_sz, _c_vp],
    ),
    "kl_paged_decode_noalloc": (
        _c_int,
        [_c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_i64, _c_int,
         _c_i64, _c_float, _c_int, _c_vp],
    ),
    "kl_paged_decode_noalloc_read_status": (_c_int, [_c_u32p, _c_int, _c_vp]),
    "kl_paged_decode_gather": (
        _c_int,
        [_c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_i64, _c_int,
         _c_i64, _c_float, _c_vp, _c_sz, _c_vp, _c_sz, _c_vp],
    ),
    "kl_ipc_alloc": (_c_int, [_c_sz, ctypes.POINTER(_c_vp), _c_vp]),
    "kl_ipc_open": (_c_int, [_c_vp, ctypes.POINTER(_c_vp)]),
    "kl_ipc_close": (_c_int, [_c_vp]),
    "kl_ipc_free": (_c_int, [_c_vp]),
}

KL_STATUS_PEER_TIMEOUT = 16
KL_GATHER_MAX_RANKS = 8
KL_IPC_HANDLE_BYTES = 64


class HeadGather(ctypes.Structure):
    """kl_head_gather_t: one call's head gather (ranks, epoch, every rank's output and flags)."""

    _fields_ = [
        ("num_ranks", ctypes.c_int),
        ("rank", ctypes.c_int),
        ("epoch", ctypes.c_uint32),
        ("out", ctypes.c_void_p * KL_GATHER_MAX_RANKS),
        ("flags", ctypes.c_void_p * KL_GATHER_MAX_RANKS),
        ("done", ctypes.c_void_p),
        ("timeout_ms", ctypes.c_uint32),
    ]

_lib: ctypes.CDLL | None = None


class KernelLabError(RuntimeError):
    def __init__(self, what: str, status: int):
        super().__init__(f"kernel_lab: {what} failed: {status_string(status)} (status {status})")
        self.status = status


def load() -> ctypes.CDLL:
    """Load the library once and declare every entry point's signature."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH.name} is not built; run `python kernel-lab_b200/build.py`")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def version() -> str:
    return load().kl_version().decode()


def status_string(status: int) -> str:
    return load().kl_status_string(status).decode()


def _check(status: int, what: str) -> None:
    if status != 0:
        raise KernelLabError(what, status)


def _stream(stream: torch.cuda.Stream | None) -> int:
    s = torch.cuda.current_stream() if stream is None else stream
    return s.cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def rms_norm(
    out: torch.Tensor,
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    residual: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """kl_rms_norm on torch tensors (x: [rows, hidden] with a contiguous last dim)."""
    x2 = x.reshape(-1, x.shape[-1])
    _check(
        load().kl_rms_norm(
            DTYPE_CODES[x.dtype], _ptr(out), _ptr(x2), _ptr(residual), _ptr(weight), x2.shape[0], x2.shape[1],
            x2.stride(0), eps, _stream(stream),
        ),
        "kl_rms_norm",
    )


def workspace_size(
    dtype: torch.dtype, batch: int, num_q_heads: int, num_kv_heads: int, head_dim: int, page_size: int,
    max_pages: int, num_splits: int = 0,
) -> tuple[int, int]:
    pb, sb = ctypes.c_size_t(0), ctypes.c_size_t(0)
    _check(
        load().kl_paged_decode_workspace_size(
            DTYPE_CODES[dtype], batch, num_q_heads, num_kv_heads, head_dim, page_size, max_pages, num_splits,
            ctypes.byref(pb), ctypes.byref(sb),
        ),
        "kl_paged_decode_workspace_size",
    )
    return pb.value, sb.value


@dataclass
class DecodeScratch:
    """Caller-owned scratch for kl_paged_decode: partials (uninitialised) and sync (zeroed)."""

    partials: torch.Tensor
    sync: torch.Tensor

    @classmethod
    def for_problem(cls, q: torch.Tensor, k_cache: torch.Tensor, block_table: torch.Tensor, num_splits: int = 0):
        batch, hq, d = q.shape
        _, page, hkv, _ = k_cache.shape
        pb, sb = workspace_size(q.dtype, batch, hq, hkv, d, page, block_table.shape[1], num_splits)
        return cls(
            partials=torch.empty(max(pb, 256), dtype=torch.uint8, device=q.device),
            sync=torch.zeros(max(sb, 256), dtype=torch.uint8, device=q.device),
        )

    def status(self, clear: bool = False, stream: torch.cuda.Stream | None = None) -> int:
        value = ctypes.c_uint32(0)
        _check(
            load().kl_paged_decode_read_status(_ptr(self.sync), ctypes.byref(value), int(clear), _stream(stream)),
            "kl_paged_decode_read_status",
        )
        return value.value


def paged_decode(
    out: torch.Tensor,
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float | None = None,
    num_splits: int = 0,
    scratch: DecodeScratch | None = None,
    stream: torch.cuda.Stream | None = None,
) -> DecodeScratch:
    """kl_paged_decode on torch tensors; returns the scratch used (reuse it across calls)."""
    batch, hq, d = q.shape
    num_pages, page, hkv, _ = k_cache.shape
    if scratch is None:
        scratch = DecodeScratch.for_problem(q, k_cache, block_table, num_splits)
    scale = d**-0.5 if scale is None else scale
    _check(
        load().kl_paged_decode(
            DTYPE_CODES[q.dtype], _ptr(out), _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(block_table),
            _ptr(seq_lens), batch, hq, hkv, d, page, block_table.stride(0), block_table.shape[1], num_pages, scale,
            num_splits, _ptr(scratch.partials), scratch.partials.numel(), _ptr(scratch.sync), scratch.sync.numel(),
            _stream(stream),
        ),
        "kl_paged_decode",
    )
    return scratch


def paged_decode_attention(
    out: torch.Tensor,
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float | None = None,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """kl_paged_decode_attention: kernel-lab's launcher argument list (stream-ordered scratch)."""
    batch, hq, d = q.shape
    _, page, hkv, _ = k_cache.shape
    scale = d**-0.5 if scale is None else scale
    _check(
        load().kl_paged_decode_attention(
            DTYPE_CODES[q.dtype], _ptr(out), _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(block_table),
            _ptr(seq_lens), batch, hq, hkv, d, page, block_table.stride(0), scale, _stream(stream),
        ),
        "kl_paged_decode_attention",
    )


def paged_kv_append(
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    k_new: torch.Tensor,
    v_new: torch.Tensor,
    block_table: torch.Tensor,
    positions: torch.Tensor,
    status: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """kl_paged_kv_append on torch tensors; ``status`` is an optional int32/uint32 device word."""
    batch = k_new.shape[0]
    num_pages, page, hkv, d = k_cache.shape
    _check(
        load().kl_paged_kv_append(
            DTYPE_CODES[k_cache.dtype], _ptr(k_cache), _ptr(v_cache), _ptr(k_new), _ptr(v_new), _ptr(block_table),
            _ptr(positions), batch, hkv, d, page, block_table.stride(0), block_table.shape[1], num_pages,
            k_new.stride(0), _ptr(status), _stream(stream),
        ),
        "kl_paged_kv_append",
    )


def paged_decode_fp8(
    out: torch.Tensor,
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    k_scale: torch.Tensor,
    v_scale: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float | None = None,
    num_splits: int = 0,
    scratch: DecodeScratch | None = None,
    stream: torch.cuda.Stream | None = None,
) -> DecodeScratch:
    """kl_paged_decode_fp8 on torch tensors (caches of torch.float8_e4m3fn or uint8 codes)."""
    batch, hq, d = q.shape
    num_pages, page, hkv, _ = k_cache.shape
    if scratch is None:
        scratch = DecodeScratch.for_problem(q, k_cache, block_table, num_splits)
    scale = d**-0.5 if scale is None else scale
    _check(
        load().kl_paged_decode_fp8(
            DTYPE_CODES[q.dtype], _ptr(out), _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(k_scale), _ptr(v_scale),
            _ptr(block_table), _ptr(seq_lens), batch, hq, hkv, d, page, block_table.stride(0), block_table.shape[1],
            num_pages, scale, num_splits, _ptr(scratch.partials), scratch.partials.numel(), _ptr(scratch.sync),
            scratch.sync.numel(), _stream(stream),
        ),
        "kl_paged_decode_fp8",
    )
    return scratch


def paged_kv_append_fp8(
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    k_new: torch.Tensor,
    v_new: torch.Tensor,
    k_scale: torch.Tensor,
    v_scale: torch.Tensor,
    block_table: torch.Tensor,
    positions: torch.Tensor,
    status: torch.Tensor | None = None,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """kl_paged_kv_append_fp8 on torch tensors."""
    batch = k_new.shape[0]
    num_pages, page, hkv, d = k_cache.shape
    _check(
        load().kl_paged_kv_append_fp8(
            DTYPE_CODES[k_new.dtype], _ptr(k_cache), _ptr(v_cache), _ptr(k_new), _ptr(v_new), _ptr(k_scale),
            _ptr(v_scale), _ptr(block_table), _ptr(positions), batch, hkv, d, page, block_table.stride(0),
            block_table.shape[1], num_pages, k_new.stride(0), _ptr(status), _stream(stream),
        ),
        "kl_paged_kv_append_fp8",
    )


def paged_decode_cascade(
    out: torch.Tensor,
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    prefix_block_table: torch.Tensor,
    prefix_lens: torch.Tensor,
    prefix_indptr: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float | None = None,
    k_scale: torch.Tensor | None = None,
    v_scale: torch.Tensor | None = None,
    scratch: DecodeScratch | None = None,
    stream: torch.cuda.Stream | None = None,
) -> DecodeScratch:
    """kl_paged_decode_cascade on torch tensors (e4m3 caches when k_scale / v_scale are given);
    returns the scratch used."""
    batch, hq, d = q.shape
    num_pages, page, hkv, _ = k_cache.shape
    groups = prefix_lens.numel()
    if scratch is None:
        pb, sb = ctypes.c_size_t(0), ctypes.c_size_t(0)
        _check(
            load().kl_paged_decode_cascade_workspace_size(
                DTYPE_CODES[q.dtype], batch, groups, hq, hkv, d, page, block_table.shape[1],
                prefix_block_table.shape[1], ctypes.byref(pb), ctypes.byref(sb),
            ),
            "kl_paged_decode_cascade_workspace_size",
        )
        scratch = DecodeScratch(
            partials=torch.empty(max(pb.value, 256), dtype=torch.uint8, device=q.device),
            sync=torch.zeros(max(sb.value, 256), dtype=torch.uint8, device=q.device),
        )
    scale = d**-0.5 if scale is None else scale
    _check(
        load().kl_paged_decode_cascade(
            DTYPE_CODES[q.dtype], _ptr(out), _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(k_scale), _ptr(v_scale),
            _ptr(prefix_block_table), _ptr(prefix_lens), _ptr(prefix_indptr), groups, prefix_block_table.stride(0),
            prefix_block_table.shape[1], _ptr(block_table), _ptr(seq_lens), batch, hq, hkv, d, page,
            block_table.stride(0), block_table.shape[1], num_pages, scale, _ptr(scratch.partials),
            scratch.partials.numel(), _ptr(scratch.sync), scratch.sync.numel(), _stream(stream),
        ),
        "kl_paged_decode_cascade",
    )
    return scratch


def paged_decode_gather(
    gather: HeadGather,
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    scale: float | None = None,
    scratch: DecodeScratch | None = None,
    stream: torch.cuda.Stream | None = None,
) -> DecodeScratch:
    """kl_paged_decode_gather: this rank's KV-head shard, its heads stored into every rank's output."""
    batch, hq, d = q.shape
    num_pages, page, hkv, _ = k_cache.shape
    if scratch is None:
        scratch = DecodeScratch.for_problem(q, k_cache, block_table)
    scale = d**-0.5 if scale is None else scale
    _check(
        load().kl_paged_decode_gather(
            DTYPE_CODES[q.dtype], ctypes.byref(gather), _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(block_table),
            _ptr(seq_lens), batch, hq, hkv, d, page, block_table.stride(0), block_table.shape[1], num_pages, scale,
            _ptr(scratch.partials), scratch.partials.numel(), _ptr(scratch.sync), scratch.sync.numel(),
            _stream(stream),
        ),
        "kl_paged_decode_gather",
    )
    return scratch


def ipc_alloc(nbytes: int) -> tuple[int, bytes]:
    """Zeroed device memory on the current device that peers can map: (pointer, handle bytes)."""
    ptr = ctypes.c_void_p(0)
    handle = ctypes.create_string_buffer(KL_IPC_HANDLE_BYTES)
    _check(load().kl_ipc_alloc(nbytes, ctypes.byref(ptr), handle), "kl_ipc_alloc")
    return int(ptr.value), handle.raw


def ipc_open(handle: bytes) -> int:
    """Map a peer's kl_ipc_alloc buffer into this process (current device); returns its address here."""
    if len(handle) != KL_IPC_HANDLE_BYTES:
        raise ValueError(f"an IPC handle has {KL_IPC_HANDLE_BYTES} bytes, not {len(handle)}")
    ptr = ctypes.c_void_p(0)
    buf = ctypes.create_string_buffer(handle, KL_IPC_HANDLE_BYTES)
    _check(load().kl_ipc_open(buf, ctypes.byref(ptr)), "kl_ipc_open")
    return int(ptr.value)


def ipc_close(ptr: int) -> None:
    _check(load().kl_ipc_close(ptr), "kl_ipc_close")


def ipc_free(ptr: int) -> None:
    _check(load().kl_ipc_free(ptr), "kl_ipc_free")


class _DeviceArray:
    """A raw device buffer described by the CUDA array interface (torch.as_tensor wraps it without a copy)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 2,
                                         "strides": None}


def device_tensor(ptr: int, shape: tuple[int, ...], dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A tensor view of `shape` over device memory at `ptr` (not owned: the memory must outlive it)."""
    typestr = {torch.float32: "<f4", torch.float16: "<f2", torch.bfloat16: "<i2"}[dtype]
    t = torch.as_tensor(_DeviceArray(ptr, tuple(shape), typestr), device=device)
    return t.view(dtype) if dtype == torch.bfloat16 else t
