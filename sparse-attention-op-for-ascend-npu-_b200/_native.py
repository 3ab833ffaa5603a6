"""ctypes binding of libtpsa.so (the C ABI declared in include/tpsa.h).

The library is built in-tree by ``build.py``.  Nothing here falls back to a
CPU or PyTorch implementation: if the library is missing, every call raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libtpsa.so"
# TPSA_ABI_VERSION of the header this binding follows (include/tpsa.h).
ABI_VERSION = 3
ADAPTER_PATH = PKG_DIR / "_tpsa_torch.so"

TPSA_OK = 0
STATUS_NAMES = {
    0: "TPSA_OK",
    1: "TPSA_ERR_INVALID_ARGUMENT",
    2: "TPSA_ERR_WORKSPACE",
    3: "TPSA_ERR_CUDA",
    4: "TPSA_ERR_UNSUPPORTED_DEVICE",
    5: "TPSA_ERR_DEVICE_FAULT",
}
DEVICE_WAIT_TIMEOUT = 0x1
DEVICE_BAD_PAGE = 0x2

# Every symbol include/tpsa.h declares.
EXPORTED_SYMBOLS = (
    "tpsa_abi_version",
    "tpsa_status_string",
    "tpsa_last_error",
    "tpsa_make_plan",
    "tpsa_plan_item",
    "tpsa_plan_tile",
    "tpsa_workspace_size",
    "tpsa_paged_attention",
    "tpsa_paged_attention_heads",
    "tpsa_paged_attention_visit",
    "tpsa_device_status",
    "tpsa_paged_attention_static_scratch",
    "tpsa_varlen_workspace_size",
    "tpsa_paged_attention_varlen",
    "tpsa_varlen_workspace_size_heads",
    "tpsa_paged_attention_varlen_heads",
    "tpsa_debug_wait_probe",
    "tpsa_dense_workspace_size",
    "tpsa_paged_attention_dense",
)


class Plan(ctypes.Structure):
    _fields_ = [
        ("query_tokens", ctypes.c_int32),
        ("query_start", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("sparse_begin", ctypes.c_int32),
        ("sparse_end", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("num_blocks", ctypes.c_int32),
        ("tail_block0", ctypes.c_int32),
        ("tail_items", ctypes.c_int32),
        ("total_items", ctypes.c_int32),
        ("split_tiles", ctypes.c_int32),
        ("grid", ctypes.c_int32),
        ("workspace_bytes", ctypes.c_int64),
        ("total_tiles", ctypes.c_int64),
        ("scale", ctypes.c_float),
        ("scale_log2", ctypes.c_float),
    ]


class Item(ctypes.Structure):
    _fields_ = [
        ("block", ctypes.c_int32),
        ("kv_head", ctypes.c_int32),
        ("split", ctypes.c_int32),
        ("num_splits", ctypes.c_int32),
        ("tile_begin", ctypes.c_int32),
        ("tile_end", ctypes.c_int32),
    ]


class TpsaError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None

_i32, _i64, _u64, _f32, _vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_float, ctypes.c_void_p
_ATTN = [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _f32]


def lib() -> ctypes.CDLL:
    """Load libtpsa.so once (raises if it has not been built)."""
    global _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing; build it with build.py")
        h = ctypes.CDLL(str(LIB_PATH))
        h.tpsa_abi_version.restype = _i32
        found = h.tpsa_abi_version()
        if found != ABI_VERSION:
            raise RuntimeError(f"{LIB_PATH} has ABI version {found}, this binding expects "
                               f"{ABI_VERSION}; rebuild it with build.py")
        h.tpsa_status_string.argtypes = [ctypes.c_int]
        h.tpsa_status_string.restype = ctypes.c_char_p
        h.tpsa_last_error.restype = ctypes.c_char_p
        h.tpsa_make_plan.argtypes = [_i64, _i64, _i64, _i64, _i32, _i32, _f32, ctypes.POINTER(Plan)]
        h.tpsa_plan_item.argtypes = [ctypes.POINTER(Plan), _i32, ctypes.POINTER(Item)]
        h.tpsa_plan_tile.argtypes = [ctypes.POINTER(Plan), _i32, _i32, ctypes.POINTER(_i32),
                                     ctypes.POINTER(_i32), ctypes.POINTER(_i32),
                                     ctypes.POINTER(_i32)]
        h.tpsa_workspace_size.argtypes = [_i64, _i64, _i64, _i64, ctypes.POINTER(_u64)]
        h.tpsa_paged_attention.argtypes = _ATTN + [_vp, _u64, _vp]
        h.tpsa_paged_attention_heads.argtypes = _ATTN + [_i32, _vp, _u64, _vp]
        h.tpsa_paged_attention_visit.argtypes = _ATTN + [_i32, _vp, _u64, _vp, _vp, _vp]
        h.tpsa_device_status.argtypes = [_i32, ctypes.POINTER(ctypes.c_uint32)]
        h.tpsa_debug_wait_probe.argtypes = [ctypes.c_uint32]
        h.tpsa_dense_workspace_size.argtypes = [_i64, _i64, _i64, ctypes.POINTER(_u64)]
        h.tpsa_paged_attention_dense.argtypes = [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                                 _i64, _f32, _vp, _u64, _vp]
        h.tpsa_paged_attention_static_scratch.argtypes = _ATTN + [_vp]
        _p64 = ctypes.POINTER(_i64)
        h.tpsa_varlen_workspace_size.argtypes = [_i32, _p64, _p64, _p64, ctypes.POINTER(_u64)]
        h.tpsa_paged_attention_varlen.argtypes = [_vp, _vp, _vp, _vp, _vp, _i32, _p64, _p64, _p64,
                                                  _i64, _i64, _f32, _vp, _u64, _vp]
        h.tpsa_varlen_workspace_size_heads.argtypes = [_i32, _p64, _p64, _p64, _i32,
                                                       ctypes.POINTER(_u64)]
        h.tpsa_paged_attention_varlen_heads.argtypes = [_vp, _vp, _vp, _vp, _vp, _i32, _p64, _p64,
                                                        _p64, _i64, _i64, _f32, _i32, _vp, _u64,
                                                        _vp]
        for name in ("tpsa_make_plan", "tpsa_plan_item", "tpsa_plan_tile", "tpsa_workspace_size",
                     "tpsa_paged_attention", "tpsa_paged_attention_heads",
                     "tpsa_paged_attention_visit", "tpsa_device_status",
                     "tpsa_paged_attention_static_scratch", "tpsa_varlen_workspace_size",
                     "tpsa_paged_attention_varlen", "tpsa_varlen_workspace_size_heads",
                     "tpsa_paged_attention_varlen_heads", "tpsa_debug_wait_probe",
                     "tpsa_dense_workspace_size", "tpsa_paged_attention_dense"):
            getattr(h, name).restype = ctypes.c_int
        _LIB = h
        return h


def check(status: int) -> None:
    if status != TPSA_OK:
        msg = lib().tpsa_last_error().decode() or lib().tpsa_status_string(status).decode()
        raise TpsaError(status, msg)


def make_plan(query_tokens: int, query_start: int, seq_len: int, prompt_len: int,
              kv_heads: int = 8, sm_count: int = 0, scale: float = 128 ** -0.5) -> Plan:
    plan = Plan()
    check(lib().tpsa_make_plan(query_tokens, query_start, seq_len, prompt_len, kv_heads, sm_count,
                               scale, ctypes.byref(plan)))
    return plan


def plan_item(plan: Plan, item: int) -> Item:
    out = Item()
    check(lib().tpsa_plan_item(ctypes.byref(plan), item, ctypes.byref(out)))
    return out


def plan_tile(plan: Plan, block: int, tile: int) -> tuple[int, int, bool, int]:
    """(first key, key count, needs mask, first key of keys 64-127)."""
    k0, w, up, m = _i32(), _i32(), _i32(), _i32()
    check(lib().tpsa_plan_tile(ctypes.byref(plan), block, tile, ctypes.byref(k0), ctypes.byref(w),
                               ctypes.byref(up), ctypes.byref(m)))
    return k0.value, w.value, bool(m.value), up.value


def workspace_size(query_tokens: int, query_start: int, seq_len: int, prompt_len: int) -> int:
    out = _u64()
    check(lib().tpsa_workspace_size(query_tokens, query_start, seq_len, prompt_len, ctypes.byref(out)))
    return out.value


def dense_workspace_size(query_tokens: int, query_start: int, seq_len: int) -> int:
    out = _u64()
    check(lib().tpsa_dense_workspace_size(query_tokens, query_start, seq_len, ctypes.byref(out)))
    return out.value


def paged_attention_dense(query, key_cache, value_cache, block_table, out, query_start: int,
                          seq_len: int, scale: float, *, workspace=None, stream=None) -> None:
    """The all-dense control (plain causal attention over the paged context)
    through the C ABI; a workspace is allocated when none is given."""
    import torch

    if stream is None:
        stream = torch.cuda.current_stream(query.device).cuda_stream
    if workspace is None:
        nbytes = dense_workspace_size(query.shape[0], query_start, seq_len)
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=query.device)
    check(lib().tpsa_paged_attention_dense(
        query.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), block_table.data_ptr(),
        out.data_ptr(), query.shape[0], key_cache.shape[0], block_table.shape[-1], query_start,
        seq_len, scale, workspace.data_ptr(), workspace.numel() * workspace.element_size(),
        stream))


def _int64_array(values) -> ctypes.Array:
    vals = [int(v) for v in values]
    return (_i64 * len(vals))(*vals)


def varlen_workspace_size(cu_seqlens_q, seq_lens, prompt_lens, *, kv_heads=None) -> int:
    """Scratch bytes of tpsa_paged_attention_varlen (or, with ``kv_heads``, of its
    head-slice form) on the current device (host metadata)."""
    batch = len(seq_lens)
    out = _u64()
    args = (batch, _int64_array(cu_seqlens_q), _int64_array(seq_lens), _int64_array(prompt_lens))
    if kv_heads is None:
        check(lib().tpsa_varlen_workspace_size(*args, ctypes.byref(out)))
    else:
        check(lib().tpsa_varlen_workspace_size_heads(*args, kv_heads, ctypes.byref(out)))
    return out.value


def paged_attention_varlen(query, key_cache, value_cache, block_tables, out, cu_seqlens_q,
                           seq_lens, prompt_lens, scale: float, *, kv_heads=None,
                           workspace=None, stream=None, value_offset_pages: int = 0) -> None:
    """Packed ragged batch through the C ABI.

    ``query``/``out`` are packed ``[cu_seqlens_q[-1], 32, 128]`` CUDA tensors and
    ``block_tables`` a ``[batch, table_cols]`` int32 CUDA tensor; the per-request
    metadata (``cu_seqlens_q``, ``seq_lens``, ``prompt_lens``) are host integer
    sequences.  With ``kv_heads`` the head-slice form runs (``[rows, 4*kv_heads,
    128]`` queries, ``kv_heads``-head caches).  A workspace is allocated from
    torch when none is given.  ``value_offset_pages`` > 0 reads V that many
    pages past the start of ``value_cache`` (see ``paged_attention``).
    """
    import torch

    batch = len(seq_lens)
    if stream is None:
        stream = torch.cuda.current_stream(query.device).cuda_stream
    if workspace is None:
        nbytes = varlen_workspace_size(cu_seqlens_q, seq_lens, prompt_lens, kv_heads=kv_heads)
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=query.device)
    common = (query.data_ptr(), key_cache.data_ptr(),
              _value_ptr(value_cache, value_offset_pages),
              block_tables.data_ptr(), out.data_ptr(), batch, _int64_array(cu_seqlens_q),
              _int64_array(seq_lens), _int64_array(prompt_lens), key_cache.shape[0],
              block_tables.shape[-1], scale)
    ws = (workspace.data_ptr(), workspace.numel() * workspace.element_size(), stream)
    if kv_heads is None:
        check(lib().tpsa_paged_attention_varlen(*common, *ws))
    else:
        check(lib().tpsa_paged_attention_varlen_heads(*common, kv_heads, *ws))


def debug_wait_probe(limit_ns: int) -> None:
    """Test hook: the next single-request launch on this thread waits, in
    every CTA, on a barrier nothing arrives on with a limit of ``limit_ns``
    before claiming work; it issues no load or store and leaves
    TPSA_DEVICE_WAIT_TIMEOUT in the device status word.  0 disarms."""
    check(lib().tpsa_debug_wait_probe(limit_ns))


def device_status(device: int = 0) -> int:
    bits = ctypes.c_uint32()
    st = lib().tpsa_device_status(device, ctypes.byref(bits))
    if st not in (TPSA_OK, 5):
        check(st)
    return bits.value


def _value_ptr(value_cache, offset_pages: int) -> int:
    """Address of V: ``offset_pages`` cache pages past ``value_cache``'s start.

    vLLM's Triton backend stores a block's K and V pages next to each other
    (``[num_blocks, 2, 128, heads, 128]``).  Viewed as ``2 * num_blocks``
    pages, block b's K page is page 2b and its V page is 2b + 1: the launch
    passes that view as both caches, the block table doubled, and V one page
    further, so that V of table entry 2b is page 2b + 1.
    """
    if not offset_pages:
        return value_cache.data_ptr()
    page_bytes = value_cache[0].numel() * value_cache.element_size()
    return value_cache.data_ptr() + offset_pages * page_bytes


def paged_attention(query, key_cache, value_cache, block_table, out, query_start: int,
                    seq_len: int, prompt_len: int, scale: float, *, kv_heads: int | None = None,
                    workspace=None, stream=None, visited=None, tile_counter=None,
                    value_offset_pages: int = 0) -> None:
    """Launch through the C ABI with torch CUDA tensors (no checks beyond the ABI's).

    ``value_offset_pages`` > 0 reads V that many pages past the start of
    ``value_cache`` (an interleaved K/V page layout, ``_value_ptr``)."""
    import torch

    if stream is None:
        stream = torch.cuda.current_stream(query.device).cuda_stream
    h = lib()
    ws_ptr = workspace.data_ptr() if workspace is not None else None
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    common = (query.data_ptr(), key_cache.data_ptr(), _value_ptr(value_cache, value_offset_pages),
              block_table.data_ptr(), out.data_ptr(), query.shape[0], key_cache.shape[0],
              block_table.shape[-1], query_start, seq_len, prompt_len, scale)
    if visited is not None:
        check(h.tpsa_paged_attention_visit(*common, kv_heads or key_cache.shape[2], ws_ptr, ws_bytes,
                                           visited.data_ptr(), tile_counter.data_ptr(), stream))
    elif kv_heads is not None:
        check(h.tpsa_paged_attention_heads(*common, kv_heads, ws_ptr, ws_bytes, stream))
    else:
        check(h.tpsa_paged_attention(*common, ws_ptr, ws_bytes, stream))


def paged_attention_static_scratch(query, key_cache, value_cache, block_table, out,
                                   query_start: int, seq_len: int, prompt_len: int, scale: float,
                                   *, stream=None) -> None:
    """Launch the variant that allocates nothing (scratch in a module-global array).

    For callers that cannot allocate device memory when they run the
    operator.  Calls on one device share the scratch, so they must be ordered on one
    stream. The first call on a device sets up the scratch address; make it
    before any stream capture.
    """
    import torch

    if stream is None:
        stream = torch.cuda.current_stream(query.device).cuda_stream
    check(lib().tpsa_paged_attention_static_scratch(
        query.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), block_table.data_ptr(),
        out.data_ptr(), query.shape[0], key_cache.shape[0], block_table.shape[-1],
        query_start, seq_len, prompt_len, scale, stream))


_ADAPTER_LOADED: str | None = None


def load_adapter(path: str | Path | None = None) -> str:
    """Load the torch op adapter once per process (refuses a second path)."""
    import torch

    global _ADAPTER_LOADED
    resolved = str(Path(path or ADAPTER_PATH).resolve())
    with _LOCK:
        if _ADAPTER_LOADED is not None:
            if _ADAPTER_LOADED != resolved:
                raise RuntimeError(
                    f"TriangleMix adapter is already loaded from {_ADAPTER_LOADED}; refusing {resolved}")
            return resolved
        if not Path(resolved).is_file():
            raise FileNotFoundError(f"TriangleMix Torch adapter does not exist: {resolved}")
        torch.ops.load_library(resolved)
        try:
            torch.ops.trianglemix.triangle_paged_sparse_attention.out
        except (AttributeError, RuntimeError) as err:
            raise RuntimeError(
                "TriangleMix adapter did not register trianglemix::triangle_paged_sparse_attention.out"
            ) from err
        _ADAPTER_LOADED = resolved
        return resolved


def adapter_loaded() -> bool:
    with _LOCK:
        return _ADAPTER_LOADED is not None
