"""ctypes binding of ``libtqb.so`` (the C ABI declared in ``include/tqb.h``).

The product path has exactly one implementation: the sm_100a kernels in
``libtqb.so``.  When the library is missing or fails to load, every entry
point raises ``TqbError``; there is no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("TQB_LIBRARY", PKG_DIR / "libtqb.so"))

TQB_OK = 0
TQB_ERR_INVALID_ARG = -1
TQB_ERR_UNSUPPORTED = -2
TQB_ERR_ALIGNMENT = -3
TQB_ERR_LAUNCH = -4
TQB_ERR_CUDA = -5

TQB_LAYOUT_SOA = 0
TQB_LAYOUT_AOS = 1
TQB_LAYOUT_SOA_K8 = 2
TQB_LAYOUT_SOA_K3 = 3
TQB_LAYOUT_SOA_K3V3 = 4

TQB_P2P_MAX_RANKS = 8
TQB_IPC_HANDLE_BYTES = 64

TQB_DTYPE_F32 = 0
TQB_DTYPE_F16 = 1
TQB_DTYPE_BF16 = 2

# Every symbol include/tqb.h declares.
EXPORTED_SYMBOLS = (
    "tqb_stage1",
    "tqb_stage2",
    "tqb_merge_partials",
    "tqb_store",
    "tqb_strerror",
    "tqb_last_error_detail",
    "tqb_version",
    "tqb_wait_timeouts",
    "tqb_decode_static",
    "tqb_stage2_typed",
    "tqb_fold_sinks",
    "tqb_rotate_query",
    "tqb_stage1_rotated",
    "tqb_p2p_buffer_bytes",
    "tqb_p2p_alloc",
    "tqb_p2p_free",
    "tqb_ipc_export",
    "tqb_ipc_import",
    "tqb_ipc_close",
    "tqb_sp_exchange",
    "tqb_sp_merge",
)


# Status names, the same text tqb_strerror() returns (usable before the
# library is loaded, e.g. for the error that says it cannot be loaded).
STATUS_TEXT = {
    TQB_OK: "ok",
    TQB_ERR_INVALID_ARG: "invalid argument",
    TQB_ERR_UNSUPPORTED: "unsupported shape or configuration",
    TQB_ERR_ALIGNMENT: "misaligned pointer or stride",
    TQB_ERR_LAUNCH: "kernel launch failed",
    TQB_ERR_CUDA: "CUDA runtime error",
}


class TqbError(RuntimeError):
    """A libtqb entry point rejected its arguments or failed to launch."""

    def __init__(self, status: int, detail: str = ""):
        self.status = status
        msg = f"tqb: {STATUS_TEXT.get(status, f'status {status}')}"
        if detail:
            msg += f": {detail}"
        super().__init__(msg)


_i32, _i64, _f32, _vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p


class Stage1Args(ctypes.Structure):
    _fields_ = [
        ("q_rot", _vp), ("q_stride_b", _i64), ("q_stride_h", _i64),
        ("kv_cache", _vp), ("layout", _i32),
        ("cache_stride_block", _i64), ("cache_stride_pos", _i64), ("cache_stride_head", _i64),
        ("num_blocks", _i64),
        ("block_table", _vp), ("block_table_stride", _i64), ("max_blocks_per_seq", _i32),
        ("seq_lens", _vp), ("centroids", _vp), ("n_centroids", _i32), ("pair_lut", _vp),
        ("num_splits_per_seq", _vp),
        ("mid_o", _vp), ("mid_stride_b", _i64), ("mid_stride_h", _i64), ("mid_stride_s", _i64),
        ("batch", _i32), ("num_q_heads", _i32), ("num_kv_heads", _i32), ("head_dim", _i32),
        ("block_size", _i32), ("num_splits", _i32), ("attn_scale", _f32),
    ]


class Stage2Args(ctypes.Structure):
    _fields_ = [
        ("mid_o", _vp), ("mid_stride_b", _i64), ("mid_stride_h", _i64), ("mid_stride_s", _i64),
        ("seq_lens", _vp), ("num_splits_per_seq", _vp),
        ("output", _vp), ("out_stride_b", _i64), ("out_stride_h", _i64),
        ("lse", _vp), ("lse_stride_b", _i64),
        ("batch", _i32), ("num_q_heads", _i32), ("head_dim", _i32), ("num_splits", _i32),
    ]


class SinkArgs(ctypes.Structure):
    _fields_ = [
        ("mid_o", _vp), ("mid_stride_b", _i64), ("mid_stride_h", _i64),
        ("seq_lens", _vp), ("sinks", _vp),
        ("batch", _i32), ("num_q_heads", _i32), ("head_dim", _i32),
    ]


class DecodeStaticArgs(ctypes.Structure):
    """``tqb_decode_static_args``: Stage1 arguments (mid_o ignored) plus the
    Stage2 outputs."""

    _fields_ = [
        ("stage1", Stage1Args),
        ("output", _vp), ("out_stride_b", _i64), ("out_stride_h", _i64),
        ("lse", _vp), ("lse_stride_b", _i64),
    ]


class RotateArgs(ctypes.Structure):
    _fields_ = [
        ("query", _vp), ("query_dtype", _i32), ("q_stride_b", _i64), ("q_stride_h", _i64),
        ("rotation", _vp), ("q_rot", _vp), ("out_stride_b", _i64), ("out_stride_h", _i64),
        ("batch", _i32), ("num_q_heads", _i32), ("head_dim", _i32),
    ]


class SpExchangeArgs(ctypes.Structure):
    _fields_ = [
        ("stage2", Stage2Args), ("rank", _i32), ("world", _i32), ("cap_rows", _i64),
        ("buffers", _vp * TQB_P2P_MAX_RANKS), ("epoch", ctypes.c_uint64),
    ]


class SpMergeArgs(ctypes.Structure):
    _fields_ = [
        ("buffer", _vp), ("world", _i32), ("batch", _i32), ("num_q_heads", _i32), ("head_dim", _i32),
        ("cap_rows", _i64), ("epoch", ctypes.c_uint64), ("output", _vp), ("out_stride_b", _i64),
        ("out_stride_h", _i64), ("lse", _vp), ("lse_stride_b", _i64),
    ]


class MergeArgs(ctypes.Structure):
    _fields_ = [
        ("partials", _vp), ("num_parts", _i32), ("batch", _i32), ("num_q_heads", _i32),
        ("head_dim", _i32), ("output", _vp), ("lse", _vp),
    ]


class StoreArgs(ctypes.Structure):
    _fields_ = [
        ("y", _vp), ("norms", _vp), ("value", _vp), ("midpoints", _vp), ("centroids", _vp),
        ("slot_mapping", _vp), ("kv_cache", _vp), ("layout", _i32),
        ("cache_stride_block", _i64), ("cache_stride_pos", _i64), ("cache_stride_head", _i64),
        ("num_blocks", _i64), ("num_tokens", _i32), ("num_kv_heads", _i32), ("head_dim", _i32),
        ("block_size", _i32), ("n_centroids", _i32), ("norm_correction", _i32),
    ]


_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load ``libtqb.so`` once; raise ``TqbError`` when it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise TqbError(TQB_ERR_CUDA, f"{LIB_PATH} is not built (run __graft_entry__.build())")
            try:
                lib = ctypes.CDLL(str(LIB_PATH))
            except OSError as exc:  # pragma: no cover - depends on the host
                raise TqbError(TQB_ERR_CUDA, f"cannot load {LIB_PATH}: {exc}") from exc
            lib.tqb_stage1.argtypes = [ctypes.POINTER(Stage1Args), _vp]
            lib.tqb_stage2.argtypes = [ctypes.POINTER(Stage2Args), _vp]
            lib.tqb_merge_partials.argtypes = [ctypes.POINTER(MergeArgs), _vp]
            lib.tqb_store.argtypes = [ctypes.POINTER(StoreArgs), _vp]
            for f in (lib.tqb_stage1, lib.tqb_stage2, lib.tqb_merge_partials, lib.tqb_store):
                f.restype = ctypes.c_int
            lib.tqb_strerror.argtypes = [ctypes.c_int]
            lib.tqb_strerror.restype = ctypes.c_char_p
            lib.tqb_last_error_detail.argtypes = []
            lib.tqb_last_error_detail.restype = ctypes.c_char_p
            lib.tqb_version.argtypes = []
            lib.tqb_version.restype = ctypes.c_int
            lib.tqb_wait_timeouts.argtypes = [ctypes.POINTER(ctypes.c_uint), ctypes.c_int]
            lib.tqb_wait_timeouts.restype = ctypes.c_int
            lib.tqb_decode_static.argtypes = [ctypes.POINTER(DecodeStaticArgs), _vp]
            lib.tqb_decode_static.restype = ctypes.c_int
            lib.tqb_stage2_typed.argtypes = [ctypes.POINTER(Stage2Args), ctypes.c_int, _vp, _vp]
            lib.tqb_stage2_typed.restype = ctypes.c_int
            lib.tqb_fold_sinks.argtypes = [ctypes.POINTER(SinkArgs), _vp]
            lib.tqb_fold_sinks.restype = ctypes.c_int
            lib.tqb_rotate_query.argtypes = [ctypes.POINTER(RotateArgs), _vp]
            lib.tqb_rotate_query.restype = ctypes.c_int
            lib.tqb_stage1_rotated.argtypes = [ctypes.POINTER(RotateArgs), ctypes.POINTER(Stage1Args), _vp]
            lib.tqb_stage1_rotated.restype = ctypes.c_int
            lib.tqb_p2p_buffer_bytes.argtypes = [_i32, _i64]
            lib.tqb_p2p_buffer_bytes.restype = _i64
            lib.tqb_p2p_alloc.argtypes = [_i64, ctypes.POINTER(_vp)]
            lib.tqb_p2p_free.argtypes = [_vp]
            lib.tqb_ipc_export.argtypes = [_vp, _vp]
            lib.tqb_ipc_import.argtypes = [_vp, ctypes.POINTER(_vp)]
            lib.tqb_ipc_close.argtypes = [_vp]
            lib.tqb_sp_exchange.argtypes = [ctypes.POINTER(SpExchangeArgs), _vp]
            lib.tqb_sp_merge.argtypes = [ctypes.POINTER(SpMergeArgs), _vp]
            for f in (lib.tqb_p2p_alloc, lib.tqb_p2p_free, lib.tqb_ipc_export, lib.tqb_ipc_import,
                      lib.tqb_ipc_close, lib.tqb_sp_exchange, lib.tqb_sp_merge):
                f.restype = ctypes.c_int
            _lib = lib
    return _lib


def strerror(status: int) -> str:
    try:
        return load().tqb_strerror(status).decode()
    except TqbError:
        return f"status {status}"


def check(status: int) -> None:
    if status != TQB_OK:
        detail = load().tqb_last_error_detail().decode()
        raise TqbError(status, detail)


def version() -> int:
    return load().tqb_version()


def wait_timeouts(reset: bool = True) -> int:
    """Bounded device waits that gave up on the current device (0 in a
    healthy run); clears the counter when ``reset``."""
    n = ctypes.c_uint(0)
    check(load().tqb_wait_timeouts(ctypes.byref(n), int(bool(reset))))
    return int(n.value)
