"""ctypes binding of ``libpcp_attn.so`` (the C ABI in ``include/pcp_attn.h``).

There is no fallback: if the library is missing this module raises
``ImportError`` with the build command, and every product entry point goes
through it.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libpcp_attn.so")

PCP_KV_E4M3 = 0
PCP_KV_BF16 = 1
PCP_EXCHANGE_DIRECT = 0
PCP_EXCHANGE_RING = 1
PCP_EXCHANGE_ALLGATHER = 2
PCP_EXCHANGE_PIPELINE = 3
PCP_KV_PATH_AUTO = 0
PCP_KV_PATH_DENSE = 1
PCP_KV_PATH_IN_PLACE = 2
KV_PATHS = {"auto": PCP_KV_PATH_AUTO, "dense": PCP_KV_PATH_DENSE, "in_place": PCP_KV_PATH_IN_PLACE}

STATUS_NAMES = {
    0: "PCP_OK",
    1: "PCP_ERR_INVALID_ARGUMENT",
    2: "PCP_ERR_UNSUPPORTED",
    3: "PCP_ERR_CUDA",
    4: "PCP_ERR_NCCL",
    5: "PCP_ERR_DEVICE_TIMEOUT",
    6: "PCP_ERR_OUT_OF_MEMORY",
    7: "PCP_ERR_PEER",
}

# Every function declared in include/pcp_attn.h: name -> (restype, argtypes).
_c = ctypes
_P = _c.c_void_p
_I32 = _c.c_int32
_PI32 = _c.POINTER(_c.c_int32)


class PcpDims(ctypes.Structure):
    _fields_ = [
        ("pcp_size", _I32),
        ("local_q_len", _I32),
        ("max_local_blocks", _I32),
        ("block_size", _I32),
        ("num_q_heads", _I32),
        ("num_kv_heads", _I32),
        ("head_dim", _I32),
        ("kv_dtype", _I32),
    ]


class PcpStats(ctypes.Structure):
    _fields_ = [
        ("attn_ms", _c.c_double),
        ("unpack_ms", _c.c_double),
        ("combine_ms", _c.c_double),
        ("comm_ms", _c.c_double),
        ("kernel_launches", _I32),
        ("attn_launches", _I32),
        ("splits", _I32),
        ("forwards", _I32),
        ("ring_bytes", _c.c_int64),
        ("keys", _c.c_int64),
        ("kv_in_place", _I32),
        ("reserved", _I32),
    ]


_PDIMS = _c.POINTER(PcpDims)

SIGNATURES = {
    "pcp_last_error": (_c.c_char_p, []),
    "pcp_abi_version": (_c.c_int, []),
    "pcp_source_valid_len": (_c.c_int64, [_c.c_int64, _I32, _I32, _I32]),
    "pcp_ring_schedule": (_c.c_int, [_I32, _I32, _I32, _PI32, _PI32, _PI32, _PI32]),
    "pcp_stream_k_plan": (_c.c_int, [_c.c_int64, _c.c_int64, _I32, _I32, _PI32, _PI32]),
    "pcp_stream_k_segments": (_c.c_int, [_I32, _I32, _I32, _I32, _PI32, _I32, _PI32]),
    "pcp_nccl_unique_id_bytes": (_c.c_int, []),
    "pcp_get_nccl_unique_id": (_c.c_int, [_P]),
    "pcp_history_attention_workspace_size": (_c.c_int, [_PDIMS, _c.c_int64, _c.POINTER(_c.c_size_t)]),
    "pcp_history_attention": (_c.c_int, [_PDIMS, _P, _P, _I32, _PI32, _P, _P, _c.c_size_t, _P]),
    "pcp_history_attention_status": (_c.c_int, [_P, _P]),
    "pcp_selftest_bounded_wait": (_c.c_int, [_I32, _PI32]),
    "pcp_history_attention_noalloc": (_c.c_int, [_PDIMS, _P, _P, _I32, _PI32, _P, _P, _P]),
    "pcp_cache_write": (_c.c_int, [_PDIMS, _I32, _I32, _c.c_int64, _I32, _P, _P, _P, _I32, _P, _c.c_int64, _P, _P]),
    "pcp_history_attention_paged": (
        _c.c_int, [_PDIMS, _P, _P, _c.c_int64, _P, _I32, _PI32, _P, _P, _c.c_size_t, _P]),
    "pcp_prefill_attention_workspace_size": (_c.c_int, [_PDIMS, _c.c_int64, _c.POINTER(_c.c_size_t)]),
    "pcp_prefill_attention": (_c.c_int, [_PDIMS, _I32, _I32, _P, _P, _I32, _PI32, _P, _P, _P, _P, _c.c_size_t, _P]),
    "pcp_create": (_c.c_int, [_PDIMS, _I32, _I32, _P, _c.POINTER(_P)]),
    "pcp_forward": (_c.c_int, [_P, _P, _P, _PI32, _P, _P]),
    "pcp_forward_bucketed": (_c.c_int, [_P, _P, _P, _P, _PI32, _P, _P]),
    "pcp_forward_paged": (_c.c_int, [_P, _P, _P, _c.c_int64, _P, _PI32, _P, _P]),
    "pcp_forward_prefill": (_c.c_int, [_P, _I32, _P, _P, _PI32, _P, _P, _P, _P]),
    "pcp_forward_host": (_c.c_int, [_P, _P, _P, _PI32, _P, _P]),
    "pcp_forward_host_async": (_c.c_int, [_P, _P, _P, _PI32, _P, _P]),
    "pcp_forward_host_wait": (_c.c_int, [_P]),
    "pcp_device_status": (_c.c_int, [_P, _I32]),
    "pcp_set_exchange": (_c.c_int, [_P, _I32]),
    "pcp_set_comm_sms": (_c.c_int, [_P, _I32]),
    "pcp_set_kv_path": (_c.c_int, [_P, _I32]),
    "pcp_set_profiling": (_c.c_int, [_P, _I32]),
    "pcp_get_stats": (_c.c_int, [_P, _c.POINTER(PcpStats)]),
    "pcp_destroy": (_c.c_int, [_P]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load the extension (once).  Raises ImportError when it was not built."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m aws_training_study_b200.build` "
                    "(the CUDA path has no fallback)"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = handle
    return _lib


class PcpError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def check(status: int) -> None:
    if status != 0:
        raise PcpError(status, lib().pcp_last_error().decode(errors="replace"))


def int32_array(values) -> ctypes.Array:
    vals = [int(v) for v in values]
    return (ctypes.c_int32 * len(vals))(*vals)


def set_default_kv_path(mode: str) -> None:
    """Process default of how history launches read the KV cache
    (``pcp_set_kv_path(NULL, ...)``): ``"auto"``, ``"dense"`` or ``"in_place"``."""
    if mode not in KV_PATHS:
        raise ValueError(f"kv path must be one of {sorted(KV_PATHS)}, got {mode!r}")
    check(lib().pcp_set_kv_path(None, KV_PATHS[mode]))

