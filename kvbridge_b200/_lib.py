"""ctypes binding of ``libkvbridge_b200.so`` (the C ABI of include/kvbridge_c.h).

The library is the product; this module only declares its symbols. Loading
fails loudly when the library is missing: there is no Python or CPU
implementation of the kernels to fall back to.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_bool, c_char_p, c_float, c_int, c_size_t, c_uint32, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libkvbridge_b200.so"
# The event-trace build of the same library (python -m kvbridge_b200.build
# --trace); loaded instead of LIB_PATH when $KVB_TRACE_LIBRARY is set to 1.
TRACE_LIB_PATH = Path(__file__).resolve().parent / "libkvbridge_b200_trace.so"

KVB_OK = 0
KVB_EINVAL = 1
KVB_ECUDA = 2


class KvbShape(ctypes.Structure):
    _fields_ = [
        ("rows", c_uint32),
        ("q_heads", c_uint32),
        ("kv_heads", c_uint32),
        ("dim", c_uint32),
        ("page_tokens", c_uint32),
        ("pages", c_uint32),
        ("tokens", c_uint32),
        ("begin", c_uint32),
        ("end", c_uint32),
        ("scale", c_float),
        ("int8", c_bool),
    ]


class KvbDeviceInput(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p),
        ("q_positions", c_void_p),
        ("k_positions", c_void_p),
        ("page_table", c_void_p),
        ("k", c_void_p),
        ("v", c_void_p),
        ("k_scales", c_void_p),
        ("v_scales", c_void_p),
    ]


class KvbBatchShape(ctypes.Structure):
    _fields_ = [
        ("batch", c_uint32),
        ("q_heads", c_uint32),
        ("kv_heads", c_uint32),
        ("dim", c_uint32),
        ("page_tokens", c_uint32),
        ("pages", c_uint32),
        ("table_stride", c_uint32),
        ("max_tokens", c_uint32),
        ("scale", c_float),
    ]


class KvbBatchInput(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p),
        ("seq_lens", c_void_p),
        ("block_table", c_void_p),
        ("k", c_void_p),
        ("v", c_void_p),
        ("k_scales", c_void_p),
        ("v_scales", c_void_p),
    ]


class KvbAppendShape(ctypes.Structure):
    _fields_ = [(n, c_uint32) for n in ("tokens", "kv_heads", "dim", "page_tokens", "pages")]


class KvbAppendInput(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("k_new", "v_new", "slots", "k", "v", "k_scales", "v_scales")]


# name -> (restype, argtypes); mirrors include/kvbridge_c.h
SIGNATURES = {
    "kvb_last_error": (c_char_p, []),
    "kvb_attention_shape_error": (c_char_p, [POINTER(KvbShape)]),
    "kvb_attention_shape_valid": (c_bool, [POINTER(KvbShape)]),
    "kvb_validate_shape": (c_int, [POINTER(KvbShape)]),
    "kvb_split_count": (c_int, [POINTER(KvbShape), POINTER(ctypes.c_uint)]),
    "kvb_scratch_elements": (c_int, [POINTER(KvbShape), POINTER(c_size_t)]),
    "kvb_output_scalar_elements": (c_int, [POINTER(KvbShape), POINTER(c_size_t)]),
    "kvb_output_numerator_elements": (c_int, [POINTER(KvbShape), POINTER(c_size_t)]),
    "kvb_attention_mma_supported": (c_bool, [POINTER(KvbShape)]),
    "kvb_preload_attention_kernels": (c_int, []),
    "kvb_preload_attention_reference_kernels": (c_int, []),
    "kvb_preload_attention_mma_kernels": (c_int, []),
    "kvb_launch_attention": (
        c_int,
        [POINTER(KvbShape), POINTER(KvbDeviceInput), c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "kvb_launch_attention_mma": (
        c_int,
        [POINTER(KvbShape), POINTER(KvbDeviceInput), c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "kvb_merge_attention": (
        c_int,
        [POINTER(KvbShape), c_void_p, ctypes.c_uint, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "kvb_attention_b200_supported": (c_bool, [POINTER(KvbShape), POINTER(KvbDeviceInput)]),
    "kvb_attention_partitions": (c_int, [POINTER(KvbShape), ctypes.c_uint, POINTER(ctypes.c_uint)]),
    "kvb_launch_attention_ex": (
        c_int,
        [
            POINTER(KvbShape),
            POINTER(KvbDeviceInput),
            ctypes.c_uint,
            c_void_p,
            c_void_p,
            c_void_p,
            c_void_p,
            c_void_p,
            c_void_p,
        ],
    ),
    "kvb_launch_attention_partials": (
        c_int,
        [POINTER(KvbShape), POINTER(KvbDeviceInput), ctypes.c_uint, c_void_p, POINTER(ctypes.c_uint), c_void_p],
    ),
    "kvb_merge_attention_ex": (
        c_int,
        [POINTER(KvbShape), c_void_p, ctypes.c_uint, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
    "kvb_batch_shape_error": (c_char_p, [POINTER(KvbBatchShape)]),
    "kvb_batch_workspace_bytes": (c_int, [POINTER(KvbBatchShape), POINTER(c_size_t)]),
    "kvb_launch_attention_batched": (
        c_int,
        [
            POINTER(KvbBatchShape),
            POINTER(KvbBatchInput),
            c_void_p,
            c_size_t,
            c_void_p,
            c_void_p,
            c_void_p,
            c_void_p,
            c_void_p,
        ],
    ),
    "kvb_append_shape_error": (c_char_p, [POINTER(KvbAppendShape)]),
    "kvb_append_kv": (c_int, [POINTER(KvbAppendShape), POINTER(KvbAppendInput), c_void_p]),
    "kvb_merge_attention_shards": (
        c_int,
        [
            ctypes.c_uint,
            ctypes.c_uint,
            ctypes.c_uint,
            c_void_p,
            c_void_p,
            c_void_p,
            c_void_p,
            c_void_p,
            c_void_p,
            c_void_p,
            c_void_p,
        ],
    ),
    "kvb_launch_attention_ex2": (
        c_int,
        [POINTER(KvbShape), POINTER(KvbDeviceInput), ctypes.c_uint] + [c_void_p] * 7,
    ),
    "kvb_merge_attention_ex2": (
        c_int,
        [POINTER(KvbShape), c_void_p, ctypes.c_uint] + [c_void_p] * 6,
    ),
    "kvb_launch_attention_batched2": (
        c_int,
        [POINTER(KvbBatchShape), POINTER(KvbBatchInput), c_void_p, c_size_t] + [c_void_p] * 6,
    ),
    "kvb_merge_attention_shards_ex": (
        c_int,
        [ctypes.c_uint, ctypes.c_uint, ctypes.c_uint, c_void_p, c_void_p, c_void_p, c_size_t] + [c_void_p] * 6,
    ),
    "kvb_peer_buffer_bytes": (c_size_t, [ctypes.c_uint, ctypes.c_uint]),
    "kvb_peer_slot": (c_void_p, [c_void_p, ctypes.c_uint, ctypes.c_uint, ctypes.c_uint]),
    "kvb_peer_buffer_alloc": (c_int, [c_size_t, POINTER(c_void_p), POINTER(ctypes.c_ubyte)]),
    "kvb_peer_buffer_open": (c_int, [POINTER(ctypes.c_ubyte), POINTER(c_void_p)]),
    "kvb_peer_buffer_close": (c_int, [c_void_p]),
    "kvb_peer_buffer_free": (c_int, [c_void_p]),
    "kvb_merge_attention_peers": (
        c_int,
        [POINTER(c_void_p), ctypes.c_uint, ctypes.c_uint, ctypes.c_uint, ctypes.c_uint, ctypes.c_uint]
        + [c_void_p] * 6,
    ),
    "kvb_debug_copy_to_device": (c_int, [c_void_p, c_void_p, c_size_t]),
    "kvb_set_wait_limit_ns": (None, [ctypes.c_ulonglong]),
    "kvb_wait_limit_ns": (ctypes.c_ulonglong, []),
    "kvb_debug_fail_launch": (c_int, [ctypes.c_uint, c_int]),
    "kvb_debug_skip_stage": (c_int, [ctypes.c_uint]),
    "kvb_set_decode_kernel": (c_int, [c_int]),
    "kvb_debug_read_tc_trace": (c_int, [POINTER(ctypes.c_ulonglong), c_size_t]),
    "kvb_debug_read_cta_trace": (c_int, [POINTER(ctypes.c_ulonglong), c_size_t]),
    "kvb_debug_read_merge_trace": (c_int, [POINTER(ctypes.c_ulonglong), c_size_t]),
    "kvb_decode_kernel": (c_int, []),
    "kvb_read_device_status": (c_int, [POINTER(c_int)]),
    "kvb_read_wait_failure": (c_int, [POINTER(ctypes.c_longlong)]),
    "kvb_schedule_cta_of": (c_uint32, [c_uint64, c_uint64, c_uint32]),
    "kvb_launch_attention_noalloc": (
        c_int,
        [POINTER(KvbShape), POINTER(KvbDeviceInput), ctypes.c_uint, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    ),
}

_lib = None


class LibraryMissing(ImportError):
    """The compiled library is absent; build it with kvbridge_b200.build."""


def load() -> ctypes.CDLL:
    """Load the library once and declare every exported function."""
    global _lib
    if _lib is not None:
        return _lib
    import os

    path = TRACE_LIB_PATH if os.environ.get("KVB_TRACE_LIBRARY") == "1" else LIB_PATH
    if not path.exists():
        raise LibraryMissing(
            f"{path} not found: run `python -m kvbridge_b200.build` (nvcc, sm_100a)"
        )
    lib = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def last_error() -> str:
    msg = load().kvb_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    """Raise the Python counterpart of the C++ exception behind a status."""
    if status == KVB_OK:
        return
    msg = last_error()
    if status == KVB_EINVAL:
        raise ValueError(msg)
    raise RuntimeError(msg)
