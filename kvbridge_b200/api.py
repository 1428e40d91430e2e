"""Python mirror of the kvbridge decode-attention interface, over the C ABI.

Names, argument meaning and error behaviour follow the reference's C++ API
(include/kvbridge/attention_shape.h and attention_common.h of
dkeryyyy/kvbridge): invalid metadata or buffers raise ``ValueError`` (the
reference's ``std::invalid_argument``) before anything is enqueued and CUDA
failures raise ``RuntimeError`` (``std::runtime_error``). Buffers are device
pointers given as ``torch.Tensor`` (their ``data_ptr()``) or plain integers;
the caller owns them, exactly as in the reference.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Any, Optional

from . import _lib
from ._lib import KvbAppendInput, KvbAppendShape, KvbBatchInput, KvbBatchShape, KvbDeviceInput, KvbShape, check

kSplitTokens = 256


def _ptr(x: Any) -> Optional[int]:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def _stream(stream: Any) -> Optional[int]:
    if stream is None:
        try:
            import torch

            if torch.cuda.is_available() and torch.cuda.is_initialized():
                return int(torch.cuda.current_stream().cuda_stream) or None
        except ImportError:  # pragma: no cover - torch is always present here
            pass
        return None
    if isinstance(stream, int):
        return stream or None
    return int(stream.cuda_stream) or None


@dataclass
class Shape:
    """kvbridge::Shape (reference attention_shape.h:9-13)."""

    rows: int
    q_heads: int
    kv_heads: int
    dim: int
    page_tokens: int
    pages: int
    tokens: int
    begin: int
    end: int
    scale: float
    int8: bool = True

    def c(self) -> KvbShape:
        return KvbShape(
            self.rows,
            self.q_heads,
            self.kv_heads,
            self.dim,
            self.page_tokens,
            self.pages,
            self.tokens,
            self.begin,
            self.end,
            self.scale,
            self.int8,
        )


@dataclass
class DeviceInput:
    """kvbridge::DeviceInput (reference attention_common.h:54-63)."""

    q: Any
    q_positions: Any
    k_positions: Any
    page_table: Any
    k: Any
    v: Any
    k_scales: Any = None
    v_scales: Any = None

    def c(self) -> KvbDeviceInput:
        return KvbDeviceInput(*(_ptr(getattr(self, f)) for f, _ in KvbDeviceInput._fields_))


# ---- shape layer (reference src/attention_shape.cpp) ----


def attention_shape_error(s: Shape) -> Optional[str]:
    msg = _lib.load().kvb_attention_shape_error(ctypes.byref(s.c()))
    return msg.decode() if msg else None


def attention_shape_valid(s: Shape) -> bool:
    return bool(_lib.load().kvb_attention_shape_valid(ctypes.byref(s.c())))


def validate_shape(s: Shape) -> None:
    check(_lib.load().kvb_validate_shape(ctypes.byref(s.c())))


def split_count(s: Shape) -> int:
    out = ctypes.c_uint()
    check(_lib.load().kvb_split_count(ctypes.byref(s.c()), ctypes.byref(out)))
    return out.value


def _size_query(fn_name: str, s: Shape) -> int:
    out = ctypes.c_size_t()
    check(getattr(_lib.load(), fn_name)(ctypes.byref(s.c()), ctypes.byref(out)))
    return out.value


def scratch_elements(s: Shape) -> int:
    return _size_query("kvb_scratch_elements", s)


def output_scalar_elements(s: Shape) -> int:
    return _size_query("kvb_output_scalar_elements", s)


def output_numerator_elements(s: Shape) -> int:
    return _size_query("kvb_output_numerator_elements", s)


def attention_mma_supported(s: Shape) -> bool:
    return bool(_lib.load().kvb_attention_mma_supported(ctypes.byref(s.c())))


# ---- kernels (reference attention_common.h:69-96) ----


def preload_attention_kernels() -> int:
    return int(_lib.load().kvb_preload_attention_kernels())


def preload_attention_reference_kernels() -> int:
    return int(_lib.load().kvb_preload_attention_reference_kernels())


def preload_attention_mma_kernels() -> int:
    return int(_lib.load().kvb_preload_attention_mma_kernels())


def launch_attention(s: Shape, inp: DeviceInput, scratch, m, l, n, stream=None) -> None:
    check(
        _lib.load().kvb_launch_attention(
            ctypes.byref(s.c()),
            ctypes.byref(inp.c()),
            _ptr(scratch),
            _ptr(m),
            _ptr(l),
            _ptr(n),
            _stream(stream),
        )
    )


def launch_attention_mma(s: Shape, inp: DeviceInput, scratch, m, l, n, stream=None) -> None:
    check(
        _lib.load().kvb_launch_attention_mma(
            ctypes.byref(s.c()),
            ctypes.byref(inp.c()),
            _ptr(scratch),
            _ptr(m),
            _ptr(l),
            _ptr(n),
            _stream(stream),
        )
    )


def merge_attention(s: Shape, scratch, splits: int, m, l, n, stream=None) -> None:
    check(
        _lib.load().kvb_merge_attention(
            ctypes.byref(s.c()), _ptr(scratch), splits, _ptr(m), _ptr(l), _ptr(n), _stream(stream)
        )
    )


# ---- B200 extensions (include/kvbridge/attention_b200.h) ----


def attention_b200_supported(s: Shape, inp: DeviceInput) -> bool:
    return bool(_lib.load().kvb_attention_b200_supported(ctypes.byref(s.c()), ctypes.byref(inp.c())))


def attention_partitions(s: Shape, requested: int = 0) -> int:
    out = ctypes.c_uint()
    check(_lib.load().kvb_attention_partitions(ctypes.byref(s.c()), requested, ctypes.byref(out)))
    return out.value


def launch_attention_ex(
    s: Shape, inp: DeviceInput, scratch, m, l, n, partitions: int = 0, out_f16=None, stream=None,
    out_bf16=None,
) -> None:
    """launch_attention with explicit partitions and optional normalised
    outputs n / l in fp16 (``out_f16``) and/or bf16 (``out_bf16``)."""
    if out_bf16 is None:
        status = _lib.load().kvb_launch_attention_ex(
            ctypes.byref(s.c()), ctypes.byref(inp.c()), partitions, _ptr(out_f16), _ptr(scratch),
            _ptr(m), _ptr(l), _ptr(n), _stream(stream))
    else:
        status = _lib.load().kvb_launch_attention_ex2(
            ctypes.byref(s.c()), ctypes.byref(inp.c()), partitions, _ptr(out_f16), _ptr(out_bf16),
            _ptr(scratch), _ptr(m), _ptr(l), _ptr(n), _stream(stream))
    check(status)


def launch_attention_partials(s: Shape, inp: DeviceInput, scratch, partitions: int = 0, stream=None) -> int:
    """Partial kernel only; returns the partition count it used."""
    used = ctypes.c_uint()
    check(
        _lib.load().kvb_launch_attention_partials(
            ctypes.byref(s.c()), ctypes.byref(inp.c()), partitions, _ptr(scratch), ctypes.byref(used), _stream(stream)
        )
    )
    return used.value


def merge_attention_ex(s: Shape, scratch, partitions: int, m, l, n, out_f16=None, stream=None,
                       out_bf16=None) -> None:
    if out_bf16 is None:
        status = _lib.load().kvb_merge_attention_ex(
            ctypes.byref(s.c()), _ptr(scratch), partitions, _ptr(m), _ptr(l), _ptr(n), _ptr(out_f16),
            _stream(stream))
    else:
        status = _lib.load().kvb_merge_attention_ex2(
            ctypes.byref(s.c()), _ptr(scratch), partitions, _ptr(m), _ptr(l), _ptr(n), _ptr(out_f16),
            _ptr(out_bf16), _stream(stream))
    check(status)


@dataclass
class BatchShape:
    batch: int
    q_heads: int
    kv_heads: int
    dim: int
    page_tokens: int
    pages: int
    table_stride: int
    max_tokens: int
    scale: float

    def c(self) -> KvbBatchShape:
        return KvbBatchShape(
            self.batch,
            self.q_heads,
            self.kv_heads,
            self.dim,
            self.page_tokens,
            self.pages,
            self.table_stride,
            self.max_tokens,
            self.scale,
        )


@dataclass
class BatchInput:
    q: Any
    seq_lens: Any
    block_table: Any
    k: Any
    v: Any
    k_scales: Any
    v_scales: Any

    def c(self) -> KvbBatchInput:
        return KvbBatchInput(*(_ptr(getattr(self, f)) for f, _ in KvbBatchInput._fields_))


def batch_shape_error(s: BatchShape) -> Optional[str]:
    msg = _lib.load().kvb_batch_shape_error(ctypes.byref(s.c()))
    return msg.decode() if msg else None


def batch_workspace_bytes(s: BatchShape) -> int:
    out = ctypes.c_size_t()
    check(_lib.load().kvb_batch_workspace_bytes(ctypes.byref(s.c()), ctypes.byref(out)))
    return out.value


def launch_attention_batched(
    s: BatchShape, inp: BatchInput, workspace, workspace_bytes: int, m, l, n, out_f16=None, stream=None,
    out_bf16=None,
) -> None:
    if out_bf16 is None:
        status = _lib.load().kvb_launch_attention_batched(
            ctypes.byref(s.c()), ctypes.byref(inp.c()), _ptr(workspace), workspace_bytes, _ptr(m), _ptr(l),
            _ptr(n), _ptr(out_f16), _stream(stream))
    else:
        status = _lib.load().kvb_launch_attention_batched2(
            ctypes.byref(s.c()), ctypes.byref(inp.c()), _ptr(workspace), workspace_bytes, _ptr(m), _ptr(l),
            _ptr(n), _ptr(out_f16), _ptr(out_bf16), _stream(stream))
    check(status)


def merge_attention_shards(
    shards: int, row_heads: int, dim: int, m_parts, l_parts, n_parts, m, l, n, out_f16=None, stream=None
) -> None:
    check(
        _lib.load().kvb_merge_attention_shards(
            shards,
            row_heads,
            dim,
            _ptr(m_parts),
            _ptr(l_parts),
            _ptr(n_parts),
            _ptr(m),
            _ptr(l),
            _ptr(n),
            _ptr(out_f16),
            _stream(stream),
        )
    )


def merge_attention_shards_ex(
    shards: int, row_heads: int, dim: int, m_parts, l_parts, n_parts, shard_stride: int, m, l, n,
    out_f16=None, out_bf16=None, stream=None,
) -> None:
    """merge_attention_shards with a shard stride in floats (0 = separate
    m/l/n arrays; row_heads * (dim + 2) = a packed [shard][m | l | n] buffer)
    and an optional bf16 output."""
    check(
        _lib.load().kvb_merge_attention_shards_ex(
            shards, row_heads, dim, _ptr(m_parts), _ptr(l_parts), _ptr(n_parts), shard_stride, _ptr(m), _ptr(l),
            _ptr(n), _ptr(out_f16), _ptr(out_bf16), _stream(stream),
        )
    )


def peer_buffer_bytes(row_heads: int, dim: int) -> int:
    """Bytes of one rank's peer buffer for merge_attention_peers."""
    n = int(_lib.load().kvb_peer_buffer_bytes(row_heads, dim))
    if n == 0:
        raise ValueError("row_heads must be positive and dim in [1, 256]")
    return n


def peer_slot(buffer: int, epoch: int, row_heads: int, dim: int) -> int:
    """Device address of the slot call ``epoch`` writes its partials into
    (packed [m | l | n] floats)."""
    return int(_lib.load().kvb_peer_slot(buffer, epoch, row_heads, dim))


def peer_buffer_alloc(nbytes: int) -> tuple[int, bytes]:
    """Allocates (cudaMalloc, zeroed) and exports a peer buffer: returns its
    device address and its 64-byte CUDA IPC handle."""
    ptr = ctypes.c_void_p()
    handle = (ctypes.c_ubyte * 64)()
    check(_lib.load().kvb_peer_buffer_alloc(nbytes, ctypes.byref(ptr), handle))
    return int(ptr.value), bytes(handle)


def peer_buffer_open(handle: bytes) -> int:
    """Maps another rank's peer buffer from its IPC handle; returns the address."""
    if len(handle) != 64:
        raise ValueError("a CUDA IPC handle is 64 bytes")
    h = (ctypes.c_ubyte * 64).from_buffer_copy(handle)
    ptr = ctypes.c_void_p()
    check(_lib.load().kvb_peer_buffer_open(h, ctypes.byref(ptr)))
    return int(ptr.value)


def peer_buffer_close(peer_buffer: int) -> None:
    check(_lib.load().kvb_peer_buffer_close(peer_buffer))


def peer_buffer_free(buffer: int) -> None:
    check(_lib.load().kvb_peer_buffer_free(buffer))


def merge_attention_peers(buffers, rank: int, epoch: int, row_heads: int, dim: int, m, l, n,
                          out_f16=None, out_bf16=None, stream=None) -> None:
    """Exchange and merge of the ranks' shard partials over NVLink peer
    memory (see include/kvbridge_c.h): ``buffers`` holds every rank's peer
    buffer address, this rank's own at ``rank``."""
    arr = (ctypes.c_void_p * len(buffers))(*[int(b) for b in buffers])
    check(
        _lib.load().kvb_merge_attention_peers(
            arr, len(buffers), rank, epoch, row_heads, dim, _ptr(m), _ptr(l), _ptr(n), _ptr(out_f16),
            _ptr(out_bf16), _stream(stream),
        )
    )


def debug_copy_to_device(dst: int, data: bytes) -> None:
    """Test hook: copies host bytes to a device address."""
    buf = ctypes.create_string_buffer(data, len(data))
    check(_lib.load().kvb_debug_copy_to_device(dst, buf, len(data)))


def set_wait_limit_ns(ns: int) -> None:
    """Bound of any single pipeline wait in later launches (0 = default 2 s)."""
    _lib.load().kvb_set_wait_limit_ns(int(ns))


def wait_limit_ns() -> int:
    return int(_lib.load().kvb_wait_limit_ns())


def debug_fail_launch(nth: int, cuda_error: int) -> None:
    """Test hook: the nth kernel launch (1 = next) on this thread fails with
    ``cuda_error`` instead of being made (0 disarms)."""
    check(_lib.load().kvb_debug_fail_launch(nth, cuda_error))


def debug_skip_stage(stage: int) -> None:
    """Test hook: the next tensor-core partial launch on this thread leaves
    pipeline stage ``stage`` of CTA 0 unarmed (a consumer wait runs out)."""
    check(_lib.load().kvb_debug_skip_stage(stage))


KERNEL_AUTO, KERNEL_WARP_MMA, KERNEL_TCGEN05, KERNEL_GENERAL = 0, 1, 2, 3


def set_decode_kernel(choice: int) -> None:
    """Which single-sequence partial kernel later calls use: KERNEL_AUTO (by
    shape), KERNEL_WARP_MMA or KERNEL_TCGEN05 (where a variant exists), or
    KERNEL_GENERAL (the CUDA-core kernel for every launch_attention call)."""
    check(_lib.load().kvb_set_decode_kernel(int(choice)))


def decode_kernel() -> int:
    return int(_lib.load().kvb_decode_kernel())


def launch_attention_noalloc(s: Shape, inp: DeviceInput, m, l, n, partitions: int = 0, out_f16=None,
                             stream=None) -> None:
    """The decode call that allocates nothing: split-K partials in the
    library's static device array (see kvb_launch_attention_noalloc)."""
    check(
        _lib.load().kvb_launch_attention_noalloc(
            ctypes.byref(s.c()), ctypes.byref(inp.c()), partitions, _ptr(m), _ptr(l), _ptr(n), _ptr(out_f16),
            _stream(stream),
        )
    )


# ---- paged KV append (quantise + write; include/kvbridge/attention_b200.h) ----


@dataclass
class AppendShape:
    tokens: int
    kv_heads: int
    dim: int
    page_tokens: int
    pages: int

    def c(self) -> KvbAppendShape:
        return KvbAppendShape(self.tokens, self.kv_heads, self.dim, self.page_tokens, self.pages)


@dataclass
class AppendInput:
    k_new: Any  # f32 [tokens, kv_heads, dim]
    v_new: Any
    slots: Any  # i64 [tokens]: page * page_tokens + position in page; < 0 skips
    k: Any
    v: Any
    k_scales: Any
    v_scales: Any

    def c(self) -> KvbAppendInput:
        return KvbAppendInput(*(_ptr(getattr(self, f)) for f, _ in KvbAppendInput._fields_))


def append_shape_error(s: AppendShape) -> Optional[str]:
    msg = _lib.load().kvb_append_shape_error(ctypes.byref(s.c()))
    return msg.decode() if msg else None


def append_kv(s: AppendShape, inp: AppendInput, stream=None) -> None:
    """Quantise rows (absmax int8 per token and KV head) into the paged pool."""
    check(_lib.load().kvb_append_kv(ctypes.byref(s.c()), ctypes.byref(inp.c()), _stream(stream)))


def read_device_status() -> int:
    """Read and clear the kernels' status word (0 = every bounded wait succeeded)."""
    status = ctypes.c_int()
    code = _lib.load().kvb_read_device_status(ctypes.byref(status))
    if code != 0:
        raise RuntimeError(f"reading the device status failed: cudaError {code}")
    return status.value


def read_wait_failure() -> dict:
    """The first bounded wait that gave up since the last read (code 0 = none)."""
    rec = (ctypes.c_longlong * 6)()
    code = _lib.load().kvb_read_wait_failure(rec)
    if code != 0:
        raise RuntimeError(f"reading the wait-failure record failed: cudaError {code}")
    return dict(zip(("code", "block", "warp", "stage", "waited_ns", "waited_cycles"), (int(x) for x in rec)))


def schedule_cta_of(stage: int, total: int, ctas: int) -> int:
    return int(_lib.load().kvb_schedule_cta_of(stage, total, ctas))
