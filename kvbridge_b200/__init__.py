"""kvbridge-b200: B200-native (sm_100a) paged INT8-KV grouped-query split-K
decode attention, drop-in for the kvbridge attention library.

The product is the C++/CUDA library ``libkvbridge_b200.so`` behind the C ABI
of ``include/kvbridge_c.h``; this package binds it with ctypes and mirrors the
reference's interface names (``Shape``, ``DeviceInput``, ``launch_attention``,
``merge_attention``, ...).
"""
from .api import (  # noqa: F401
    AppendInput,
    AppendShape,
    append_kv,
    append_shape_error,
    BatchInput,
    BatchShape,
    DeviceInput,
    Shape,
    attention_b200_supported,
    attention_mma_supported,
    attention_partitions,
    attention_shape_error,
    attention_shape_valid,
    batch_shape_error,
    batch_workspace_bytes,
    kSplitTokens,
    launch_attention,
    launch_attention_batched,
    launch_attention_ex,
    launch_attention_mma,
    launch_attention_partials,
    merge_attention,
    merge_attention_ex,
    merge_attention_shards,
    merge_attention_shards_ex,
    set_wait_limit_ns,
    wait_limit_ns,
    debug_fail_launch,
    debug_skip_stage,
    launch_attention_noalloc,
    output_numerator_elements,
    output_scalar_elements,
    preload_attention_kernels,
    preload_attention_mma_kernels,
    preload_attention_reference_kernels,
    read_device_status,
    read_wait_failure,
    schedule_cta_of,
    scratch_elements,
    split_count,
    validate_shape,
)
from ._lib import LIB_PATH, LibraryMissing  # noqa: F401
