"""The C-ABI library: it loads, exports every symbol the public headers
declare, and reports invalid calls with the reference's error behaviour
(status instead of exception) without touching a GPU."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

import kvbridge_b200 as kvb
from kvbridge_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
INCLUDE = ROOT / "include"


def c_declared() -> set:
    text = (INCLUDE / "kvbridge_c.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(kvb_\w+)\s*\(", text))


def cpp_declared() -> set:
    names = set()
    for h in ("attention_shape.h", "attention_common.h", "attention_b200.h"):
        text = (INCLUDE / "kvbridge" / h).read_text()
        text = re.sub(r"//.*", "", text)
        for m in re.finditer(r"^\s*(?:[\w:<>]+\s+)+\**(\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return names - {"if", "return"}


def exported(demangle: bool) -> str:
    args = ["nm", "-D", "--defined-only"] + (["-C"] if demangle else []) + [str(_lib.LIB_PATH)]
    return subprocess.run(args, capture_output=True, text=True, check=True).stdout


def test_every_c_symbol_is_exported(kvb_lib):
    syms = exported(False)
    missing = [n for n in sorted(c_declared()) if not re.search(rf"\bT {n}$", syms, flags=re.M)]
    assert not missing, missing
    assert len(c_declared()) >= 25
    # and the ctypes table covers every declaration
    assert c_declared() == set(_lib.SIGNATURES)


def test_every_cpp_entry_point_is_exported(kvb_lib):
    syms = exported(True)
    names = cpp_declared()
    for expected in ("launch_attention", "launch_attention_mma", "merge_attention", "split_count",
                     "preload_attention_kernels", "attention_mma_supported", "launch_attention_batched"):
        assert expected in names
    missing = [n for n in sorted(names)
               if f"kvbridge::{n}(" not in syms and f"kvbridge::detail::{n}(" not in syms]
    assert not missing, missing


def _shape(**kw):
    base = dict(rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, pages=64, tokens=4096,
                begin=0, end=4096, scale=0.088, int8=True)
    base.update(kw)
    return kvb.Shape(**base)


FAKE = 0x10000  # never dereferenced: every call below fails validation first


def test_invalid_calls_fail_before_cuda(kvb_lib):
    inp = kvb.DeviceInput(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE)
    with pytest.raises(ValueError, match="dim must be in"):
        kvb.launch_attention(_shape(dim=0), inp, FAKE, FAKE, FAKE, FAKE)
    with pytest.raises(ValueError, match="non-null"):
        kvb.launch_attention(_shape(), kvb.DeviceInput(FAKE, FAKE, FAKE, FAKE, None, FAKE, FAKE, FAKE),
                             FAKE, FAKE, FAKE, FAKE)
    with pytest.raises(ValueError, match="4-byte aligned"):
        kvb.launch_attention(_shape(), kvb.DeviceInput(FAKE, FAKE, FAKE, FAKE, FAKE + 1, FAKE, FAKE, FAKE),
                             FAKE, FAKE, FAKE, FAKE)
    with pytest.raises(ValueError, match="scratch, m, l and n"):
        kvb.launch_attention(_shape(), inp, None, FAKE, FAKE, FAKE)
    with pytest.raises(ValueError, match="requires int8 KV"):
        kvb.launch_attention_mma(_shape(), inp, FAKE, FAKE, FAKE, FAKE)
    with pytest.raises(ValueError, match="split count"):
        kvb.merge_attention(_shape(), FAKE, 3, FAKE, FAKE, FAKE)
    with pytest.raises(ValueError, match="exceed"):
        kvb.merge_attention_ex(_shape(), FAKE, 17, FAKE, FAKE, FAKE)
    with pytest.raises(ValueError, match="tensor-core geometry"):
        kvb.launch_attention_partials(_shape(dim=96), inp, FAKE)


def test_status_codes_and_thread_local_message(kvb_lib):
    lib = _lib.load()
    s = _shape(q_heads=25).c()
    out = ctypes.c_uint()
    assert lib.kvb_split_count(ctypes.byref(s), ctypes.byref(out)) == _lib.KVB_EINVAL
    assert _lib.last_error() == "q_heads must be divisible by kv_heads"
    ok = _shape().c()
    assert lib.kvb_split_count(ctypes.byref(ok), ctypes.byref(out)) == _lib.KVB_OK
    assert out.value == 16 and _lib.last_error() == ""
    assert lib.kvb_attention_shape_error(None) == b"shape pointer is null"


def test_batch_shape_validation(kvb_lib):
    good = kvb.BatchShape(32, 32, 8, 128, 64, 10000, 512, 32768, 0.088)
    assert kvb.batch_shape_error(good) is None
    assert "max_tokens" in kvb.batch_shape_error(kvb.BatchShape(32, 32, 8, 128, 64, 10000, 511, 32768, 0.088))
    assert "page_tokens" in kvb.batch_shape_error(kvb.BatchShape(32, 32, 8, 128, 48, 10000, 512, 32768, 0.088))
    assert "divisible" in kvb.batch_shape_error(kvb.BatchShape(32, 30, 8, 128, 64, 10000, 512, 32768, 0.088))


def test_b200_predicate(kvb_lib):
    aligned = kvb.DeviceInput(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE)
    assert kvb.attention_b200_supported(_shape(), aligned)
    assert not kvb.attention_b200_supported(_shape(int8=False), aligned)
    assert not kvb.attention_b200_supported(_shape(dim=96), aligned)
    assert not kvb.attention_b200_supported(_shape(page_tokens=128, pages=32), aligned)
    # the reference's native shape: 48 query columns per KV head, in 6 column groups
    assert kvb.attention_b200_supported(_shape(rows=8, q_heads=24, kv_heads=4, dim=256, page_tokens=32,
                                               pages=128), aligned)
    # more than 64 query columns per KV head: general kernel
    assert not kvb.attention_b200_supported(_shape(rows=16, q_heads=24, kv_heads=4, dim=256, page_tokens=32,
                                                   pages=128), aligned)
    shifted = kvb.DeviceInput(FAKE, FAKE, FAKE, FAKE, FAKE + 4, FAKE, FAKE, FAKE)
    assert not kvb.attention_b200_supported(_shape(), shifted)


def test_wait_limit_setting(kvb_lib):
    """The bound of the kernels' pipeline waits is a launch parameter the host
    sets (no GPU needed to read it back)."""
    assert kvb.wait_limit_ns() == 2_000_000_000
    kvb.set_wait_limit_ns(5_000_000)
    assert kvb.wait_limit_ns() == 5_000_000
    kvb.set_wait_limit_ns(0)
    assert kvb.wait_limit_ns() == 2_000_000_000


def test_decode_kernel_switch(kvb_lib):
    """The process-wide kernel choice (auto, warp-level MMA, tcgen05, general
    CUDA-core kernel) round-trips through the C ABI; unknown values fall back
    to auto. Host-side state only, no GPU needed."""
    try:
        for choice in (kvb.KERNEL_WARP_MMA, kvb.KERNEL_TCGEN05, kvb.KERNEL_GENERAL, kvb.KERNEL_AUTO):
            kvb.set_decode_kernel(choice)
            assert kvb.decode_kernel() == choice
        kvb.set_decode_kernel(7)
        assert kvb.decode_kernel() == kvb.KERNEL_AUTO
    finally:
        kvb.set_decode_kernel(kvb.KERNEL_AUTO)


def test_launch_failure_hook_does_not_mask_validation(kvb_lib):
    """An armed launch-failure hook only replaces a launch: a call that fails
    validation first still reports KVB_EINVAL, and disarming is a no-op."""
    inp = kvb.DeviceInput(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE)
    kvb.debug_fail_launch(1, 2)
    try:
        with pytest.raises(ValueError, match="dim must be in"):
            kvb.launch_attention(_shape(dim=0), inp, FAKE, FAKE, FAKE, FAKE)
    finally:
        kvb.debug_fail_launch(0, 0)
    with pytest.raises(ValueError, match="shard_stride"):
        kvb.merge_attention_shards_ex(2, 32, 128, FAKE, FAKE, FAKE, 16, FAKE, FAKE, FAKE)
