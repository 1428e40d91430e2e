"""Failure detection, provoked without faulting the GPU.

* A pipeline wait that runs out: a test hook makes the producer of CTA 0
  leave one stage unarmed (no copy, no publication), so the consumer of
  that stage waits until the wait limit (set to 1 ms here), records the
  failure and the kernel returns. The status word reads 1 (consumer wait),
  the failure record names block 0, the consumer warp and the stage, the
  call ends within milliseconds, and the next call on the same device is
  correct.
* A page-table entry equal to `pages` (one past the pool): the producer
  issues no copy for it, flags status 4 and the call returns; the next
  call with a good table is correct. Single-sequence (64- and 16-token
  pages) and batched calls.
* Host-side fault injection at the C ABI: a kernel launch reported as
  failed (cudaErrorMemoryAllocation, cudaErrorLaunchOutOfResources) gives
  KVB_ECUDA and the CUDA error text, leaves no pending CUDA error, no
  device memory held by the library and no kernel status, and the next call
  is correct.
"""
from __future__ import annotations

import ctypes
import time

import pytest
import torch

import kvbridge_b200 as kvb
import oracle
from kvbridge_b200 import _lib, synth
from kvb_testutil import check_against_oracle, outputs_for, run_single

pytestmark = pytest.mark.gpu

CUDA_ERROR_MEMORY_ALLOCATION = 2
CUDA_ERROR_LAUNCH_OUT_OF_RESOURCES = 701
STATUS_FULL_WAIT_TIMEOUT = 1
STATUS_BAD_PAGE = 4


@pytest.fixture(autouse=True)
def _clean(cuda_device):
    kvb.read_device_status()
    kvb.read_wait_failure()
    yield
    kvb.set_wait_limit_ns(0)
    kvb.debug_fail_launch(0, 0)
    torch.cuda.synchronize()
    kvb.read_device_status()
    kvb.read_wait_failure()


def _cfg1(device, page_tokens=64, seed=0xC0FFEE + 1):
    return synth.make_single(rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=page_tokens, tokens=4096,
                             seed=seed, device=device)


@pytest.mark.parametrize("page_tokens", [64, 16])
def test_wait_timeout_is_reported_and_the_next_call_is_correct(cuda_device, page_tokens):
    case = _cfg1(cuda_device, page_tokens)
    ref = oracle.reference_case(case, threads=8)
    good = run_single(case, partitions=8)  # warm: modules loaded, occupancy cached
    check_against_oracle(good, case.shape, ref, "before")
    assert kvb.read_device_status() == 0
    kvb.set_wait_limit_ns(1_000_000)
    assert kvb.wait_limit_ns() == 1_000_000
    stage = 2  # CTA 0 owns 8 stages at 8 partitions; stage 2 goes to consumer warp 2
    kvb.debug_skip_stage(stage)
    t0 = time.perf_counter()
    run_single(case, partitions=8)  # returns; its outputs are not valid
    elapsed = time.perf_counter() - t0
    assert elapsed < 1.0, elapsed
    assert kvb.read_device_status() == STATUS_FULL_WAIT_TIMEOUT
    rec = kvb.read_wait_failure()
    assert rec["code"] == STATUS_FULL_WAIT_TIMEOUT
    assert rec["block"] == 0 and rec["warp"] == stage % 4 and rec["stage"] == stage, rec
    assert 1_000_000 <= rec["waited_ns"] < 1_000_000_000, rec
    # The hook was one-shot; the device and the library carry on.
    kvb.set_wait_limit_ns(0)
    again = run_single(case, partitions=8)
    assert kvb.read_device_status() == 0
    check_against_oracle(again, case.shape, ref, "after")
    for k in ("m", "l", "n", "out"):
        assert torch.equal(again[k], good[k]), k


@pytest.mark.parametrize("page_tokens", [64, 16])
def test_page_table_entry_past_the_pool(cuda_device, page_tokens):
    case = _cfg1(cuda_device, page_tokens, seed=41)
    ref = oracle.reference_case(case, threads=8)
    bad_table = case.page_table.clone()
    bad_table[5] = case.shape.pages  # one past the last physical page
    bad = synth.SingleCase(case.shape, case.q, case.q_positions, case.k_positions, bad_table,
                           case.k, case.v, case.k_scales, case.v_scales)
    run_single(bad)
    assert kvb.read_device_status() == STATUS_BAD_PAGE
    assert kvb.read_wait_failure()["code"] == 0  # no wait gave up
    res = run_single(case)
    assert kvb.read_device_status() == 0
    check_against_oracle(res, case.shape, ref, "after bad page")


def test_block_table_entry_past_the_pool(cuda_device):
    lens = [3000, 64, 1500]
    bc = synth.make_batched(32, 8, 128, 64, lens, seed=43, device=cuda_device)
    s = bc.shape
    ws_bytes = kvb.batch_workspace_bytes(s)
    ws = torch.empty(ws_bytes // 4 + 16, device=cuda_device)
    m = torch.empty(s.batch * s.q_heads, device=cuda_device)
    l = torch.empty_like(m)
    n = torch.empty(s.batch * s.q_heads * s.dim, device=cuda_device)
    table = bc.block_table.clone()
    table[0, 7] = s.pages
    bad = synth.BatchCase(s, bc.q, bc.seq_lens, table, bc.k, bc.v, bc.k_scales, bc.v_scales, bc.lens)
    kvb.launch_attention_batched(s, bad.batch_input(), ws, ws_bytes, m, l, n)
    torch.cuda.synchronize()
    assert kvb.read_device_status() == STATUS_BAD_PAGE
    kvb.launch_attention_batched(s, bc.batch_input(), ws, ws_bytes, m, l, n)
    torch.cuda.synchronize()
    assert kvb.read_device_status() == 0


def _free_bytes():
    torch.cuda.synchronize()
    return torch.cuda.mem_get_info()[0]


@pytest.mark.parametrize("nth,code,where", [
    (1, CUDA_ERROR_MEMORY_ALLOCATION, "decode partial launch"),
    (2, CUDA_ERROR_LAUNCH_OUT_OF_RESOURCES, "attention merge launch"),
])
def test_injected_launch_failure_through_the_c_abi(cuda_device, nth, code, where):
    case = _cfg1(cuda_device, seed=47)
    good = run_single(case, partitions=8)  # every kernel of the path loaded once
    scratch, m, l, n = outputs_for(case.shape, cuda_device)
    out = torch.empty(kvb.output_numerator_elements(case.shape), dtype=torch.float16, device=cuda_device)
    free_before = _free_bytes()
    lib = _lib.load()
    assert lib.kvb_debug_fail_launch(nth, code) == _lib.KVB_OK
    rc = lib.kvb_launch_attention_ex(ctypes.byref(case.shape.c()), ctypes.byref(case.device_input().c()), 8,
                                     out.data_ptr(), scratch.data_ptr(), m.data_ptr(), l.data_ptr(),
                                     n.data_ptr(), None)
    assert rc == _lib.KVB_ECUDA
    msg = _lib.last_error()
    assert msg.startswith(where), msg
    expected_text = {CUDA_ERROR_MEMORY_ALLOCATION: "out of memory",
                     CUDA_ERROR_LAUNCH_OUT_OF_RESOURCES: "too many resources"}[code]
    assert expected_text in msg, msg
    torch.cuda.synchronize()  # no sticky or pending CUDA error
    assert _free_bytes() == free_before  # the library holds no memory it took on the failed call
    assert kvb.read_device_status() == 0
    again = run_single(case, partitions=8)
    for k in ("m", "l", "n", "out"):
        assert torch.equal(again[k], good[k]), k


def test_injected_failure_on_append(cuda_device):
    s = kvb.AppendShape(tokens=4, kv_heads=2, dim=64, page_tokens=16, pages=4)
    dev = cuda_device
    inp = kvb.AppendInput(torch.randn(4, 2, 64, device=dev), torch.randn(4, 2, 64, device=dev),
                          torch.arange(4, dtype=torch.int64, device=dev),
                          torch.zeros(4, 2, 16, 64, dtype=torch.int8, device=dev),
                          torch.zeros(4, 2, 64, 16, dtype=torch.int8, device=dev),
                          torch.zeros(4, 2, 16, device=dev), torch.zeros(4, 2, 16, device=dev))
    kvb.debug_fail_launch(1, CUDA_ERROR_MEMORY_ALLOCATION)
    with pytest.raises(RuntimeError, match="append launch: out of memory"):
        kvb.append_kv(s, inp)
    torch.cuda.synchronize()
    assert torch.all(inp.k_scales == 0)  # nothing ran
    kvb.append_kv(s, inp)
    torch.cuda.synchronize()
    assert torch.all(inp.k_scales[0, :, :4] > 0)
