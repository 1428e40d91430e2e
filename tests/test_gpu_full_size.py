"""The BASELINE configurations at their stated sizes, through the C ABI,
against the FP64 oracle (every sequence and every head is checked).

* cfg3: batch 32, lengths U[1024, 32768] (seeded), 32/8 heads, dim 128,
  64-token pages in one shared shuffled pool (about 1.1 GB of KV).
* cfg4: batch 64 x 16,384 tokens, 64/8 heads (GQA 8), 16-token pages (the
  four-page gather loads), 1 % of tokens with 10x outliers (2.2 GB).
* cfg5: one full 1,048,576-token sequence through launch_attention_ex, and
  a batched call over 4 x 1,048,576 tokens plus one short sequence whose
  shared pool holds more than 2^32 bytes of K (and of V), with pages beyond
  the 2^32-byte mark in use, so that the kernels' 64-bit pool offsets are
  exercised.

The achieved errors are reported through kvb_testutil.report.
"""
from __future__ import annotations

import os

import pytest
import torch

import kvbridge_b200 as kvb
import oracle
from kvbridge_b200 import synth
from kvb_testutil import check_against_oracle, check_batched, check_bf16, host_pool, report, run_single

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 8


@pytest.fixture(autouse=True)
def _status_clean(cuda_device):
    kvb.read_device_status()
    yield
    assert kvb.read_device_status() == 0, "a kernel reported a bounded-wait timeout or bad page"
    torch.cuda.empty_cache()


def _run_batched(bc, device, bf16=True):
    s = bc.shape
    ws_bytes = kvb.batch_workspace_bytes(s)
    ws = torch.empty(ws_bytes // 4 + 16, device=device)
    B, H, D = s.batch, s.q_heads, s.dim
    m = torch.full((B * H,), float("nan"), device=device)
    l = torch.full((B * H,), float("nan"), device=device)
    n = torch.full((B * H * D,), float("nan"), device=device)
    out = torch.full((B * H * D,), float("nan"), dtype=torch.float16, device=device)
    out_bf16 = torch.full((B * H * D,), float("nan"), dtype=torch.bfloat16, device=device) if bf16 else None
    kvb.launch_attention_batched(s, bc.batch_input(), ws, ws_bytes, m, l, n, out, out_bf16=out_bf16)
    torch.cuda.synchronize()
    return m, l, n, out, out_bf16


def test_cfg3_full_size(cuda_device):
    lens = synth.ragged_lengths(32, 1024, 32768, seed=0xC0FFEE + 3)
    bc = synth.make_batched(32, 8, 128, 64, lens, seed=0xC0FFEE + 3, device=cuda_device)
    m, l, n, out, out_bf16 = _run_batched(bc, cuda_device)
    ma, rl = check_batched(bc, m, l, n, out, "cfg3", THREADS, out_bf16=out_bf16)
    report("cfg3 full (batch 32, U[1K,32K], Page64)", max_abs=ma, rel_l2=rl, tokens=sum(lens))


def test_cfg4_full_size(cuda_device):
    lens = [16384] * 64
    bc = synth.make_batched(64, 8, 128, 16, lens, seed=0xC0FFEE + 4, device=cuda_device, outlier_frac=0.01)
    m, l, n, out, out_bf16 = _run_batched(bc, cuda_device)
    ma, rl = check_batched(bc, m, l, n, out, "cfg4", THREADS, out_bf16=out_bf16)
    report("cfg4 full (batch 64 x 16K, GQA 8, Page16, 1% outliers)", max_abs=ma, rel_l2=rl, tokens=sum(lens))


def test_cfg5_one_full_sequence(cuda_device):
    """One 1,048,576-token sequence (16,384 shuffled 64-token pages) through
    the single-sequence launcher, fp16 and bf16 outputs."""
    case = synth.make_single(rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=1 << 20,
                             seed=0xC0FFEE + 5, device=cuda_device)
    s = case.shape
    scratch = torch.empty(kvb.scratch_elements(s), device=cuda_device)
    rh, nd = kvb.output_scalar_elements(s), kvb.output_numerator_elements(s)
    m = torch.empty(rh, device=cuda_device)
    l = torch.empty(rh, device=cuda_device)
    n = torch.empty(nd, device=cuda_device)
    out = torch.empty(nd, dtype=torch.float16, device=cuda_device)
    out_bf16 = torch.empty(nd, dtype=torch.bfloat16, device=cuda_device)
    kvb.launch_attention_ex(s, case.device_input(), scratch, m, l, n, out_f16=out, out_bf16=out_bf16)
    torch.cuda.synchronize()
    ref = oracle.reference_case(case, threads=THREADS)
    res = {"m": m.cpu(), "l": l.cpu(), "n": n.cpu(), "out": out.cpu()}
    ma, rl = check_against_oracle(res, s, ref, "cfg5 one sequence")
    check_bf16(out_bf16.cpu(), s, ref, "cfg5 one sequence bf16")
    report("cfg5 one 1M-token sequence (launch_attention_ex)", max_abs=ma, rel_l2=rl, tokens=s.end)


def test_cfg5_batched_pool_beyond_4gib(cuda_device):
    """Four 1M-token sequences and one of 4,096 tokens in one shuffled pool
    of 65,600 pages: K alone spans 65,600 * 8 * 64 * 128 B > 2^32 B, and the
    shuffled block table sends pages of the long sequences past that mark."""
    lens = [1 << 20] * 4 + [4096]
    bc = synth.make_batched(32, 8, 128, 64, lens, seed=0xC0FFEE + 55, device=cuda_device)
    s = bc.shape
    k_bytes = s.pages * s.kv_heads * s.page_tokens * s.dim
    assert k_bytes > 1 << 32, k_bytes
    beyond = (1 << 32) // (s.kv_heads * s.page_tokens * s.dim)  # first page past 2^32 bytes
    high = [int((bc.block_table[b, : (lens[b] + 63) // 64] >= beyond).sum()) for b in range(4)]
    assert all(h > 0 for h in high), high
    m, l, n, out, out_bf16 = _run_batched(bc, cuda_device)
    ma, rl = check_batched(bc, m, l, n, out, "cfg5 pool>4GiB", THREADS, out_bf16=out_bf16)
    report("cfg5 batched 4 x 1M + 4K, pool > 2^32 B", max_abs=ma, rel_l2=rl, tokens=sum(lens),
           k_pool_bytes=k_bytes, pages_beyond_4gib=sum(high))
