"""The fused merge (LaunchOptions::merge_counters / kvb_launch_attention_ex3):
with many partitions per KV head the partial kernel's CTAs merge the
partials themselves (the reference split-K merge of
src/attention_shared.cu:295-335, as a two-level reduction inside the kernel)
instead of a merge kernel. Through the C ABI: outputs agree with the call
without counters and with the FP64 oracle, repeat bitwise over calls (the
counters return to zero), and the scratch stays a valid decomposition that
merge_attention reproduces. Calls with few partitions ignore the counters.
"""
from __future__ import annotations

import pytest
import torch

import kvbridge_b200 as kvb
import oracle
from kvbridge_b200 import synth
from kvb_testutil import check_against_oracle, errors, normalized, outputs_for, report

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean(cuda_device):
    kvb.read_device_status()
    yield
    assert kvb.read_device_status() == 0, "a kernel reported a bounded-wait timeout or bad page"


def _call(case, partitions, counters):
    scratch, m, l, n = outputs_for(case.shape, case.q.device)
    nd = kvb.output_numerator_elements(case.shape)
    out = torch.full((nd,), float("nan"), dtype=torch.float16, device=case.q.device)
    bf = torch.full((nd,), float("nan"), dtype=torch.bfloat16, device=case.q.device)
    kvb.launch_attention_ex(case.shape, case.device_input(), scratch, m, l, n, partitions=partitions,
                            out_f16=out, out_bf16=bf, merge_counters=counters)
    torch.cuda.synchronize()
    return {"m": m.cpu(), "l": l.cpu(), "n": n.cpu(), "out": out.cpu(), "bf16": bf.cpu(), "scratch": scratch}


CASES = [
    # id: rows, q_heads, kv_heads, dim, page_tokens, tokens, partitions (0 = automatic)
    ("one-kv-head-cfg2-share", 1, 4, 1, 128, 64, 65536, 0),
    ("two-kv-heads-cfg2-share", 1, 8, 2, 128, 64, 65536, 0),
    ("ragged-last-group", 1, 4, 1, 128, 64, 20000, 100),
    ("gqa8-page16", 1, 8, 1, 128, 16, 16384, 64),
    ("causal-rows2-8-columns", 2, 8, 2, 128, 32, 24000, 80),
    ("dim64", 1, 4, 1, 64, 64, 30000, 0),
    ("dim256-page32", 1, 4, 1, 256, 32, 16384, 64),
]


@pytest.mark.parametrize("label,rows,qh,kvh,dim,P,tokens,parts", CASES, ids=[c[0] for c in CASES])
def test_fused_merge_matches_merge_kernel_and_oracle(cuda_device, label, rows, qh, kvh, dim, P, tokens, parts):
    qpos = [tokens - rows + r for r in range(rows)] if rows > 1 else None
    case = synth.make_single(rows=rows, q_heads=qh, kv_heads=kvh, dim=dim, page_tokens=P, tokens=tokens,
                             seed=0xF05E + tokens + dim + qh, device=cuda_device, q_positions=qpos)
    s = case.shape
    used = kvb.attention_partitions(s, parts)
    assert used >= 64, "the case must take the fused merge"
    counters = torch.zeros(kvb.fused_merge_counter_words(s), dtype=torch.int32, device=cuda_device)
    plain = _call(case, parts, None)
    runs = [_call(case, parts, counters) for _ in range(3)]
    assert int(counters.abs().sum()) == 0, "the kernel must return its counters to zero"
    for later in runs[1:]:
        for key in ("m", "l", "n", "out", "bf16"):
            assert torch.equal(later[key], runs[0][key]), key
    fused = runs[0]
    ref = oracle.reference_case(case, threads=16)
    ma, rl = check_against_oracle(fused, s, ref, f"fused-{label}")
    between = errors(normalized(fused, s), normalized(plain, s))
    assert between[0] <= 1e-5 and between[1] <= 1e-5, between
    report(f"fused merge {label} ({used} partitions)", max_abs=ma, rel_l2=rl, vs_merge_kernel_max_abs=between[0])
    # The scratch holds a valid decomposition: merging all its splits gives m, l, n again.
    m2 = torch.empty_like(fused["m"], device=cuda_device)
    l2 = torch.empty_like(fused["l"], device=cuda_device)
    n2 = torch.empty_like(fused["n"], device=cuda_device)
    kvb.merge_attention(s, fused["scratch"], kvb.split_count(s), m2, l2, n2)
    torch.cuda.synchronize()
    again = {"m": m2.cpu(), "l": l2.cpu(), "n": n2.cpu()}
    re = errors(normalized(again, s), normalized(fused, s))
    assert re[0] <= 1e-5 and re[1] <= 1e-6, re


def test_few_partitions_ignore_the_counters(cuda_device):
    """BASELINE cfg1 with 8 partitions: below the fused merge's threshold the
    call runs the merge kernel, bitwise as without counters, and leaves the
    counters untouched."""
    case = synth.make_single(rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=4096,
                             seed=0xC0FFEE + 1, device=cuda_device)
    counters = torch.zeros(kvb.fused_merge_counter_words(case.shape), dtype=torch.int32, device=cuda_device)
    a = _call(case, 8, None)
    b = _call(case, 8, counters)
    for key in ("m", "l", "n", "out", "bf16"):
        assert torch.equal(a[key], b[key]), key
    assert int(counters.abs().sum()) == 0
