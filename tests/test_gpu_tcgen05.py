"""The tcgen05 (TMEM accumulator) partial kernel against the FP64 oracle.

Each case runs with the kernel forced to tcgen05 (kvb_set_decode_kernel) and
with the warp-level MMA kernel, both through the C ABI; each must meet the
path tolerance against the oracle. Shapes: the reference's native
rows-8 / group-6 / dim-256 / 32-token-page shape (48 query columns in one
CTA), fewer columns, causal rows, partial and one-token ranges, odd stage
counts (a last tile of one stage), explicit partitions, and the 64-token-page
dim-128 variant at BASELINE cfg2's geometry.
"""
from __future__ import annotations

import pytest
import torch

import kvbridge_b200 as kvb
import oracle
from kvbridge_b200 import synth
from kvb_testutil import check_against_oracle, report, run_single

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _reset(cuda_device):
    kvb.read_device_status()
    kvb.set_wait_limit_ns(200_000_000)  # a broken pipeline reports within 0.2 s
    yield
    kvb.set_decode_kernel(kvb.KERNEL_AUTO)
    kvb.set_wait_limit_ns(0)
    assert kvb.read_device_status() == 0, kvb.read_wait_failure()


CASES = [
    # rows, q_heads, kv_heads, dim, page, tokens, begin, end, partitions
    (8, 24, 4, 256, 32, 4096, 0, None, 0),     # native shape
    (8, 24, 4, 256, 32, 4096, 0, None, 5),     # odd stage counts per piece
    (8, 24, 4, 256, 32, 1000, 96, 777, 3),     # partial range, ragged pages
    (3, 24, 4, 256, 32, 2500, 0, None, 0),     # 18 columns
    (1, 24, 4, 256, 32, 3000, 0, None, 0),     # 6 columns
    (8, 24, 4, 256, 32, 300, 150, 151, 0),     # one token
    (1, 32, 8, 128, 64, 8192, 0, None, 0),     # cfg2 geometry on the dim-128 variant
    (2, 32, 8, 128, 64, 5000, 0, None, 3),     # 8 columns, causal rows
]


@pytest.mark.parametrize("rows,q_heads,kv_heads,dim,page,tokens,begin,end,partitions", CASES)
def test_tcgen05_kernel_matches_oracle(cuda_device, rows, q_heads, kv_heads, dim, page, tokens, begin, end,
                                       partitions):
    qpos = [tokens - rows + r for r in range(rows)] if rows > 1 else None
    case = synth.make_single(rows=rows, q_heads=q_heads, kv_heads=kv_heads, dim=dim, page_tokens=page,
                             tokens=tokens, seed=tokens + rows + dim, device=cuda_device, begin=begin, end=end,
                             q_positions=qpos)
    assert kvb.attention_b200_supported(case.shape, case.device_input())
    ref = oracle.reference_case(case, threads=16)
    results = {}
    for name, choice in (("tcgen05", kvb.KERNEL_TCGEN05), ("warp-mma", kvb.KERNEL_WARP_MMA)):
        kvb.set_decode_kernel(choice)
        res = run_single(case, partitions=partitions)
        assert kvb.read_device_status() == 0, (name, kvb.read_wait_failure())
        ma, rl = check_against_oracle(res, case.shape, ref, f"{name} {rows}x{q_heads}/{kv_heads} d{dim} P{page}")
        results[name] = (ma, rl)
    report(f"tcgen05 vs oracle {rows}x{q_heads}/{kv_heads} d{dim} P{page} [{begin},{end or tokens}) "
           f"parts {partitions}", tc_max_abs=results["tcgen05"][0], tc_rel_l2=results["tcgen05"][1],
           warp_max_abs=results["warp-mma"][0], warp_rel_l2=results["warp-mma"][1])


def test_tcgen05_reference_fixture(cuda_device):
    """The reference's own fixture (make_fixture(513), three-splits case)
    through launch_attention_mma on the tcgen05 kernel."""
    from test_gpu_reference_fixtures import fixture_case, strict_gate

    kvb.set_decode_kernel(kvb.KERNEL_TCGEN05)
    for test in range(7):
        case = fixture_case(test, cuda_device)
        ref = oracle.reference_case(case, threads=8)
        res = run_single(case, fp16_out=False, api="mma")
        ma, rl = check_against_oracle(res, case.shape, ref, f"tc fixture {test}")
        ok, worst, ratio = strict_gate(res, case.shape, ref)
        report(f"tcgen05 reference self-test {test}", max_abs=ma, rel_l2=rl, strict_gate_pass=ok,
               strict_worst_over_allowance=ratio)
        again = run_single(case, fp16_out=False, api="mma")
        for k in ("m", "l", "n"):
            assert torch.equal(again[k], res[k]), k
