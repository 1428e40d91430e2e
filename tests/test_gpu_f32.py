"""fp32 KV (Shape.int8 = False, reference src/attention_shared.cu:350-353):
the streaming partial kernel (decode_f32.cuh) through the C ABI against the
FP64 oracle, against the general CUDA-core kernel on the same inputs, and on
its edge cases (ragged begin/end, causal and fully masked rows, several
column groups, explicit partitions, a page id outside the pool).

K and V are fp32 ~N(0,1) in the reference layout
(include/kvbridge/attention_common.h: K [(page*kv+h)*P + s][D],
V [(page*kv+h)*D + d][P]); the scale pointers are ignored.
"""
from __future__ import annotations

import pytest
import torch

import kvbridge_b200 as kvb
import oracle
from kvbridge_b200 import synth
from kvb_testutil import check_against_oracle, errors, normalized, report, run_single

pytestmark = pytest.mark.gpu

STATUS_BAD_PAGE = 4


@pytest.fixture(autouse=True)
def _status_clean(cuda_device):
    kvb.read_device_status()
    kvb.set_decode_kernel(kvb.KERNEL_AUTO)
    yield
    kvb.set_decode_kernel(kvb.KERNEL_AUTO)
    assert kvb.read_device_status() == 0, "a kernel reported a bounded-wait timeout or bad page"


def make_f32(device, rows, q_heads, kv_heads, dim, page_tokens, tokens, seed, begin=0, end=None,
             q_positions=None):
    """A single-sequence case with fp32 K/V ~N(0,1) (shuffled pages, fp16-exact Q)."""
    base = synth.make_single(rows=rows, q_heads=q_heads, kv_heads=kv_heads, dim=dim, page_tokens=page_tokens,
                             tokens=tokens, seed=seed, device=device, begin=begin, end=end,
                             q_positions=q_positions)
    pages = base.shape.pages
    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 0x5EED)
    k = torch.randn((pages, kv_heads, page_tokens, dim), generator=gen, device=device)
    v = torch.randn((pages, kv_heads, dim, page_tokens), generator=gen, device=device)
    shape = kvb.Shape(**{**base.shape.__dict__, "int8": False})
    return synth.SingleCase(shape, base.q, base.q_positions, base.k_positions, base.page_table,
                            k.reshape(-1), v.reshape(-1), None, None)


def ref_of(case, threads=16):
    return oracle.reference(case.shape, case.q, case.q_positions, case.k_positions, case.page_table,
                            case.k, case.v, threads=threads)


CASES = [
    # id: (rows, q_heads, kv_heads, dim, page_tokens, tokens, begin, end, q_positions, partitions)
    ("cfg1-geometry", (1, 32, 8, 128, 64, 4096, 0, None, None, 0)),
    ("dim64-page32", (1, 32, 8, 64, 32, 3000, 0, None, None, 0)),
    ("dim64-page16-gqa4", (1, 8, 2, 64, 16, 800, 0, None, None, 0)),
    ("page16-ragged-range-gqa8", (1, 64, 8, 128, 16, 5000, 37, 4999, None, 0)),
    ("causal-rows2-page16", (2, 16, 4, 128, 16, 2000, 0, None, [1990, 1999], 0)),
    ("rows4-16-columns", (4, 16, 4, 128, 32, 1000, 0, None, [996, 997, 998, 999], 0)),
    ("masked-row", (2, 8, 2, 128, 64, 700, 0, None, [-1, 699], 0)),
    ("three-partitions", (1, 32, 8, 128, 64, 2500, 100, 2400, None, 3)),
    ("one-partition-many-stages", (1, 32, 8, 128, 32, 6000, 0, None, None, 1)),
]


@pytest.mark.parametrize("label,args", CASES, ids=[c[0] for c in CASES])
def test_f32_kv_against_oracle(cuda_device, label, args):
    rows, qh, kvh, dim, P, tokens, begin, end, qpos, parts = args
    case = make_f32(cuda_device, rows, qh, kvh, dim, P, tokens, seed=0xF32 + tokens + dim, begin=begin, end=end,
                    q_positions=qpos)
    res = run_single(case, partitions=parts)
    ma, rl = check_against_oracle(res, case.shape, ref_of(case), f"fp32-{label}")
    report(f"fp32 KV {label}", max_abs=ma, rel_l2=rl)


def test_f32_kv_cfg2_size_matches_oracle_and_general_kernel(cuda_device):
    """cfg2's geometry with fp32 KV (65,536 tokens, 32/8 heads, dim 128,
    64-token shuffled pages): the streaming kernel and the general kernel
    both meet the oracle bar, and their outputs differ (different kernels ran)."""
    case = make_f32(cuda_device, 1, 32, 8, 128, 64, 65536, seed=0xF32C2)
    ref = ref_of(case)
    fast = run_single(case)
    ma, rl = check_against_oracle(fast, case.shape, ref, "fp32-cfg2")
    kvb.set_decode_kernel(kvb.KERNEL_GENERAL)
    general = run_single(case)
    kvb.set_decode_kernel(kvb.KERNEL_AUTO)
    mg, rg = check_against_oracle(general, case.shape, ref, "fp32-cfg2-general")
    report("fp32 KV cfg2 geometry (65,536 tokens)", max_abs=ma, rel_l2=rl, general_max_abs=mg,
           general_rel_l2=rg)
    assert not torch.equal(fast["n"], general["n"]), "the streaming kernel did not run"
    between = errors(normalized(fast, case.shape), normalized(general, case.shape))
    assert between[0] <= 2e-3 and between[1] <= 1e-3, between


def test_f32_kv_bitwise_repeatable(cuda_device):
    case = make_f32(cuda_device, 2, 16, 4, 128, 16, 3000, seed=0xF32B, q_positions=[2990, 2999])
    a = run_single(case)
    b = run_single(case)
    for key in ("m", "l", "n", "out"):
        assert torch.equal(a[key], b[key]), key


def test_f32_kv_page_past_the_pool(cuda_device):
    """A page-table entry equal to `pages`: no copy is issued for it, status
    4, the call returns; the next call on good inputs is correct."""
    case = make_f32(cuda_device, 1, 32, 8, 128, 64, 4096, seed=0xF32D)
    bad_table = case.page_table.clone()
    bad_table[5] = case.shape.pages
    bad = synth.SingleCase(case.shape, case.q, case.q_positions, case.k_positions, bad_table,
                           case.k, case.v, None, None)
    run_single(bad)
    assert kvb.read_device_status() == STATUS_BAD_PAGE
    res = run_single(case)
    assert kvb.read_device_status() == 0
    check_against_oracle(res, case.shape, ref_of(case), "fp32 after bad page")


def test_f32_kv_unaligned_buffers_use_general_kernel(cuda_device):
    """V starting 4 bytes past a 16-byte boundary is still served (general kernel)."""
    case = make_f32(cuda_device, 1, 16, 4, 128, 64, 900, seed=0xF32E)
    vbuf = torch.empty(case.v.numel() + 1, dtype=torch.float32, device=cuda_device)
    vbuf[1:] = case.v
    shifted = synth.SingleCase(case.shape, case.q, case.q_positions, case.k_positions, case.page_table,
                               case.k, vbuf[1:], None, None)
    res = run_single(shifted)
    check_against_oracle(res, case.shape, ref_of(case), "fp32 unaligned v")
