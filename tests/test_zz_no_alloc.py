"""The decode call that allocates nothing (kvb_launch_attention_noalloc).

Its users are callers that cannot call cudaMalloc when they decode: an
inference server whose memory pool reserved every byte of HBM up front for its
KV cache, or a host whose decode path must not allocate. It keeps the split-K
partials in a static device array of the library instead of a caller-provided
scratch buffer.

Through the C ABI, two calls in a row must each agree with the existing entry
point (kvb_launch_attention_ex with caller scratch) within the path's
tolerance, and with the FP64 oracle. The cases cover a shape whose requested
partitions do not fit the array (the launcher clamps them), 16-token pages,
an empty token range and a shape too large for the array (rejected). This
file is named to be collected last and also runs alone in a fresh process (it
builds the library and initialises CUDA itself).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import kvbridge_b200 as kvb
import oracle
from kvbridge_b200 import _lib, synth
from kvb_testutil import MAX_ABS, REL_L2, check_against_oracle, errors, normalized

pytestmark = pytest.mark.gpu

# Floats in the library's static array (include/kvbridge_c.h).
ARRAY_FLOATS = 524288


def _noalloc(case, m, l, n, out, partitions=0):
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.kvb_launch_attention_noalloc(
        ctypes.byref(case.shape.c()), ctypes.byref(case.device_input().c()), partitions,
        m.data_ptr(), l.data_ptr(), n.data_ptr(), out.data_ptr() if out is not None else None,
        stream or None)
    _lib.check(rc)


def _nan_outputs(shape, device):
    rh, nd = kvb.output_scalar_elements(shape), kvb.output_numerator_elements(shape)
    return (torch.full((rh,), float("nan"), device=device), torch.full((rh,), float("nan"), device=device),
            torch.full((nd,), float("nan"), device=device),
            torch.full((nd,), float("nan"), dtype=torch.float16, device=device))


CASES = [
    # (rows, q_heads, kv_heads, dim, page_tokens, tokens, partitions)
    (1, 32, 8, 128, 64, 4096, 8),      # BASELINE cfg1
    (1, 32, 8, 128, 64, 65536, 0),     # BASELINE cfg2, automatic partitions
    (1, 64, 8, 128, 16, 8192, 0),      # 16-token pages (gather loads), GQA 8
    # rows 8 x group 8 at dim 256: rows * q_heads * (dim + 2) = 132,096 floats
    # a partition, so only 3 of the 16 requested fit and the launcher clamps.
    (8, 64, 8, 256, 32, 4096, 16),
]


@pytest.mark.parametrize("rows,q_heads,kv_heads,dim,page_tokens,tokens,partitions", CASES)
def test_noalloc_matches_scratch_entry_point_and_oracle(cuda_device, rows, q_heads, kv_heads, dim, page_tokens,
                                                        tokens, partitions):
    qpos = [tokens - rows + r for r in range(rows)] if rows > 1 else None
    case = synth.make_single(rows=rows, q_heads=q_heads, kv_heads=kv_heads, dim=dim, page_tokens=page_tokens,
                             tokens=tokens, seed=0xC0FFEE + 7 + dim + rows, device=cuda_device, q_positions=qpos)
    s = case.shape
    assert kvb.attention_b200_supported(s, case.device_input())
    per_partition = rows * q_heads * (dim + 2)
    clamps = kvb.attention_partitions(s, partitions) > ARRAY_FLOATS // per_partition
    if (rows, dim) == (8, 256):
        assert clamps, "this case must exercise the partition clamp"
    scratch = torch.empty(kvb.scratch_elements(s), device=cuda_device)
    m0, l0, n0, out0 = _nan_outputs(s, cuda_device)
    kvb.launch_attention_ex(s, case.device_input(), scratch, m0, l0, n0, partitions=partitions, out_f16=out0)
    torch.cuda.synchronize()
    ref = {"m": m0.cpu(), "l": l0.cpu(), "n": n0.cpu()}
    ref_norm = normalized(ref, s)
    expect = oracle.reference_case(case, threads=16)
    for call in range(2):  # the shared static array keeps the previous call's contents
        m, l, n, out = _nan_outputs(s, cuda_device)
        _noalloc(case, m, l, n, out, partitions)
        torch.cuda.synchronize()
        got = {"m": m.cpu(), "l": l.cpu(), "n": n.cpu(), "out": out.cpu()}
        ma, rl = errors(normalized(got, s), ref_norm)
        assert ma <= MAX_ABS and rl <= REL_L2, (call, ma, rl)
        ma16, rl16 = errors(out.cpu().double().numpy(), out0.cpu().double().numpy())
        assert ma16 <= MAX_ABS and rl16 <= REL_L2, (call, ma16, rl16)
        assert np.allclose(m.cpu().numpy(), ref["m"].numpy(), rtol=1e-5, atol=1e-5)
        check_against_oracle(got, s, expect, f"noalloc call {call}")
        if not clamps:
            # Same partitions and merge order as the scratch entry point.
            assert torch.equal(got["out"], out0.cpu()), call
    assert kvb.read_device_status() == 0


def test_noalloc_empty_range(cuda_device):
    """begin == end: nothing is attended; every row comes back empty."""
    case = synth.make_single(rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=512, seed=12,
                             device=cuda_device, begin=256, end=256)
    for _ in range(2):
        m, l, n, out = _nan_outputs(case.shape, cuda_device)
        _noalloc(case, m, l, n, out)
        torch.cuda.synchronize()
        assert torch.all(torch.isneginf(m.cpu())) and torch.all(l.cpu() == 0)
        assert torch.all(n.cpu() == 0) and torch.all(out.cpu() == 0)
    assert kvb.read_device_status() == 0


def test_noalloc_rejects_what_does_not_fit(cuda_device):
    # Outside the tensor-core geometry (dim 96).
    case = synth.make_single(rows=1, q_heads=8, kv_heads=2, dim=96, page_tokens=64, tokens=256, seed=3,
                             device=cuda_device)
    t = torch.empty(64 * 96, device=cuda_device)
    out = torch.empty(64 * 96, dtype=torch.float16, device=cuda_device)
    with pytest.raises(ValueError, match="tensor-core geometry"):
        _noalloc(case, t, t, t, out)
    # Tensor-core geometry, but one partition alone is larger than the array:
    # rows 8 x group 8 x 32 KV heads x (256 + 2) = 528,384 floats > 524,288.
    big = synth.make_single(rows=8, q_heads=256, kv_heads=32, dim=256, page_tokens=32, tokens=64, seed=4,
                            device=cuda_device, q_positions=[56 + r for r in range(8)])
    assert kvb.attention_b200_supported(big.shape, big.device_input())
    assert 8 * 256 * (256 + 2) > ARRAY_FLOATS
    m, l, n, out = _nan_outputs(big.shape, cuda_device)
    with pytest.raises(ValueError, match="static scratch"):
        _noalloc(big, m, l, n, out)
    assert kvb.read_device_status() == 0
