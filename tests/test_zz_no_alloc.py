"""The decode call that allocates nothing (kvb_launch_attention_noalloc).

Its users are callers that cannot allocate device memory when they make the
call: a serving loop whose HBM is fully reserved up front by its KV-cache
allocator, or a decode step issued inside CUDA-graph stream capture, where
cudaMalloc is not permitted. It keeps the split-K partials in a static device
array instead of a caller-provided scratch buffer.

Through the C ABI, two calls in a row must each agree with the existing
entry point (kvb_launch_attention_ex with caller scratch) within the path's
tolerance. This file is named to be collected last and also runs alone in a
fresh process (it builds the library and initialises CUDA itself).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import kvbridge_b200 as kvb
from kvbridge_b200 import _lib, synth
from kvb_testutil import MAX_ABS, REL_L2, errors, normalized

pytestmark = pytest.mark.gpu


def _noalloc(case, m, l, n, out, partitions=0):
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.kvb_launch_attention_noalloc(
        ctypes.byref(case.shape.c()), ctypes.byref(case.device_input().c()), partitions,
        m.data_ptr(), l.data_ptr(), n.data_ptr(), out.data_ptr(), stream or None)
    _lib.check(rc)


@pytest.mark.parametrize("tokens,partitions", [(4096, 8), (65536, 0)])
def test_noalloc_matches_scratch_entry_point(cuda_device, tokens, partitions):
    case = synth.make_single(rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=tokens,
                             seed=0xC0FFEE + 7, device=cuda_device)
    s = case.shape
    rh, nd = kvb.output_scalar_elements(s), kvb.output_numerator_elements(s)
    scratch = torch.empty(kvb.scratch_elements(s), device=cuda_device)
    m0, l0, n0 = (torch.empty(rh, device=cuda_device), torch.empty(rh, device=cuda_device),
                  torch.empty(nd, device=cuda_device))
    out0 = torch.empty(nd, dtype=torch.float16, device=cuda_device)
    kvb.launch_attention_ex(s, case.device_input(), scratch, m0, l0, n0, partitions=partitions, out_f16=out0)
    torch.cuda.synchronize()
    ref = {"m": m0.cpu(), "l": l0.cpu(), "n": n0.cpu()}
    ref_norm = normalized(ref, s)
    for call in range(2):  # the shared static array keeps the previous call's contents
        m, l, n = (torch.full((rh,), float("nan"), device=cuda_device),
                   torch.full((rh,), float("nan"), device=cuda_device),
                   torch.full((nd,), float("nan"), device=cuda_device))
        out = torch.full((nd,), float("nan"), dtype=torch.float16, device=cuda_device)
        _noalloc(case, m, l, n, out, partitions)
        torch.cuda.synchronize()
        got = {"m": m.cpu(), "l": l.cpu(), "n": n.cpu()}
        ma, rl = errors(normalized(got, s), ref_norm)
        assert ma <= MAX_ABS and rl <= REL_L2, (call, ma, rl)
        ma16, rl16 = errors(out.cpu().double().numpy(), out0.cpu().double().numpy())
        assert ma16 <= MAX_ABS and rl16 <= REL_L2, (call, ma16, rl16)
        assert np.allclose(m.cpu().numpy(), ref["m"].numpy(), rtol=1e-5, atol=1e-5)
    assert kvb.read_device_status() == 0


def test_noalloc_rejects_what_does_not_fit(cuda_device):
    case = synth.make_single(rows=1, q_heads=8, kv_heads=2, dim=96, page_tokens=64, tokens=256, seed=3,
                             device=cuda_device)
    t = torch.empty(64 * 96, device=cuda_device)
    out = torch.empty(64 * 96, dtype=torch.float16, device=cuda_device)
    with pytest.raises(ValueError, match="tensor-core geometry"):
        _noalloc(case, t, t, t, out)
