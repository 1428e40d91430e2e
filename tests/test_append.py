"""Paged KV append: the absmax int8 quantisation of new K/V rows and their
placement into the reference's pool layout (K slot-major, V dim-major,
per-(page, kv head, slot) fp32 scales; attention_common.h:11-46).

The reference ships no quantiser (its fixtures write codes and scales
directly), so the rule is the one the benchmark configurations state: scale =
max|x| / 127, code = clamp(rint(x / scale), -127, 127) in fp32 with ties to
even, scale 0 and codes 0 for an all-zero row. The C oracle
(oracle/kvb_oracle.c kvbo_append_kv) is checked against the independent torch
restatement (kvbridge_b200.synth.quantize_kv); the kernel is checked against
the oracle bit for bit, and a decode over an appended cache against the FP64
attention oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import kvbridge_b200 as kvb
import oracle
from kvbridge_b200 import synth


def _rows(tokens, kv_heads, dim, seed, outliers=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((tokens, kv_heads, dim), generator=g)
    if outliers:
        hit = torch.rand((tokens, kv_heads), generator=g) < 0.05
        x = torch.where(hit.unsqueeze(-1), x * 10.0, x)
    if tokens > 2:
        x[1, 0] = 0.0  # all-zero row: scale 0, codes 0
        # exact ties: max 127 gives scale 1, so 2.5 -> 2, -3.5 -> -4, 0.5 -> 0
        x[2, 0] = 0.0
        x[2, 0, :4] = torch.tensor([127.0, 2.5, -3.5, 0.5])
    return x


def _pools(pages, kv_heads, page_tokens, dim, fill=0):
    k = np.full((pages, kv_heads, page_tokens, dim), fill, dtype=np.int8)
    v = np.full((pages, kv_heads, dim, page_tokens), fill, dtype=np.int8)
    ks = np.full((pages, kv_heads, page_tokens), -7.0, dtype=np.float32)
    vs = np.full((pages, kv_heads, page_tokens), -7.0, dtype=np.float32)
    return k, v, ks, vs


@pytest.mark.parametrize("kv_heads,dim,page_tokens", [(8, 128, 64), (8, 128, 16), (1, 256, 32), (3, 40, 16)])
def test_oracle_matches_torch_rule(kv_heads, dim, page_tokens):
    tokens = 200
    pages = (tokens + page_tokens - 1) // page_tokens + 3
    kn, vn = _rows(tokens, kv_heads, dim, 1), _rows(tokens, kv_heads, dim, 2)
    rng = np.random.default_rng(3)
    slots = rng.permutation(pages * page_tokens)[:tokens].astype(np.int64)
    assert slots.shape == (tokens,)
    k, v, ks, vs = _pools(pages, kv_heads, page_tokens, dim, fill=55)
    assert oracle.append_kv(kn, vn, slots, k, v, ks, vs, pages, page_tokens) == 0
    kc, ksc = synth.quantize_kv(kn)
    vc, vsc = synth.quantize_kv(vn)
    page, s = slots // page_tokens, slots % page_tokens
    assert np.array_equal(k[page, :, s, :], kc.numpy())
    assert np.array_equal(v[page, :, :, s], vc.numpy())
    assert np.array_equal(ks[page, :, s], ksc.numpy())
    assert np.array_equal(vs[page, :, s], vsc.numpy())
    # the fixed cases
    if dim >= 4:
        assert np.all(k[page[1], 0, s[1]] == 0) and ks[page[1], 0, s[1]] == 0
        assert list(k[page[2], 0, s[2], :4]) == [127, 2, -4, 0] and ks[page[2], 0, s[2]] == 1.0
    # untouched slots keep their contents
    written = np.zeros((pages, page_tokens), dtype=bool)
    written[page, s] = True
    assert np.all(k.transpose(0, 2, 1, 3)[~written] == 55)
    assert np.all(v.transpose(0, 3, 1, 2)[~written] == 55)
    assert np.all(ks.transpose(0, 2, 1)[~written] == -7.0)


def test_oracle_skips_negative_and_out_of_range_slots():
    kv_heads, dim, P, pages = 2, 64, 16, 4
    kn, vn = _rows(5, kv_heads, dim, 4), _rows(5, kv_heads, dim, 5)
    slots = np.array([-1, 3, pages * P, 17, -5], dtype=np.int64)
    k, v, ks, vs = _pools(pages, kv_heads, P, dim, fill=9)
    assert oracle.append_kv(kn, vn, slots, k, v, ks, vs, pages, P) == 1
    touched = np.zeros((pages, P), dtype=bool)
    touched[0, 3] = touched[1, 1] = True
    assert np.all(k.transpose(0, 2, 1, 3)[~touched] == 9)
    assert np.all(v.transpose(0, 3, 1, 2)[~touched] == 9)
    assert np.all(ks.transpose(0, 2, 1)[touched] >= 0) and np.all(ks.transpose(0, 2, 1)[~touched] == -7.0)


def test_append_shape_validation(kvb_lib):
    ok = kvb.AppendShape(1, 8, 128, 64, 16)
    assert kvb.append_shape_error(ok) is None
    assert "kv_heads" in kvb.append_shape_error(kvb.AppendShape(1, 0, 128, 64, 16))
    assert "dim" in kvb.append_shape_error(kvb.AppendShape(1, 8, 257, 64, 16))
    assert "page_tokens" in kvb.append_shape_error(kvb.AppendShape(1, 8, 128, 0, 16))
    assert "pages" in kvb.append_shape_error(kvb.AppendShape(1, 8, 128, 64, 0))
    assert "2^48" in kvb.append_shape_error(kvb.AppendShape(1, 8, 256, 1 << 16, 1 << 22))
    # no GPU work: validation fails first, and zero tokens launch nothing
    with pytest.raises(ValueError, match="dim"):
        kvb.append_kv(kvb.AppendShape(1, 8, 0, 64, 16), kvb.AppendInput(*([0x10000] * 7)))
    with pytest.raises(ValueError, match="non-null"):
        kvb.append_kv(kvb.AppendShape(1, 8, 128, 64, 16),
                      kvb.AppendInput(0x10000, None, 0x10000, 0x10000, 0x10000, 0x10000, 0x10000))
    kvb.append_kv(kvb.AppendShape(0, 8, 128, 64, 16), kvb.AppendInput(*([None] * 7)))


# ---------------------------------------------------------------------------
# GPU


def _device_pools(np_pools, device):
    return [torch.from_numpy(a.copy()).to(device) for a in np_pools]


@pytest.mark.gpu
@pytest.mark.parametrize("kv_heads,dim,page_tokens", [(8, 128, 64), (8, 128, 16), (1, 256, 32), (4, 64, 16), (3, 40, 32)])
def test_append_kernel_matches_oracle(cuda_device, kv_heads, dim, page_tokens):
    tokens = 300
    pages = (tokens + page_tokens - 1) // page_tokens + 3
    kn, vn = _rows(tokens, kv_heads, dim, 11), _rows(tokens, kv_heads, dim, 12)
    rng = np.random.default_rng(13)
    slots = rng.permutation(pages * page_tokens)[:tokens].astype(np.int64)
    assert slots.shape == (tokens,)
    slots[::17] = -1
    ref = _pools(pages, kv_heads, page_tokens, dim, fill=-3)
    dev = _device_pools(ref, cuda_device)
    assert oracle.append_kv(kn, vn, slots, *ref, pages, page_tokens) == 0
    kvb.read_device_status()
    kvb.append_kv(kvb.AppendShape(tokens, kv_heads, dim, page_tokens, pages),
                  kvb.AppendInput(kn.to(cuda_device), vn.to(cuda_device), torch.from_numpy(slots).to(cuda_device),
                                  *dev))
    torch.cuda.synchronize()
    assert kvb.read_device_status() == 0
    for got, want in zip(dev, ref):
        assert np.array_equal(got.cpu().numpy(), want)


@pytest.mark.gpu
def test_append_out_of_range_slot_is_skipped_and_reported(cuda_device):
    kv_heads, dim, P, pages = 2, 128, 64, 4
    kn, vn = _rows(3, kv_heads, dim, 21), _rows(3, kv_heads, dim, 22)
    slots = np.array([5, pages * P + 1, 70], dtype=np.int64)
    ref = _pools(pages, kv_heads, P, dim, fill=1)
    dev = _device_pools(ref, cuda_device)
    assert oracle.append_kv(kn, vn, slots, *ref, pages, P) == 1
    kvb.read_device_status()
    kvb.append_kv(kvb.AppendShape(3, kv_heads, dim, P, pages),
                  kvb.AppendInput(kn.to(cuda_device), vn.to(cuda_device), torch.from_numpy(slots).to(cuda_device),
                                  *dev))
    torch.cuda.synchronize()
    assert kvb.read_device_status() == 6
    for got, want in zip(dev, ref):
        assert np.array_equal(got.cpu().numpy(), want)


@pytest.mark.gpu
def test_decode_over_appended_cache(cuda_device):
    """Append a 3,000-token sequence token by token in chunks through a
    shuffled page table, then decode it: the pool equals the one built with
    the torch rule, and the decode matches the FP64 oracle."""
    from kvb_testutil import check_against_oracle, run_single

    kv_heads, dim, P, q_heads, tokens = 8, 128, 64, 32, 3000
    pages = (tokens + P - 1) // P
    g = torch.Generator().manual_seed(31)
    kf = torch.randn((tokens, kv_heads, dim), generator=g)
    vf = torch.randn((tokens, kv_heads, dim), generator=g)
    table = torch.randperm(pages, generator=g).to(torch.int32)
    slots = (table.long()[torch.arange(tokens) // P] * P + torch.arange(tokens) % P)
    k = torch.zeros((pages, kv_heads, P, dim), dtype=torch.int8, device=cuda_device)
    v = torch.zeros((pages, kv_heads, dim, P), dtype=torch.int8, device=cuda_device)
    ks = torch.zeros((pages, kv_heads, P), device=cuda_device)
    vs = torch.zeros((pages, kv_heads, P), device=cuda_device)
    for t0 in range(0, tokens, 700):  # several appends, as decode steps would do
        t1 = min(tokens, t0 + 700)
        kvb.append_kv(kvb.AppendShape(t1 - t0, kv_heads, dim, P, pages),
                      kvb.AppendInput(kf[t0:t1].to(cuda_device), vf[t0:t1].to(cuda_device),
                                      slots[t0:t1].to(cuda_device), k, v, ks, vs))
    torch.cuda.synchronize()
    assert kvb.read_device_status() == 0
    kc, ksc = synth.quantize_kv(kf)
    vc, vsc = synth.quantize_kv(vf)
    pg, s = slots // P, slots % P
    assert torch.equal(k.cpu()[pg, :, s, :], kc) and torch.equal(v.cpu()[pg, :, :, s], vc)
    assert torch.equal(ks.cpu()[pg, :, s], ksc) and torch.equal(vs.cpu()[pg, :, s], vsc)
    shape = kvb.Shape(1, q_heads, kv_heads, dim, P, pages, tokens, 0, tokens, dim ** -0.5, True)
    q = torch.randn((1, q_heads, dim), generator=g).half().float()
    case = synth.SingleCase(shape, q.to(cuda_device),
                            torch.tensor([tokens - 1], dtype=torch.int64, device=cuda_device),
                            torch.arange(tokens, dtype=torch.int64, device=cuda_device),
                            table.to(cuda_device), k, v, ks, vs)
    res = run_single(case, partitions=5)
    check_against_oracle(res, shape, oracle.reference_case(case, threads=8), "appended")
