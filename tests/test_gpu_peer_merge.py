"""The NVLink peer merge (merge_attention_peers) on one GPU, in the forms
that need no second GPU and no kernel waiting on another kernel: one rank;
two emulated ranks whose buffers share the GPU, rank 1's publication written
from the host before rank 0's launch (its slot contents too), over both
slots; and a publication that never comes, so that the bounded wait runs out
(status 7) and the kernel returns. Results are compared with
merge_attention_shards_ex on the same partials (the all-gather form)."""
from __future__ import annotations

import struct

import numpy as np
import pytest
import torch

import kvbridge_b200 as kvb

pytestmark = pytest.mark.gpu

RH, DIM = 96, 128


@pytest.fixture(autouse=True)
def _status(cuda_device):
    kvb.read_device_status()
    yield


def _partials(seed: int, empty_every: int = 7):
    """Random (m, l, n) of one shard; every `empty_every`-th row-head empty."""
    g = np.random.default_rng(seed)
    m = g.normal(0, 3, RH).astype(np.float32)
    l = g.uniform(0.5, 40, RH).astype(np.float32)
    n = g.normal(0, 5, (RH, DIM)).astype(np.float32)
    m[::empty_every] = -np.inf
    l[::empty_every] = 0
    return m, l, n


def _packed(m, l, n) -> bytes:
    return m.tobytes() + l.tobytes() + n.tobytes()


def _reference(shards, device):
    """merge_attention_shards_ex over a packed [shard][m | l | n] tensor."""
    buf = torch.tensor(np.concatenate([np.frombuffer(_packed(*s), dtype=np.float32) for s in shards]),
                       device=device)
    m = torch.empty(RH, device=device)
    l = torch.empty(RH, device=device)
    n = torch.empty(RH * DIM, device=device)
    out = torch.empty(RH * DIM, dtype=torch.float16, device=device)
    kvb.merge_attention_shards_ex(len(shards), RH, DIM, buf, buf[RH:], buf[2 * RH:], RH * (DIM + 2), m, l, n,
                                  out_f16=out)
    torch.cuda.synchronize()
    return m.cpu(), l.cpu(), n.cpu(), out.cpu()


def _outputs(device):
    return (torch.empty(RH, device=device), torch.empty(RH, device=device), torch.empty(RH * DIM, device=device),
            torch.empty(RH * DIM, dtype=torch.float16, device=device))


def _check(got, ref):
    for name, a, b in zip(("m", "l", "n"), got[:3], ref[:3]):
        a, b = a.cpu(), b
        assert torch.allclose(a, b, rtol=1e-6, atol=1e-6, equal_nan=True), name
    assert torch.allclose(got[3].cpu().float(), ref[3].float(), rtol=2e-3, atol=2e-3)


def test_one_rank(cuda_device):
    size = kvb.peer_buffer_bytes(RH, DIM)
    own, handle = kvb.peer_buffer_alloc(size)
    assert len(handle) == 64
    try:
        shard = _partials(1)
        kvb.debug_copy_to_device(kvb.peer_slot(own, 1, RH, DIM), _packed(*shard))
        got = _outputs(cuda_device)
        kvb.merge_attention_peers([own], 0, 1, RH, DIM, *got[:3], out_f16=got[3])
        torch.cuda.synchronize()
        assert kvb.read_device_status() == 0
        _check(got, _reference([shard], cuda_device))
    finally:
        kvb.peer_buffer_free(own)


def test_two_emulated_ranks_both_slots(cuda_device):
    """Rank 0's merge with rank 1's buffer on the same GPU: rank 1's slot and
    its flag word in rank 0's buffer are written from the host before each
    launch, so rank 0's kernel waits only for its own publication."""
    size = kvb.peer_buffer_bytes(RH, DIM)
    b0, _ = kvb.peer_buffer_alloc(size)
    b1, _ = kvb.peer_buffer_alloc(size)
    try:
        for epoch in (1, 2, 3):
            s0, s1 = _partials(10 * epoch), _partials(10 * epoch + 1, empty_every=5)
            kvb.debug_copy_to_device(kvb.peer_slot(b0, epoch, RH, DIM), _packed(*s0))
            kvb.debug_copy_to_device(kvb.peer_slot(b1, epoch, RH, DIM), _packed(*s1))
            kvb.debug_copy_to_device(b0 + 4, struct.pack("<I", epoch))  # rank 1's flag in rank 0's buffer
            got = _outputs(cuda_device)
            kvb.merge_attention_peers([b0, b1], 0, epoch, RH, DIM, *got[:3], out_f16=got[3])
            torch.cuda.synchronize()
            assert kvb.read_device_status() == 0
            _check(got, _reference([s0, s1], cuda_device))
    finally:
        kvb.peer_buffer_free(b0)
        kvb.peer_buffer_free(b1)


def test_peer_wait_runs_out(cuda_device):
    """Rank 1 never publishes: the wait ends at the limit with status 7, the
    kernel returns and the device stays usable."""
    size = kvb.peer_buffer_bytes(RH, DIM)
    b0, _ = kvb.peer_buffer_alloc(size)
    b1, _ = kvb.peer_buffer_alloc(size)
    limit = kvb.wait_limit_ns()
    try:
        kvb.set_wait_limit_ns(2_000_000)  # 2 ms
        got = _outputs(cuda_device)
        kvb.merge_attention_peers([b0, b1], 0, 1, RH, DIM, *got[:3], out_f16=got[3])
        torch.cuda.synchronize()
        assert kvb.read_device_status() == 7
        rec = kvb.read_wait_failure()
        assert rec["code"] == 7 and rec["stage"] == 1  # the wait for rank 1 gave up
        assert rec["waited_ns"] >= 2_000_000
    finally:
        kvb.set_wait_limit_ns(limit)
        kvb.peer_buffer_free(b0)
        kvb.peer_buffer_free(b1)
    # The context still works.
    x = torch.ones(4, device=cuda_device)
    assert float((x * 2).sum()) == 8.0


def test_rejects(cuda_device):
    size = kvb.peer_buffer_bytes(RH, DIM)
    b0, _ = kvb.peer_buffer_alloc(size)
    try:
        got = _outputs(cuda_device)
        for bad in (dict(epoch=0), dict(rank=1)):
            kw = dict(rank=0, epoch=1)
            kw.update(bad)
            with pytest.raises(ValueError):
                kvb.merge_attention_peers([b0], kw["rank"], kw["epoch"], RH, DIM, *got[:3])
        with pytest.raises(ValueError):
            kvb.peer_buffer_bytes(0, DIM)
    finally:
        kvb.peer_buffer_free(b0)
