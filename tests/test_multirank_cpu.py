"""Multi-rank host logic on CPU ``gloo`` ranks (world size 2 and 3).

Sequence sharding: every rank computes the FP64 oracle partial (m, l, n) of
its page-aligned range, the partials are exchanged with the same
all-gather the GPU path uses, and the log-sum-exp merge equals the
single-rank oracle over the whole range. KV-head sharding: the head ranges
of the ranks tile the heads and each rank's heads equal the matching slice
of the full computation.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kvbridge_b200 import sharding


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    import oracle
    from kvbridge_b200 import synth

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        case = synth.make_single(rows=1, q_heads=8, kv_heads=4, dim=64, page_tokens=32, tokens=1000, seed=123)
        ranges = sharding.sequence_ranges(case.shape.tokens, case.shape.page_tokens, world)
        b, e = ranges[rank]

        def local_partial():
            case.shape.begin, case.shape.end = b, e
            o = oracle.reference_case(case)
            m = torch.from_numpy(o["m"].reshape(-1).copy())
            l = torch.from_numpy(o["l"].reshape(-1).copy())
            n = torch.from_numpy((o["normalized"] * o["l"][..., None]).reshape(8, 64).copy())
            return m, l, n

        def merge(mp, lp, np_):
            return oracle.merge(mp.numpy(), lp.numpy(), np_.numpy())

        m, l, n = sharding.sequence_sharded_decode(local_partial, merge)
        case.shape.begin, case.shape.end = 0, case.shape.tokens
        full = oracle.reference_case(case)
        ok = np.allclose(n / l[:, None], full["normalized"].reshape(8, 64), rtol=1e-12, atol=1e-14)
        ok = ok and np.array_equal(m, full["m"].reshape(-1))
        h0, h1 = sharding.kv_head_range(4, 2, rank % 2)
        results[rank] = (bool(ok), (b, e), (h0, h1))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sequence_sharded_merge_gloo(oracle_lib, world):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(results[r][0] for r in range(world))
    spans = [results[r][1] for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == 1000
    assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))


def test_range_planning():
    assert sharding.sequence_ranges(1_048_576, 64, 8) == [(i * 131072, (i + 1) * 131072) for i in range(8)]
    r = sharding.sequence_ranges(1000, 64, 3)
    assert r[0][0] == 0 and r[-1][1] == 1000 and all(a % 64 == 0 for a, _ in r)
    assert sharding.sequence_ranges(10, 64, 4) == [(0, 0), (0, 0), (0, 0), (0, 10)]
    assert sharding.kv_head_range(8, 8, 3) == (3, 4)
    with pytest.raises(ValueError):
        sharding.kv_head_range(8, 3, 0)
    assert sharding.local_pages([(64, 200)], 0, 64) == (1, 4)


def _peer_worker(rank, world, port, results):
    """PeerExchange's host logic with the buffer calls faked (no GPU): each
    rank 'allocates' a buffer at a rank-specific address with a rank-specific
    handle, and the exchange must map exactly the other ranks' handles, count
    epochs alike, address the alternating slots (the library's own
    arithmetic) and release everything once."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    from kvbridge_b200 import api

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        base = lambda r: 0x7F0000000000 + (r << 32)  # noqa: E731
        handle = lambda r: bytes([r + 1]) * 64  # noqa: E731
        opened, closed, freed = [], [], []
        api.peer_buffer_alloc = lambda nbytes: (base(rank), handle(rank))
        api.peer_buffer_open = lambda h: (opened.append(h), base(h[0] - 1))[1]
        api.peer_buffer_close = lambda b: closed.append(b)
        api.peer_buffer_free = lambda b: freed.append(b)
        rh, dim = 96, 128
        ex = sharding.PeerExchange(rh, dim)
        ok = ex.buffers == [base(r) for r in range(world)]
        ok = ok and sorted(opened) == sorted(handle(r) for r in range(world) if r != rank)
        slot_bytes = rh * (dim + 2) * 4
        for epoch in (1, 2, 3):
            m, l, n = ex.slot()
            want = base(rank) + 256 + (epoch & 1) * slot_bytes
            ok = ok and ex.epoch == epoch and (m, l, n) == (want, want + 4 * rh, want + 8 * rh)
        ex.close()
        ex.close()
        ok = ok and sorted(closed) == [base(r) for r in range(world) if r != rank] and freed == [base(rank)]
        try:
            ex.slot()
            ok = False
        except RuntimeError:
            pass
        results[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


def test_peer_exchange_host_logic_gloo():
    world = 3
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(results[r] for r in range(world))
