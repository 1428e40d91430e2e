"""Sequence sharding across GPUs (one process per GPU, NCCL): each rank decodes
its page-aligned token range with launch_attention_ex, and the (m, l, n)
partials are either all-gathered over NCCL and merged with
merge_attention_shards, or exchanged and merged in one kernel over NVLink
peer memory (sharding.PeerExchange, merge_attention_peers) for several calls
that alternate between two cases; the result matches the FP64 oracle over
the whole range. Runs on 2 to 4 GPUs; skipped with fewer than 2."""
from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs"),
]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results, mode="nccl"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    import numpy as np
    import torch.distributed as dist

    import kvbridge_b200 as kvb
    import oracle
    from kvb_testutil import MAX_ABS, REL_L2, errors
    from kvbridge_b200 import sharding, synth

    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=device)
    try:
        if mode == "peers":
            _peer_worker(rank, world, device, results)
            dist.barrier(device_ids=[rank])
            return
        case = synth.make_single(rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=20000,
                                 seed=4242, device=device)
        shape = case.shape
        ranges = sharding.sequence_ranges(shape.tokens, shape.page_tokens, world)
        b, e = ranges[rank]
        rh = kvb.output_scalar_elements(shape)

        def local_partial():
            local = kvb.Shape(shape.rows, shape.q_heads, shape.kv_heads, shape.dim, shape.page_tokens,
                              shape.pages, shape.tokens, b, e, shape.scale, True)
            scratch = torch.empty(kvb.scratch_elements(local), device=device)
            m = torch.empty(rh, device=device)
            l = torch.empty(rh, device=device)
            n = torch.empty(rh * shape.dim, device=device)
            kvb.launch_attention_ex(local, case.device_input(), scratch, m, l, n)
            return m, l, n

        m, l, n, out = sharding.sequence_sharded_decode(local_partial, sharding.gpu_shard_merge(rh, shape.dim))
        torch.cuda.synchronize()
        status = kvb.read_device_status()
        ok = status == 0
        if rank == 0:
            cpu = synth.SingleCase(*([shape] + [getattr(case, f).cpu() for f in
                                                ("q", "q_positions", "k_positions", "page_table", "k", "v",
                                                 "k_scales", "v_scales")]))
            ref = oracle.reference_case(cpu, threads=8)
            got = (n.cpu().double().numpy().reshape(shape.rows, shape.q_heads, shape.dim)
                   / l.cpu().double().numpy().reshape(shape.rows, shape.q_heads, 1))
            ma, rl = errors(got, ref["normalized"])
            ok = ok and ma <= MAX_ABS and rl <= REL_L2
            ok = ok and np.allclose(m.cpu().numpy(), ref["m"].reshape(-1), rtol=1e-5, atol=1e-5)
            results[rank] = (bool(ok), float(ma), float(rl), status)
        else:
            results[rank] = (bool(ok), 0.0, 0.0, status)
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


def _peer_worker(rank, world, device, results):
    """Four calls over a PeerExchange, alternating between two cases (so
    that a slot read one call late would not match); every call is checked
    against the oracle on rank 0."""
    import numpy as np
    import torch.distributed as dist

    import kvbridge_b200 as kvb
    import oracle
    from kvb_testutil import MAX_ABS, REL_L2, errors
    from kvbridge_b200 import sharding, synth

    cases = [synth.make_single(rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=20000,
                               seed=4242 + i, device=device) for i in range(2)]
    shape = cases[0].shape
    b, e = sharding.sequence_ranges(shape.tokens, shape.page_tokens, world)[rank]
    rh = kvb.output_scalar_elements(shape)
    local = kvb.Shape(shape.rows, shape.q_heads, shape.kv_heads, shape.dim, shape.page_tokens, shape.pages,
                      shape.tokens, b, e, shape.scale, True)
    scratch = torch.empty(kvb.scratch_elements(local), device=device)
    refs = []
    if rank == 0:
        for c in cases:
            cpu = synth.SingleCase(*([shape] + [getattr(c, f).cpu() for f in
                                                ("q", "q_positions", "k_positions", "page_table", "k", "v",
                                                 "k_scales", "v_scales")]))
            refs.append(oracle.reference_case(cpu, threads=8))
    ex = sharding.PeerExchange(rh, shape.dim)
    ok, worst = True, (0.0, 0.0)
    try:
        m = torch.empty(rh, device=device)
        l = torch.empty(rh, device=device)
        n = torch.empty(rh * shape.dim, device=device)
        out = torch.empty(rh * shape.dim, dtype=torch.float16, device=device)
        for call in range(4):
            c = cases[call % 2]
            pm, pl, pn = ex.slot()
            kvb.launch_attention_ex(local, c.device_input(), scratch, pm, pl, pn)
            ex.merge(m, l, n, out)
            torch.cuda.synchronize()
            ok = ok and kvb.read_device_status() == 0
            if rank == 0:
                ref = refs[call % 2]
                got = (n.cpu().double().numpy().reshape(shape.rows, shape.q_heads, shape.dim)
                       / l.cpu().double().numpy().reshape(shape.rows, shape.q_heads, 1))
                ma, rl = errors(got, ref["normalized"])
                ok = ok and ma <= MAX_ABS and rl <= REL_L2
                ok = ok and np.allclose(m.cpu().numpy(), ref["m"].reshape(-1), rtol=1e-5, atol=1e-5)
                worst = (max(worst[0], float(ma)), max(worst[1], float(rl)))
    finally:
        torch.cuda.synchronize()
        dist.barrier(device_ids=[rank])  # every rank's kernels are done with every buffer
        ex.close()
    results[rank] = (bool(ok), worst[0], worst[1], 0)


def _run(mode):
    import torch.multiprocessing as mp

    world = min(4, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, results, mode)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=240)
        for p in procs:
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        res = dict(results)
    assert len(res) == world and all(v[0] for v in res.values()), res


def test_sequence_sharded_decode_over_nccl():
    _run("nccl")


def test_sequence_sharded_decode_over_peer_memory():
    _run("peers")
