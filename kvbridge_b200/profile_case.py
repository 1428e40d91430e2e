"""Run a named decode workload a few times through the public API (for
profilers such as ncu): ``python -m kvbridge_b200.profile_case --case cfg4
--calls 3``. Inputs are the seeded synthetic data of the benchmark
configurations; the device status word is checked at the end.

Cases (BASELINE configurations, or slices of them small enough for a
profiler's replay passes):
  cfg1            B1, 4,096 ctx, 32/8 heads, dim 128, Page64, 8 partitions
  cfg2            B1, 65,536 ctx, 32/8 heads, dim 128, Page64 shuffled
  cfg2-rank4      one rank's share of cfg2 split over 4 GPUs (8/2 heads)
  cfg2-rank8      one rank's share of cfg2 split over 8 GPUs (4/1 heads)
  cfg3            the whole cfg3 batch: 32 ragged lengths U[1K, 32K], Page64 shared pool
  cfg3-slice      batch 8 of the cfg3 ragged lengths, Page64 shared pool
  cfg4-slice      batch 8 x 16,384, 64/8 heads, Page16, 1 % 10x outliers
  cfg4-slice-p64  the same on 64-token pages (the page size's own cost)
  cfg5-slice      batch 4 x 131,072 tokens (one eighth of each cfg5 sequence)
  native          the reference's native shape: rows 8, 24/4 heads, dim 256,
                  Page32, 32,768 ctx
  f32             cfg2's geometry with fp32 KV ~N(0,1) (537 MB of K/V)
  peer-merge      merge_attention_peers with one rank (cfg5's partial shape: 4 x
                  32 row-heads, dim 128), the kernel's own work without NVLink
``--kernel warp|tcgen05|general`` forces the single-sequence partial kernel.
"""
from __future__ import annotations

import argparse
import sys

import torch

from . import api, build, synth

CASES = ("peer-merge", "cfg1", "cfg2", "cfg2-rank4", "cfg2-rank8", "cfg3", "cfg3-slice", "cfg4-slice", "cfg4-slice-p64", "cfg5-slice", "native", "f32")


def _single(case: synth.SingleCase, partitions: int):
    s = case.shape
    scratch = torch.empty(api.scratch_elements(s), device=case.q.device)
    rh, nd = api.output_scalar_elements(s), api.output_numerator_elements(s)
    m = torch.empty(rh, device=case.q.device)
    l = torch.empty(rh, device=case.q.device)
    n = torch.empty(nd, device=case.q.device)
    out = torch.empty(nd, dtype=torch.float16, device=case.q.device)
    inp = case.device_input()

    def call():
        api.launch_attention_ex(s, inp, scratch, m, l, n, partitions=partitions, out_f16=out)

    return call


def _batched(bc: synth.BatchCase):
    s = bc.shape
    dev = bc.q.device
    ws_bytes = api.batch_workspace_bytes(s)
    ws = torch.empty(ws_bytes // 4 + 16, device=dev)
    B, H, D = s.batch, s.q_heads, s.dim
    m = torch.empty(B * H, device=dev)
    l = torch.empty(B * H, device=dev)
    n = torch.empty(B * H * D, device=dev)
    out = torch.empty(B * H * D, dtype=torch.float16, device=dev)
    inp = bc.batch_input()

    def call():
        api.launch_attention_batched(s, inp, ws, ws_bytes, m, l, n, out)

    return call


def _peer_merge(device):
    import numpy as np

    rh, dim = 4 * 32, 128
    own, _ = api.peer_buffer_alloc(api.peer_buffer_bytes(rh, dim))
    g = np.random.default_rng(7)
    m = g.normal(0, 3, rh).astype(np.float32)
    l = g.uniform(0.5, 40, rh).astype(np.float32)
    n = g.normal(0, 5, rh * dim).astype(np.float32)
    for epoch in (1, 2):
        api.debug_copy_to_device(api.peer_slot(own, epoch, rh, dim), m.tobytes() + l.tobytes() + n.tobytes())
    mo = torch.empty(rh, device=device)
    lo = torch.empty(rh, device=device)
    no = torch.empty(rh * dim, device=device)
    out = torch.empty(rh * dim, dtype=torch.float16, device=device)
    state = {"epoch": 0}

    def call():
        state["epoch"] += 1
        api.merge_attention_peers([own], 0, state["epoch"], rh, dim, mo, lo, no, out)

    return call


def make_call(name: str, device):
    seed = 0xC0FFEE
    if name == "peer-merge":
        return _peer_merge(device)
    if name == "cfg1":
        return _single(synth.make_single(1, 32, 8, 128, 64, 4096, seed + 1, device), 8)
    if name == "cfg2":
        return _single(synth.make_single(1, 32, 8, 128, 64, 65536, seed + 2, device), 0)
    if name in ("cfg2-rank4", "cfg2-rank8"):
        kv = 2 if name == "cfg2-rank4" else 1
        return _single(synth.make_single(1, 4 * kv, kv, 128, 64, 65536, seed + 2, device), 0)
    if name in ("cfg3", "cfg3-slice"):
        lens = synth.ragged_lengths(32, 1024, 32768, seed=seed + 3)
        lens = lens if name == "cfg3" else lens[:8]
        return _batched(synth.make_batched(32, 8, 128, 64, lens, seed + 3, device))
    if name in ("cfg4-slice", "cfg4-slice-p64"):
        page = 16 if name == "cfg4-slice" else 64
        return _batched(synth.make_batched(64, 8, 128, page, [16384] * 8, seed + 4, device, outlier_frac=0.01))
    if name == "cfg5-slice":
        return _batched(synth.make_batched(32, 8, 128, 64, [131072] * 4, seed + 5, device))
    if name == "native":
        tokens, rows = 32768, 8
        case = synth.make_single(rows, 24, 4, 256, 32, tokens, seed + 8, device,
                                 q_positions=[tokens - rows + r for r in range(rows)])
        return _single(case, 0)
    if name == "f32":
        base = synth.make_single(1, 32, 8, 128, 64, 65536, seed + 32, device)
        shape = api.Shape(**{**base.shape.__dict__, "int8": False})
        gen = torch.Generator(device=device)
        gen.manual_seed(seed + 0xF32)
        k = torch.randn(shape.pages * 8 * 64 * 128, generator=gen, device=device)
        v = torch.randn(shape.pages * 8 * 128 * 64, generator=gen, device=device)
        return _single(synth.SingleCase(shape, base.q, base.q_positions, base.k_positions, base.page_table,
                                        k, v, None, None), 0)
    raise ValueError(f"unknown case {name!r}; one of {', '.join(CASES)}")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--case", choices=CASES, required=True)
    ap.add_argument("--calls", type=int, default=3)
    ap.add_argument("--kernel", choices=["auto", "warp", "tcgen05", "general"], default="auto")
    args = ap.parse_args(argv)
    build.build()
    device = torch.device("cuda", 0)
    api.set_decode_kernel({"auto": api.KERNEL_AUTO, "warp": api.KERNEL_WARP_MMA,
                           "tcgen05": api.KERNEL_TCGEN05, "general": api.KERNEL_GENERAL}[args.kernel])
    call = make_call(args.case, device)
    torch.cuda.synchronize()
    for _ in range(args.calls):
        call()
    torch.cuda.synchronize()
    status = api.read_device_status()
    if status != 0:
        print(f"device status {status}: {api.read_wait_failure()}", file=sys.stderr)
        return 1
    print(f"{args.case}: {args.calls} calls ok")
    return 0


if __name__ == "__main__":
    sys.exit(main())
