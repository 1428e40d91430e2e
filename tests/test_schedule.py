"""The split-K schedule arithmetic (kvbridge_b200/csrc/kvb_schedule.h and the
piece walk of decode_tma.cuh / merge.cuh), restated in Python and checked
for the properties the kernels rely on: CTA ranges tile the stages with at
most one stage of imbalance, every (CTA, segment) piece gets a distinct
partial slot inside the workspace the host sizes, and the merge finds
exactly the pieces the partial kernel wrote. The exported host function
kvb_schedule_cta_of is compared with the restatement."""
from __future__ import annotations

import random

import kvbridge_b200 as kvb

STAGE = 64


def cta_begin(c, total, ctas):
    return c * total // ctas


def cta_of(x, total, ctas):
    return ((x + 1) * ctas - 1) // total


def stages_of_range(lo, hi):
    return 0 if hi <= lo else (hi + STAGE - 1) // STAGE - lo // STAGE


def pieces_batched(lens, kv_heads, ctas):
    """(cta, seq, head, j0, j1, slot) for every piece, walking like the kernel."""
    T = [stages_of_range(0, n) for n in lens]
    total = kv_heads * sum(T)
    pref = [0]
    for t in T:
        pref.append(pref[-1] + t)
    out = []
    for c in range(ctas):
        x, x1 = cta_begin(c, total, ctas), cta_begin(c + 1, total, ctas)
        while x < x1:
            b = next(i for i in range(len(lens)) if (pref[i + 1]) * kv_heads > x)
            seg_base = pref[b] * kv_heads
            h = (x - seg_base) // T[b]
            seg_off = seg_base + h * T[b]
            j0 = x - seg_off
            j1 = min(T[b], x1 - seg_off)
            out.append((c, b, h, j0, j1, c + b * kv_heads + h))
            x = seg_off + j1
    return out, total, pref, T


def test_host_export_matches_restatement(kvb_lib):
    rng = random.Random(5)
    for _ in range(3000):
        total = rng.randrange(1, 1 << rng.choice([4, 10, 20, 34]))
        ctas = rng.randrange(1, 4096)
        x = rng.randrange(0, total)
        assert kvb.schedule_cta_of(x, total, ctas) == cta_of(x, total, ctas)
        c = cta_of(x, total, ctas)
        assert cta_begin(c, total, ctas) <= x < cta_begin(c + 1, total, ctas)


def test_ranges_tile_and_balance():
    rng = random.Random(6)
    for _ in range(500):
        total = rng.randrange(0, 100000)
        ctas = rng.randrange(1, 600)
        sizes = [cta_begin(c + 1, total, ctas) - cta_begin(c, total, ctas) for c in range(ctas)]
        assert sum(sizes) == total
        assert max(sizes) - min(sizes) <= 1


def test_single_sequence_partitions_align_with_heads():
    for kv_heads in (1, 2, 8):
        for T in (1, 7, 64, 1024):
            for P in range(1, min(T, 40) + 1):
                ctas = P * kv_heads
                total = kv_heads * T
                for h in range(kv_heads):
                    first = cta_of(h * T, total, ctas)
                    last = cta_of(h * T + T - 1, total, ctas)
                    assert first == h * P and last == h * P + P - 1


def test_batched_slots_unique_and_merge_finds_them():
    rng = random.Random(7)
    for _ in range(200):
        batch = rng.randrange(1, 40)
        lens = [rng.choice([0, 1, 63, 64, 65, rng.randrange(0, 40000)]) for _ in range(batch)]
        kv = rng.choice([1, 2, 8])
        ctas = rng.choice([1, 7, 148, 296])
        pieces, total, pref, T = pieces_batched(lens, kv, ctas)
        slots = [p[5] for p in pieces]
        assert len(set(slots)) == len(slots)
        assert all(0 <= s < ctas + batch * kv for s in slots)
        # every segment's stages are covered exactly once, in order
        for b in range(batch):
            for h in range(kv):
                mine = sorted((p[3], p[4], p[0], p[5]) for p in pieces if p[1] == b and p[2] == h)
                if T[b] == 0:
                    assert not mine
                    continue
                assert mine[0][0] == 0 and mine[-1][1] == T[b]
                assert all(mine[i][1] == mine[i + 1][0] for i in range(len(mine) - 1))
                # merge geometry (merge.cuh): c_first .. c_last and slot = c + seg
                seg_off = pref[b] * kv + h * T[b]
                c_first = cta_of(seg_off, total, ctas)
                c_last = cta_of(seg_off + T[b] - 1, total, ctas)
                owning = [c for c in range(c_first, c_last + 1)
                          if cta_begin(c + 1, total, ctas) > cta_begin(c, total, ctas)]
                assert [m[2] for m in mine] == owning
                assert [m[3] for m in mine] == [c + b * kv + h for c in owning]
