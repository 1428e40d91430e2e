"""GPU parity of the sm_100a kernels against the FP64 oracle (through the C ABI).

Covers the BASELINE configurations at sizes the oracle finishes in seconds,
the reference's own GPU self-test cases (examples/attention_bench.cu:156-186:
identity/reversed pages, partial range, fully masked, empty range, causal
prefix, three splits with a partial last page) restated at the B200 geometry,
and the general-geometry kernel (fp32 KV, odd dims, wide groups, unaligned
buffers, the reference's native rows-8/group-6/dim-256 shape).
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import kvbridge_b200 as kvb
import oracle
from kvbridge_b200 import synth
from kvb_testutil import MAX_ABS, REL_L2, check_against_oracle, errors, normalized, outputs_for, run_single, to_device

pytestmark = pytest.mark.gpu


def make(device, **kw):
    return synth.make_single(device=device, **kw)


@pytest.fixture(autouse=True)
def _status_clean(cuda_device):
    kvb.read_device_status()
    yield
    assert kvb.read_device_status() == 0, "a kernel reported a bounded-wait timeout or bad page"


def test_cfg1_eight_partitions(cuda_device):
    """BASELINE cfg1: B1, ctx 4096, 32/8 heads, dim 128, Page64 shuffled, 8 partitions."""
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=4096, seed=0xC0FFEE + 1)
    assert kvb.attention_b200_supported(case.shape, case.device_input())
    assert kvb.attention_partitions(case.shape, 8) == 8
    res = run_single(case, partitions=8)
    ref = oracle.reference_case(case, threads=8)
    check_against_oracle(res, case.shape, ref, "cfg1")


@pytest.mark.parametrize("page_tokens", [16, 32, 64])
@pytest.mark.parametrize("partitions", [0, 1, 3])
def test_pages_and_partitions(cuda_device, page_tokens, partitions):
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=page_tokens,
                tokens=3000, seed=11 + page_tokens)
    res = run_single(case, partitions=partitions)
    check_against_oracle(res, case.shape, oracle.reference_case(case, threads=8), f"P{page_tokens}/{partitions}")


SELF_TEST = [
    ("identity-pages", dict(tokens=256)),
    ("partial-range", dict(tokens=256, begin=32, end=239)),
    ("fully-masked", dict(tokens=256, q_positions=[-1])),
    ("empty-range", dict(tokens=256, begin=256, end=256)),
    ("causal-prefix", dict(tokens=256, q_positions=[17])),
    ("three-splits-partial-last-page", dict(tokens=513, q_positions=[250])),
    ("mid-page-begin", dict(tokens=700, begin=77, end=611)),
    ("one-token", dict(tokens=300, begin=150, end=151)),
]


@pytest.mark.parametrize("name,kw", SELF_TEST, ids=[s[0] for s in SELF_TEST])
@pytest.mark.parametrize("page_tokens", [16, 64])
def test_reference_self_test_cases(cuda_device, name, kw, page_tokens):
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=page_tokens, seed=5, **kw)
    res = run_single(case)
    check_against_oracle(res, case.shape, oracle.reference_case(case, threads=8), name)


@pytest.mark.parametrize(
    "rows,q_heads,kv_heads,dim,qpos",
    [
        (2, 32, 8, 128, [1000, 1300]),  # 8 query rows per KV head
        (4, 32, 8, 128, [900, 1100, 1300, 1499]),  # 16 query rows: two n-tiles
        (1, 64, 8, 128, None),  # GQA 8
        (1, 16, 2, 64, None),  # dim 64
        (2, 8, 4, 64, [600, 1499]),  # dim 64, two rows
        (1, 32, 4, 256, None),  # dim 256
        (1, 32, 32, 64, None),  # group 1, 32 KV heads
    ],
)
@pytest.mark.parametrize("partitions", [0, 3])
def test_geometries(cuda_device, rows, q_heads, kv_heads, dim, qpos, partitions):
    """Auto partitions (= split_count here) and three partitions (fewer than
    split_count: the merge also marks the unused splits empty)."""
    case = make(cuda_device, rows=rows, q_heads=q_heads, kv_heads=kv_heads, dim=dim, page_tokens=32,
                tokens=1500, seed=rows * 100 + dim, q_positions=qpos)
    assert kvb.attention_b200_supported(case.shape, case.device_input())
    res = run_single(case, partitions=partitions)
    check_against_oracle(res, case.shape, oracle.reference_case(case, threads=8),
                         f"{rows}x{q_heads}/{kv_heads}d{dim}/P{partitions}")


@pytest.mark.parametrize(
    "rows,q_heads,kv_heads,dim,page_tokens",
    [
        (1, 8, 8, 128, 64),   # 1 query column per KV head
        (1, 16, 8, 256, 32),  # 2 columns, dim 256
        (3, 8, 8, 64, 16),    # 3 causal rows of group 1, dim 64, Page16
        (2, 16, 8, 256, 64),  # 4 columns: 2 rows x group 2, dim 256
        (4, 4, 4, 128, 32),   # 4 causal rows of group 1
        (1, 32, 8, 128, 16),  # cfg2 geometry on 16-token pages
    ],
)
def test_four_column_layout(cuda_device, rows, q_heads, kv_heads, dim, page_tokens):
    """At most 4 query columns per KV head take the four-column layout
    (lane pairs splitting the Q and P digits, three P digits): every column
    count 1-4, every dim and page size, causal rows whose visible ranges end
    inside a stage."""
    tokens = 2500
    qpos = [tokens - 37 * (rows - r) for r in range(rows)] if rows > 1 else None
    case = make(cuda_device, rows=rows, q_heads=q_heads, kv_heads=kv_heads, dim=dim, page_tokens=page_tokens,
                tokens=tokens, seed=rows * 1000 + dim + page_tokens, q_positions=qpos)
    assert kvb.attention_b200_supported(case.shape, case.device_input())
    for partitions in (0, 5):
        res = run_single(case, partitions=partitions)
        check_against_oracle(res, case.shape, oracle.reference_case(case, threads=8),
                             f"{rows}x{q_heads}/{kv_heads}d{dim}P{page_tokens}/{partitions}")


@pytest.mark.parametrize("kv_heads", [1, 2])
@pytest.mark.parametrize("partitions", [0, 148, 256])
def test_few_kv_heads_many_partials(cuda_device, kv_heads, partitions):
    """One rank's share of cfg2 split over 8 or 4 GPUs (1 or 2 KV heads, 65,536
    tokens): automatic partitions (256 at one KV head, 128 at two: whole
    merge rounds), 148 (a full and a partial round) or 256 per row-head,
    merged by the many-partials merge (one CTA per 32 dims, rounds of 128
    partials)."""
    case = make(cuda_device, rows=1, q_heads=4 * kv_heads, kv_heads=kv_heads, dim=128, page_tokens=64,
                tokens=65536, seed=900 + kv_heads)
    assert kvb.attention_partitions(case.shape, partitions) > 40
    res = run_single(case, partitions=partitions)
    check_against_oracle(res, case.shape, oracle.reference_case(case, threads=8), f"kv{kv_heads}/P{partitions}")


def test_outlier_scales_page16_gqa8(cuda_device):
    """cfg4 flavour: GQA 8, Page16, 1% of tokens with 10x scales."""
    case = make(cuda_device, rows=1, q_heads=64, kv_heads=8, dim=128, page_tokens=16, tokens=4096,
                seed=0xC0FFEE + 4, outlier_frac=0.01)
    res = run_single(case)
    check_against_oracle(res, case.shape, oracle.reference_case(case, threads=8), "cfg4-small")


def test_large_and_tiny_scales(cuda_device):
    """P is kept relative to a running power-of-two vscale exponent and Q is
    rescaled by a power of two, so scales far outside f16 range still work."""
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=2000, seed=77)
    case.v_scales.mul_(1e6)
    case.k_scales.mul_(1e-6)
    case.q.mul_(3e4)
    res = run_single(case)
    ref = oracle.reference_case(case, threads=8)
    got = normalized(res, case.shape)
    ma, rl = errors(got, ref["normalized"])
    assert rl <= REL_L2, rl


def test_fp32_query_not_fp16_exact(cuda_device):
    """Q that is not fp16-exact takes the hi/lo split path."""
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=2048, seed=9)
    case.q.add_(torch.randn_like(case.q) * 1e-3)
    res = run_single(case)
    check_against_oracle(res, case.shape, oracle.reference_case(case, threads=8), "fp32-q")


def test_repeatable_bitwise(cuda_device):
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=5000, seed=3)
    a = run_single(case)
    b = run_single(case)
    for k in ("m", "l", "n", "out"):
        assert torch.equal(a[k], b[k]), k


def test_reference_api_and_merge_compat(cuda_device):
    """launch_attention (reference signature) and merge_attention over the full
    split_count of the scratch it leaves behind reproduce the same m/l/n."""
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=4096, seed=21)
    res = run_single(case, api="ref", fp16_out=False)
    check_against_oracle(res, case.shape, oracle.reference_case(case, threads=8), "ref-api")
    _, m2, l2, n2 = outputs_for(case.shape, cuda_device)
    kvb.merge_attention(case.shape, res["scratch"], kvb.split_count(case.shape), m2, l2, n2)
    torch.cuda.synchronize()
    assert torch.equal(m2.cpu(), res["m"]) and torch.equal(l2.cpu(), res["l"]) and torch.equal(n2.cpu(), res["n"])


def test_page_permutation_invariance_full_cfg2(cuda_device):
    """BASELINE cfg2 at full size (64K ctx): a different physical placement of
    the same logical KV gives bitwise-identical outputs, and the result
    matches the FP64 oracle."""
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=65536, seed=0xC0FFEE + 2)
    res = run_single(case)
    ref = oracle.reference_case(case, threads=16)
    check_against_oracle(res, case.shape, ref, "cfg2")
    # Move every logical page to a new physical slot.
    g = torch.Generator(device="cpu").manual_seed(1234)
    perm = torch.randperm(case.shape.pages, generator=g).to(cuda_device)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel(), device=cuda_device)
    moved = synth.SingleCase(case.shape, case.q, case.q_positions, case.k_positions,
                             perm[case.page_table.long()].to(torch.int32),
                             case.k[inv], case.v[inv], case.k_scales[inv], case.v_scales[inv])
    res2 = run_single(moved)
    for k in ("m", "l", "n", "out"):
        assert torch.equal(res[k], res2[k]), k


def test_general_geometry_kernel(cuda_device):
    """Shapes outside the tensor-core kernel run the general kernel."""
    cases = [
        dict(rows=1, q_heads=12, kv_heads=1, dim=96, page_tokens=8, tokens=700),  # group 12, dim 96, P8
        dict(rows=16, q_heads=24, kv_heads=4, dim=256, page_tokens=32, tokens=1100),  # 96 query columns
        dict(rows=1, q_heads=4, kv_heads=2, dim=33, page_tokens=5, tokens=123),  # odd everything
    ]
    for i, kw in enumerate(cases):
        qpos = None
        if kw["rows"] > 1:
            qpos = [kw["tokens"] - kw["rows"] + r for r in range(kw["rows"])]
        case = make(cuda_device, seed=40 + i, q_positions=qpos, **kw)
        assert not kvb.attention_b200_supported(case.shape, case.device_input())
        res = run_single(case)
        check_against_oracle(res, case.shape, oracle.reference_case(case, threads=8), f"general{i}")


@pytest.mark.parametrize(
    "rows,q_heads,kv_heads,dim,page_tokens",
    [
        (8, 24, 4, 256, 32),  # the reference's native shape: 48 columns, 6 groups of 8
        (3, 24, 4, 256, 32),  # 18 columns: 3 groups, the last one 2 columns wide
        (6, 32, 8, 128, 64),  # 24 columns: 2 groups of 16, the last one half used
        (8, 64, 8, 128, 16),  # 64 columns: 4 groups of 16
        (5, 64, 8, 64, 32),   # 40 columns at dim 64: 3 groups
    ],
)
def test_query_column_groups(cuda_device, rows, q_heads, kv_heads, dim, page_tokens):
    """More query columns per KV head than one CTA holds (rows x group > 16,
    > 8 at dim 256): the tensor-core kernel runs one CTA per column group and
    KV range, with the rows' causal positions, against the FP64 oracle."""
    tokens = 1500
    qpos = [tokens - rows + r for r in range(rows)]
    case = make(cuda_device, rows=rows, q_heads=q_heads, kv_heads=kv_heads, dim=dim, page_tokens=page_tokens,
                tokens=tokens, seed=rows * 7 + dim, q_positions=qpos)
    assert kvb.attention_b200_supported(case.shape, case.device_input())
    ref = oracle.reference_case(case, threads=8)
    for partitions in (0, 3):
        res = run_single(case, partitions=partitions)
        check_against_oracle(res, case.shape, ref, f"groups {rows}x{q_heads // kv_heads} d{dim} P{partitions}")


def test_causal_visibility_of_every_row(cuda_device):
    """40 query rows with group 1 (five column groups) whose positions fall
    with the row index, so that the rows past the first 32 are the ones that
    see the fewest tokens: each CTA's whole-piece visibility test must cover
    the rows of its own columns."""
    tokens, rows = 3000, 40
    qpos = [tokens - 1 - 9 * r for r in range(rows)]
    case = make(cuda_device, rows=rows, q_heads=4, kv_heads=4, dim=128, page_tokens=64, tokens=tokens, seed=77,
                q_positions=qpos)
    assert kvb.attention_b200_supported(case.shape, case.device_input())
    ref = oracle.reference_case(case, threads=8)
    for partitions in (0, 7):
        res = run_single(case, partitions=partitions)
        check_against_oracle(res, case.shape, ref, f"falling positions P{partitions}")


def test_mma_launcher_contract(cuda_device):
    """launch_attention_mma keeps the reference predicate: its native shape
    runs, BASELINE shapes are rejected with ValueError before launch."""
    native = make(cuda_device, rows=8, q_heads=24, kv_heads=4, dim=256, page_tokens=32, tokens=600, seed=8,
                  q_positions=[592 + r for r in range(8)])
    assert kvb.attention_mma_supported(native.shape)
    res = run_single(native, api="mma", fp16_out=False)
    check_against_oracle(res, native.shape, oracle.reference_case(native, threads=8), "mma-native")
    base = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=256, seed=8)
    with pytest.raises(ValueError):
        run_single(base, api="mma", fp16_out=False)


def test_fp32_kv(cuda_device):
    case = make(cuda_device, rows=1, q_heads=8, kv_heads=2, dim=64, page_tokens=16, tokens=800, seed=12)
    kf = (case.k.float() * case.k_scales.unsqueeze(-1)).contiguous()
    vf = (case.v.float() * case.v_scales.unsqueeze(-2)).contiguous()
    shape = kvb.Shape(**{**case.shape.__dict__, "int8": False})
    fcase = synth.SingleCase(shape, case.q, case.q_positions, case.k_positions, case.page_table, kf, vf, None, None)
    res = run_single(fcase)
    ref = oracle.reference(shape, case.q, case.q_positions, case.k_positions, case.page_table, kf, vf)
    check_against_oracle(res, shape, ref, "fp32-kv")


def test_unaligned_buffers_use_general_kernel(cuda_device):
    case = make(cuda_device, rows=1, q_heads=8, kv_heads=2, dim=128, page_tokens=64, tokens=500, seed=13)
    kbuf = torch.empty(case.k.numel() + 4, dtype=torch.int8, device=cuda_device)
    kbuf[4:] = case.k.reshape(-1)
    shifted = synth.SingleCase(case.shape, case.q, case.q_positions, case.k_positions, case.page_table,
                               kbuf[4:], case.v, case.k_scales, case.v_scales)
    assert not kvb.attention_b200_supported(shifted.shape, shifted.device_input())
    res = run_single(shifted)
    check_against_oracle(res, case.shape, oracle.reference_case(case, threads=8), "unaligned")


def test_invalid_arguments_raise_before_launch(cuda_device):
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=256, seed=1)
    scratch, m, l, n = outputs_for(case.shape, cuda_device)
    bad = kvb.Shape(**{**case.shape.__dict__, "dim": 257})
    with pytest.raises(ValueError, match="dim must be in"):
        kvb.launch_attention(bad, case.device_input(), scratch, m, l, n)
    inp = case.device_input()
    inp.k = None
    with pytest.raises(ValueError, match="non-null"):
        kvb.launch_attention(case.shape, inp, scratch, m, l, n)
    with pytest.raises(ValueError, match="split count"):
        kvb.merge_attention(case.shape, scratch, 7, m, l, n)


@pytest.mark.parametrize(
    "q_heads,kv_heads,dim,page_tokens,outliers",
    [
        (32, 8, 128, 64, 0.0),   # cfg3 flavour
        (64, 8, 128, 16, 0.01),  # cfg4 flavour: GQA 8, Page16 (four-page gather loads), outliers
        (16, 2, 64, 16, 0.0),    # dim 64, Page16
        (24, 8, 256, 32, 0.0),   # group 3 (four-column layout), dim 256
        (8, 8, 128, 64, 0.01),   # group 1 (four-column layout), outliers
    ],
)
def test_batched_ragged(cuda_device, q_heads, kv_heads, dim, page_tokens, outliers):
    """Ragged batch over one shared shuffled page pool; lengths that end
    inside a stage or a page take the per-page copies beside the gathers."""
    lens = synth.ragged_lengths(12, 1, 5000, seed=31) + [0, 64, 65, 17, 4096]
    bc = synth.make_batched(q_heads, kv_heads, dim, page_tokens, lens, seed=0xC0FFEE + 3, device=cuda_device,
                            outlier_frac=outliers)
    P, Hkv = page_tokens, kv_heads
    ws_bytes = kvb.batch_workspace_bytes(bc.shape)
    ws = torch.empty(ws_bytes // 4 + 1, dtype=torch.float32, device=cuda_device)
    B, H, D = bc.shape.batch, bc.shape.q_heads, bc.shape.dim
    m = torch.empty(B * H, device=cuda_device)
    l = torch.empty(B * H, device=cuda_device)
    n = torch.empty(B * H * D, device=cuda_device)
    out = torch.empty(B * H * D, dtype=torch.float16, device=cuda_device)
    kvb.launch_attention_batched(bc.shape, bc.batch_input(), ws, ws_bytes, m, l, n, out)
    torch.cuda.synchronize()
    m, l, n, out = m.cpu(), l.cpu(), n.cpu(), out.cpu()
    for b, length in enumerate(lens):
        sl = slice(b * H, (b + 1) * H)
        if length == 0:
            assert torch.all(l[sl] == 0) and torch.all(torch.isneginf(m[sl]))
            continue
        npg = (length + P - 1) // P
        table = bc.block_table[b, :npg].cpu()
        shape = kvb.Shape(1, H, Hkv, D, P, bc.shape.pages, length, 0, length, bc.shape.scale, True)
        ref = oracle.reference(shape, bc.q[b].cpu(), torch.tensor([length - 1]), torch.arange(length),
                               torch.cat([table, torch.zeros(bc.shape.pages - npg, dtype=torch.int32)]),
                               bc.k.cpu(), bc.v.cpu(), bc.k_scales.cpu(), bc.v_scales.cpu(), threads=8)
        res = {"m": m[sl], "l": l[sl], "n": n[b * H * D:(b + 1) * H * D],
               "out": out[b * H * D:(b + 1) * H * D]}
        check_against_oracle(res, shape, ref, f"batch{b}")


def test_shard_merge_matches_full_range(cuda_device):
    """Sequence sharding: four disjoint page-aligned ranges computed
    separately and merged with merge_attention_shards equal the full call."""
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=8192, seed=55)
    cuts = [0, 2048, 4096, 6144, 8192]
    parts = []
    for a, b in zip(cuts[:-1], cuts[1:]):
        shape = kvb.Shape(**{**case.shape.__dict__, "begin": a, "end": b})
        sub = synth.SingleCase(shape, case.q, case.q_positions, case.k_positions, case.page_table,
                               case.k, case.v, case.k_scales, case.v_scales)
        parts.append(run_single(sub, fp16_out=False))
    mp = torch.stack([p["m"] for p in parts]).to(cuda_device)
    lp = torch.stack([p["l"] for p in parts]).to(cuda_device)
    npart = torch.stack([p["n"] for p in parts]).to(cuda_device)
    rh, D = 32, 128
    m = torch.empty(rh, device=cuda_device)
    l = torch.empty(rh, device=cuda_device)
    n = torch.empty(rh * D, device=cuda_device)
    out = torch.empty(rh * D, dtype=torch.float16, device=cuda_device)
    kvb.merge_attention_shards(4, rh, D, mp, lp, npart, m, l, n, out)
    torch.cuda.synchronize()
    res = {"m": m.cpu(), "l": l.cpu(), "n": n.cpu(), "out": out.cpu()}
    check_against_oracle(res, case.shape, oracle.reference_case(case, threads=8), "shards")


@pytest.mark.skipif(not oracle.RefCuda.available(), reason="reference CUDA build absent")
def test_matches_reference_simt_kernel(cuda_device):
    """Same device inputs through the reference's own SIMT launcher (compiled
    for sm_100a from its sources) and through ours: n/l agree within the
    path tolerance."""
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=4096, seed=0xC0FFEE + 1)
    ours = run_single(case)
    ref_gpu = oracle.RefCuda()
    scratch, m, l, n = outputs_for(case.shape, cuda_device)
    ptrs = [t.data_ptr() for t in (case.q, case.q_positions, case.k_positions, case.page_table,
                                   case.k, case.v, case.k_scales, case.v_scales)]
    rc = ref_gpu.launch(case.shape, ptrs, scratch.data_ptr(), m.data_ptr(), l.data_ptr(), n.data_ptr(), 0)
    assert rc == 0
    torch.cuda.synchronize()
    theirs = {"m": m.cpu(), "l": l.cpu(), "n": n.cpu()}
    ma, rl = errors(normalized(ours, case.shape), normalized(theirs, case.shape))
    assert ma <= MAX_ABS and rl <= REL_L2, (ma, rl)
    ref = oracle.reference_case(case, threads=8)
    ma_ref, rl_ref = errors(normalized(theirs, case.shape), ref["normalized"])
    assert ma_ref <= MAX_ABS and rl_ref <= REL_L2, (ma_ref, rl_ref)


def test_pipeline_graph_replay_stress(cuda_device):
    """Back-to-back calls over several KV layers, replayed as a CUDA graph:
    the copy ring must never let a warp pass a stage that has not landed
    (the bounded waits would record it in the status word), and every replay
    must reproduce the eager results bit for bit."""
    layers = [make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=65536,
                   seed=900 + i) for i in range(3)]
    shape = layers[0].shape
    scratch, m, l, n = outputs_for(shape, cuda_device)
    outs = [torch.empty(kvb.output_numerator_elements(shape), dtype=torch.float16, device=cuda_device)
            for _ in layers]
    inputs = [c.device_input() for c in layers]
    stream = torch.cuda.Stream(device=cuda_device)
    with torch.cuda.stream(stream):
        for i, inp in enumerate(inputs):
            kvb.launch_attention_ex(shape, inp, scratch, m, l, n, out_f16=outs[i])
    torch.cuda.synchronize()
    eager = [o.clone() for o in outs]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for rep in range(8):
            for i, inp in enumerate(inputs):
                kvb.launch_attention_ex(shape, inp, scratch, m, l, n, out_f16=outs[i])
    for o in outs:
        o.zero_()
    with torch.cuda.stream(stream):
        for _ in range(10):
            graph.replay()
    torch.cuda.synchronize()
    assert kvb.read_device_status() == 0, kvb.read_wait_failure()
    for a, b in zip(outs, eager):
        assert torch.equal(a, b)


@pytest.mark.parametrize("name", __import__("golden_util").golden_names())
def test_golden_vectors(cuda_device, name):
    """The committed golden vectors (expected outputs computed by the
    reference's own FP64 oracle) through the C ABI."""
    from golden_util import load

    g = load(name)
    s = kvb.Shape(**g["shape"])
    dev = cuda_device
    case = synth.SingleCase(
        s, torch.from_numpy(g["q"]).to(dev), torch.from_numpy(g["q_positions"]).to(dev),
        torch.from_numpy(g["k_positions"]).to(dev),
        torch.from_numpy(g["page_table"].astype(np.int64)).to(torch.int32).to(dev),
        torch.from_numpy(g["k"]).to(dev), torch.from_numpy(g["v"]).to(dev),
        torch.from_numpy(g["k_scales"]).to(dev), torch.from_numpy(g["v_scales"]).to(dev))
    for api in ("ex", "ref"):
        res = run_single(case, fp16_out=(api == "ex"), api=api)
        ref = {"normalized": g["normalized"], "visible": g["visible"],
               "m": None, "l": None}
        got = normalized(res, s)
        vis = res["l"].numpy().reshape(s.rows, s.q_heads) > 0
        assert np.array_equal(vis, g["visible"]), name
        ma, rl = errors(got, g["normalized"])
        assert ma <= MAX_ABS and rl <= REL_L2, (name, api, ma, rl)


def test_negative_and_mixed_sign_v_scales(cuda_device):
    """The contract asks for finite scales only; negative V scales flip the
    sign of P, which the signed fixed-point P limbs carry."""
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=32, tokens=3000, seed=61)
    flip = torch.rand(case.v_scales.shape, generator=torch.Generator(device=cuda_device).manual_seed(5),
                      device=cuda_device) < 0.3
    case.v_scales[flip] *= -1.0
    res = run_single(case)
    check_against_oracle(res, case.shape, oracle.reference_case(case, threads=8), "neg-vscale")


def _scratch_garbage(shape, device, seed):
    """A scratch full of arbitrary bit patterns (NaNs and infinities included)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    bits = torch.randint(-2**31, 2**31 - 1, (kvb.scratch_elements(shape),), generator=g, dtype=torch.int32)
    return bits.view(torch.float32).to(device)


def _close(a, b):
    """Same partials merged over more (empty) splits: equal to fp32 rounding."""
    return torch.allclose(a, b, rtol=1e-5, atol=1e-6 * float(b.abs().max()))


def test_uninitialised_scratch_repeats_and_full_remerge(cuda_device):
    """An arbitrary initial scratch (NaN and infinity bit patterns included),
    repeated calls on the same scratch and the two halves called separately
    (partials, then merge_attention_ex) all agree bit for bit; merge_attention
    over all split_count splits of the scratch afterwards (live partials plus
    the empty-split markers, whose n is left undefined) reproduces the
    result."""
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=16384, seed=77)
    shape = case.shape
    splits = kvb.split_count(shape)
    inp = case.device_input()
    assert kvb.attention_partitions(shape, 0) < splits
    ref = oracle.reference_case(case, threads=8)
    results = []
    for seed in (1, 2):
        scratch = _scratch_garbage(shape, cuda_device, seed)
        _, m, l, n = outputs_for(shape, cuda_device)
        out = torch.empty(kvb.output_numerator_elements(shape), dtype=torch.float16, device=cuda_device)
        for _ in range(3):
            kvb.launch_attention_ex(shape, inp, scratch, m, l, n, out_f16=out)
            torch.cuda.synchronize()
            res = {"m": m.cpu(), "l": l.cpu(), "n": n.cpu(), "out": out.cpu()}
            check_against_oracle(res, shape, ref, "garbage-scratch")
            results.append(res)
        # Re-merge everything the scratch holds (live partials + empty markers).
        _, m2, l2, n2 = outputs_for(shape, cuda_device)
        kvb.merge_attention(shape, scratch, splits, m2, l2, n2)
        torch.cuda.synchronize()
        assert torch.equal(m2.cpu(), res["m"])
        assert _close(l2.cpu(), res["l"]) and _close(n2.cpu(), res["n"])
    for r in results[1:]:
        for k in ("m", "l", "n", "out"):
            assert torch.equal(r[k], results[0][k]), k
    # The two halves called separately.
    scratch, m3, l3, n3 = outputs_for(shape, cuda_device)
    parts = kvb.launch_attention_partials(shape, inp, scratch)
    kvb.merge_attention_ex(shape, scratch, parts, m3, l3, n3)
    torch.cuda.synchronize()
    for k, v in (("m", m3), ("l", l3), ("n", n3)):
        assert torch.equal(v.cpu(), results[0][k]), k


@pytest.mark.parametrize("rows,q_heads,kv_heads,dim,page_tokens,tokens",
                         [(1, 32, 8, 128, 64, 16384), (3, 24, 4, 256, 32, 9000), (5, 64, 8, 64, 16, 5000)])
def test_partials_mark_every_other_split_empty(cuda_device, rows, q_heads, kv_heads, dim, page_tokens, tokens):
    """launch_attention_partials alone (no merge_attention_ex) leaves a
    complete reference scratch: every split past the partitions used reads as
    an empty partial (m = -inf, l = 0), so a merge over all split_count splits
    of a garbage-initialised scratch reproduces launch_attention_ex."""
    qpos = [tokens - rows + r for r in range(rows)] if rows > 1 else None
    case = make(cuda_device, rows=rows, q_heads=q_heads, kv_heads=kv_heads, dim=dim, page_tokens=page_tokens,
                tokens=tokens, seed=tokens + dim, q_positions=qpos)
    shape = case.shape
    splits = kvb.split_count(shape)
    inp = case.device_input()
    scratch = _scratch_garbage(shape, cuda_device, 9)
    want = max(1, splits // 3)  # fewer partitions than splits, whichever kernel runs
    parts = kvb.launch_attention_partials(shape, inp, scratch, partitions=want)
    assert 0 < parts < splits
    rows_view = scratch.view(kvb.output_scalar_elements(shape), splits, dim + 2)
    torch.cuda.synchronize()
    assert torch.all(rows_view[:, parts:, 0].cpu() == float("-inf"))
    assert torch.all(rows_view[:, parts:, 1].cpu() == 0)
    _, m, l, n = outputs_for(shape, cuda_device)
    kvb.merge_attention(shape, scratch, splits, m, l, n)
    _, m2, l2, n2 = outputs_for(shape, cuda_device)
    kvb.launch_attention_ex(shape, inp, _scratch_garbage(shape, cuda_device, 10), m2, l2, n2, partitions=want)
    torch.cuda.synchronize()
    assert torch.equal(m.cpu(), m2.cpu())
    assert _close(l.cpu(), l2.cpu()) and _close(n.cpu(), n2.cpu())


def test_independent_streams(cuda_device):
    """Calls on two streams with their own scratch buffers run concurrently
    without sharing state: interleaved launches reproduce each case's own
    result bit for bit."""
    cases = [make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=32768,
                  seed=500 + i) for i in range(2)]
    shape = cases[0].shape
    bufs = [outputs_for(shape, cuda_device) for _ in cases]
    outs = [torch.empty(kvb.output_numerator_elements(shape), dtype=torch.float16, device=cuda_device)
            for _ in cases]
    for c, (sc, m, l, n), o in zip(cases, bufs, outs):
        kvb.launch_attention_ex(shape, c.device_input(), sc, m, l, n, out_f16=o)
    torch.cuda.synchronize()
    expect = [o.clone() for o in outs]
    for o in outs:
        o.zero_()
    streams = [torch.cuda.Stream(device=cuda_device) for _ in cases]
    for _ in range(20):
        for c, (sc, m, l, n), o, st in zip(cases, bufs, outs, streams):
            with torch.cuda.stream(st):
                kvb.launch_attention_ex(shape, c.device_input(), sc, m, l, n, out_f16=o)
    torch.cuda.synchronize()
    for o, e in zip(outs, expect):
        assert torch.equal(o, e)


@pytest.mark.parametrize("page_tokens", [64, 16])
def test_bf16_output(cuda_device, page_tokens):
    """The bf16 epilogue (beside the fp16 one): each element is n * (1 / l)
    in fp32 rounded to nearest-even bf16, within the path tolerance of the
    FP64 oracle; both outputs come from the same merge."""
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=page_tokens, tokens=6000,
                seed=0xC0FFEE + 9)
    s = case.shape
    scratch, m, l, n = outputs_for(s, cuda_device)
    nd = kvb.output_numerator_elements(s)
    out16 = torch.full((nd,), float("nan"), dtype=torch.float16, device=cuda_device)
    outbf = torch.full((nd,), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    kvb.launch_attention_ex(s, case.device_input(), scratch, m, l, n, out_f16=out16, out_bf16=outbf)
    torch.cuda.synchronize()
    ref = oracle.reference_case(case, threads=8)
    res = {"m": m.cpu(), "l": l.cpu(), "n": n.cpu(), "out": out16.cpu()}
    check_against_oracle(res, s, ref, "bf16 run")
    from kvb_testutil import check_bf16

    check_bf16(outbf.cpu(), s, ref, "bf16")
    lh = res["l"].repeat_interleave(s.dim)
    expect = (res["n"] * torch.where(lh > 0, 1.0 / lh, torch.zeros_like(lh))).to(torch.bfloat16)
    assert torch.equal(outbf.cpu().view(torch.int16), expect.view(torch.int16))
    # bf16 alone (no fp16 buffer) through merge_attention_ex over the same scratch.
    outbf2 = torch.empty_like(outbf)
    _, m2, l2, n2 = outputs_for(s, cuda_device)
    parts = kvb.attention_partitions(s, 0)
    kvb.merge_attention_ex(s, scratch, parts, m2, l2, n2, out_bf16=outbf2)
    torch.cuda.synchronize()
    assert torch.equal(outbf2.cpu().view(torch.int16), outbf.cpu().view(torch.int16))


def test_packed_shard_merge(cuda_device):
    """Sequence sharding with one packed exchange buffer per rank
    ([m | l | n] of every row-head, as one all-gather delivers them): the
    strided shard merge equals the separate-array merge bit for bit and the
    full-range result within tolerance."""
    case = make(cuda_device, rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=8192, seed=56)
    rh, D = 32, 128
    cuts = [0, 1024, 4096, 6144, 8192]
    packed = torch.empty(len(cuts) - 1, rh * (D + 2), device=cuda_device)
    for i, (a, b) in enumerate(zip(cuts[:-1], cuts[1:])):
        shape = kvb.Shape(**{**case.shape.__dict__, "begin": a, "end": b})
        scratch = torch.empty(kvb.scratch_elements(shape), device=cuda_device)
        blk = packed[i]
        kvb.launch_attention_ex(shape, case.device_input(), scratch, blk[:rh], blk[rh:2 * rh], blk[2 * rh:])
    outs = []
    for stride, parts in ((rh * (D + 2), (packed, packed[:, rh:], packed[:, 2 * rh:])),
                          (0, (packed[:, :rh].contiguous(), packed[:, rh:2 * rh].contiguous(),
                               packed[:, 2 * rh:].contiguous()))):
        m = torch.empty(rh, device=cuda_device)
        l = torch.empty(rh, device=cuda_device)
        n = torch.empty(rh * D, device=cuda_device)
        out = torch.empty(rh * D, dtype=torch.float16, device=cuda_device)
        kvb.merge_attention_shards_ex(len(cuts) - 1, rh, D, *parts, stride, m, l, n, out_f16=out)
        torch.cuda.synchronize()
        outs.append({"m": m.cpu(), "l": l.cpu(), "n": n.cpu(), "out": out.cpu()})
    for k in ("m", "l", "n", "out"):
        assert torch.equal(outs[0][k], outs[1][k]), k
    check_against_oracle(outs[0], case.shape, oracle.reference_case(case, threads=8), "packed shards")
