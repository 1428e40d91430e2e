"""Host shape layer: bit-exact parity with the reference (no GPU needed).

1. The checks of the reference's tests/shape_test.cpp:29-89 restated through
   this library's C ABI.
2. The reference's own tests/shape_test.cpp compiled unchanged against this
   repository's include/kvbridge headers and shape implementation.
3. Randomised and boundary shapes: error message, sizes and the MMA
   predicate equal the reference's compiled shape layer (oracle/_ref).
"""
from __future__ import annotations

import random
import subprocess
from pathlib import Path

import pytest

import kvbridge_b200 as kvb
import oracle

ROOT = Path(__file__).resolve().parents[1]
REF = oracle.REFERENCE_DIR
U32 = 0xFFFFFFFF

BASE = dict(rows=8, q_heads=24, kv_heads=4, dim=256, page_tokens=32, pages=2048, tokens=65536,
            begin=0, end=65536, scale=0.0625, int8=True)


def shape(**kw):
    return kvb.Shape(**{**BASE, **kw})


def rejected(s):
    assert not kvb.attention_shape_valid(s)
    assert kvb.attention_shape_error(s) is not None
    assert not kvb.attention_mma_supported(s)
    with pytest.raises(ValueError):
        kvb.scratch_elements(s)


def test_reference_shape_checks(kvb_lib):
    base = shape()
    assert kvb.attention_shape_valid(base)
    assert kvb.attention_mma_supported(base)
    assert kvb.split_count(base) == 256
    assert kvb.output_scalar_elements(base) == 192
    assert kvb.output_numerator_elements(base) == 49152
    assert kvb.scratch_elements(base) == 192 * 256 * 258

    for kw in [
        dict(rows=0), dict(q_heads=0), dict(kv_heads=0), dict(q_heads=25), dict(kv_heads=48),
        dict(dim=0), dict(dim=257), dict(pages=0), dict(page_tokens=0), dict(tokens=0, end=0),
        dict(begin=33, end=32), dict(end=65537), dict(pages=2047), dict(scale=float("inf")),
        dict(scale=float("nan")), dict(rows=U32), dict(pages=U32), dict(kv_heads=0xFFFFFFFE, q_heads=0xFFFFFFFE),
    ]:
        rejected(shape(**kw))

    s = shape(begin=32, end=32)
    assert kvb.attention_shape_valid(s) and kvb.attention_mma_supported(s)
    assert kvb.split_count(s) == 1 and kvb.scratch_elements(s) == 192 * 258
    s = shape(begin=32, end=33)
    assert kvb.attention_mma_supported(s) and kvb.split_count(s) == 1
    assert kvb.split_count(shape(begin=32, end=289)) == 2
    s = shape(begin=31, end=289)
    assert kvb.attention_shape_valid(s) and not kvb.attention_mma_supported(s)
    for kw in [dict(int8=False), dict(rows=1), dict(dim=1), dict(q_heads=36)]:
        s = shape(**kw)
        assert kvb.attention_shape_valid(s) and not kvb.attention_mma_supported(s)
    assert kvb.attention_mma_supported(shape(tokens=65535, end=65535))
    big = kvb.Shape(1, 1, 1, 1, 256, 65536, 16777216, 0, 16776960, 1.0, True)
    assert kvb.split_count(big) == 65535
    rejected(kvb.Shape(1, 1, 1, 1, 256, 65536, 16777216, 0, 16776961, 1.0, True))
    edge = kvb.Shape(1, 1, 1, 1, 1, U32, U32, 0xFFFFFFFE, U32, 1.0, True)
    assert kvb.split_count(edge) == 1
    edge.begin = edge.end
    assert kvb.split_count(edge) == 1


def test_error_messages_and_exception_kind(kvb_lib):
    with pytest.raises(ValueError, match="q_heads must be divisible by kv_heads"):
        kvb.validate_shape(shape(q_heads=25))
    assert kvb.attention_shape_error(shape(dim=257)) == "dim must be in [1,256]"
    assert kvb.attention_shape_error(shape()) is None


@pytest.mark.skipif(not (REF / "tests" / "shape_test.cpp").exists(), reason="reference sources absent")
def test_reference_shape_test_binary_against_our_layer(tmp_path):
    exe = tmp_path / "shape_test"
    subprocess.run(
        ["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}",
         str(REF / "tests" / "shape_test.cpp"), str(ROOT / "kvbridge_b200" / "csrc" / "attention_shape.cpp"),
         "-o", str(exe)],
        check=True,
    )
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True)
    assert out.stdout.startswith("PASS 98 host shape/API checks")


BOUNDARY = [0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 15, 16, 31, 32, 33, 63, 64, 65, 127, 128, 255, 256, 257, 4096,
            65535, 65536, 65537, 16776960, 16777216, 0x7FFFFFFF, 0x80000000, 0xFFFFFFFE, U32]


def random_shape(rng: random.Random) -> dict:
    def pick():
        if rng.random() < 0.5:
            return rng.choice(BOUNDARY)
        return rng.randrange(0, 1 << rng.choice([4, 8, 12, 16, 20, 24, 32]))

    f = {k: pick() for k in ("rows", "q_heads", "kv_heads", "dim", "page_tokens", "pages", "tokens")}
    if rng.random() < 0.6:  # mostly plausible geometry so deep checks are reached
        f["kv_heads"] = rng.choice([1, 2, 4, 8])
        f["q_heads"] = f["kv_heads"] * rng.choice([1, 2, 4, 6, 8, 9])
        f["dim"] = rng.choice([1, 64, 128, 256, 257])
        f["page_tokens"] = rng.choice([16, 32, 64, 256])
        f["rows"] = rng.choice([1, 8, 0x7FFFFFFF])
        f["tokens"] = rng.randrange(1, 1 << 25)
        f["pages"] = -(-f["tokens"] // f["page_tokens"]) + rng.choice([0, 0, 1, -1])
        f["pages"] = max(0, min(U32, f["pages"]))
    f["end"] = rng.choice([f["tokens"], rng.randrange(0, max(1, f["tokens"] + 2)), pick()])
    f["begin"] = rng.choice([0, rng.randrange(0, f["end"] + 2), f["end"], pick()])
    f["end"] = min(f["end"], U32)
    f["begin"] = min(f["begin"], U32)
    f["scale"] = rng.choice([0.0625, 1.0, float("inf"), float("nan"), -3.0])
    f["int8"] = rng.random() < 0.8
    return f


@pytest.mark.skipif(not oracle.RefOracle.available(), reason="reference oracle build absent")
def test_fuzz_parity_with_reference_shape_layer(kvb_lib):
    ref = oracle.RefOracle()
    rng = random.Random(20261201)
    valid = 0
    for _ in range(20000):
        f = random_shape(rng)
        ours = kvb.Shape(**f)
        err = kvb.attention_shape_error(ours)
        assert err == ref.shape_error(f), f
        assert kvb.attention_mma_supported(ours) == ref.mma_supported(f), f
        sizes = ref.sizes(f)
        if sizes is None:
            assert err is not None
            with pytest.raises(ValueError):
                kvb.split_count(ours)
        else:
            valid += 1
            assert (kvb.split_count(ours), kvb.scratch_elements(ours), kvb.output_scalar_elements(ours),
                    kvb.output_numerator_elements(ours)) == sizes, f
    assert valid > 1000
