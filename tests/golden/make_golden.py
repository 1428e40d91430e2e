#!/usr/bin/env python3
"""Generates the golden vectors in tests/golden/*.npz.

Each case's inputs come from kvbridge_b200.synth (seeded, CPU) or from the
reference's deterministic fixture (oracle.make_reference_fixture), and its
expected output is computed by the REFERENCE'S OWN FP64 oracle
(kvbridge_example::reference(), compiled from the reference sources into
oracle/_ref by oracle/Makefile). Inputs are stored with the outputs so the
fixtures do not depend on the generator's RNG.

Run from the repository root where the reference sources are available:
    python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from kvbridge_b200 import synth  # noqa: E402

FIELDS = ("rows", "q_heads", "kv_heads", "dim", "page_tokens", "pages", "tokens", "begin", "end")


def synth_case(**kw):
    c = synth.make_single(device="cpu", **kw)
    s = c.shape
    return dict(
        shape={f: getattr(s, f) for f in FIELDS} | {"scale": s.scale, "int8": True},
        q=c.q.numpy().reshape(-1), q_positions=c.q_positions.numpy(), k_positions=c.k_positions.numpy(),
        page_table=c.page_table.numpy().astype(np.uint32), k=c.k.numpy().reshape(-1),
        v=c.v.numpy().reshape(-1), k_scales=c.k_scales.numpy().reshape(-1), v_scales=c.v_scales.numpy().reshape(-1),
    )


CASES = {
    # BASELINE cfg1 geometry (dim 128, GQA 4, Page64, shuffled), short context.
    "g1_gqa4_p64": lambda: synth_case(rows=1, q_heads=16, kv_heads=4, dim=128, page_tokens=64, tokens=192, seed=101),
    # Two query rows, causal mask inside the range, mid-page begin, Page16.
    "g2_rows2_p16_causal": lambda: synth_case(rows=2, q_heads=8, kv_heads=2, dim=64, page_tokens=16, tokens=300,
                                              begin=17, end=290, q_positions=[150, 299], seed=102),
    # GQA 8 with 10x outlier tokens (cfg4 flavour), Page16.
    "g3_gqa8_outliers": lambda: synth_case(rows=1, q_heads=16, kv_heads=2, dim=128, page_tokens=16, tokens=256,
                                           outlier_frac=0.05, seed=103),
    # The reference's own deterministic fixture (rows 8, 24/4, dim 256, Page32), reversed pages.
    "g4_reference_fixture": lambda: oracle.make_reference_fixture(64, permute=True),
    # Fully masked rows (q position before every key) and partial visibility.
    "g5_masked_rows": lambda: synth_case(rows=2, q_heads=4, kv_heads=1, dim=64, page_tokens=32, tokens=100,
                                         q_positions=[-1, 40], seed=105),
}


def main() -> None:
    ref = oracle.RefOracle()
    for name, make in CASES.items():
        c = make()
        run = ref.prepare(c["shape"], c["q"], c["q_positions"], c["k_positions"], c["page_table"],
                          c["k"], c["v"], c["k_scales"], c["v_scales"])
        run.run(1)
        res = run.result()
        s = c["shape"]
        np.savez_compressed(
            HERE / f"{name}.npz",
            shape=np.array([s[f] for f in FIELDS], dtype=np.uint32),
            scale=np.float32(s["scale"]),
            q=c["q"], q_positions=c["q_positions"], k_positions=c["k_positions"], page_table=c["page_table"],
            k=c["k"], v=c["v"], k_scales=c["k_scales"], v_scales=c["v_scales"],
            normalized=res["normalized"], visible=res["visible"],
        )
        print(name, "written")


if __name__ == "__main__":
    main()
