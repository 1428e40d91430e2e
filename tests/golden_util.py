"""Loader of the golden vectors in tests/golden (see tests/golden/make_golden.py)."""
from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
FIELDS = ("rows", "q_heads", "kv_heads", "dim", "page_tokens", "pages", "tokens", "begin", "end")


def golden_names():
    return sorted(p.stem for p in GOLDEN.glob("*.npz"))


def load(name: str) -> dict:
    z = np.load(GOLDEN / f"{name}.npz")
    shape = {f: int(v) for f, v in zip(FIELDS, z["shape"])}
    shape["scale"] = float(z["scale"])
    shape["int8"] = True
    out = {k: z[k] for k in z.files if k not in ("shape", "scale")}
    out["shape"] = shape
    return out
