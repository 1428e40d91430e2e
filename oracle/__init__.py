"""TEST INFRASTRUCTURE - CPU checkers for kvbridge-b200.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this package, and only as the checker; the product path never calls it.

* ``reference()``  - this repository's FP64 C oracle (oracle/kvb_oracle.c),
  a restatement of the reference's ``kvbridge_example::reference()``
  (examples/attention_reference.h:53-89).
* ``RefOracle``    - the reference's own oracle and host shape layer, compiled
  from the reference sources into oracle/_ref (present only where the
  reference was available at build time).
* ``RefCuda``      - the reference's own CUDA launchers compiled for sm_100a.
* ``make_reference_fixture()`` - the reference's deterministic fixture
  generator (examples/attention_reference.h:19-48) restated in numpy.
* ``append_kv()``  - the paged KV append (absmax int8 quantisation into the
  pool layout) restated in C; the reference ships no quantiser, so this
  follows the benchmark configurations' stated rule and is cross-checked
  against the independent torch restatement in kvbridge_b200.synth.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_int32, c_uint8, c_uint32, c_uint64, c_void_p
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
# The reference checkout the checkers are built from: $KVB_REFERENCE_DIR when
# set, else a directory named `reference` beside this repository. Only build
# steps read it; nothing at test or bench time does.
REFERENCE_DIR = Path(os.environ.get("KVB_REFERENCE_DIR") or (HERE.parent.parent / "reference"))
ORACLE_LIB = HERE / "libkvb_oracle.so"
REF_ORACLE_LIB = HERE / "_ref" / "libkvbref_oracle.so"
REF_CUDA_LIB = HERE / "_ref" / "libkvbref_cuda.so"


class _Shape(ctypes.Structure):
    _fields_ = [
        ("rows", c_uint32),
        ("q_heads", c_uint32),
        ("kv_heads", c_uint32),
        ("dim", c_uint32),
        ("page_tokens", c_uint32),
        ("pages", c_uint32),
        ("tokens", c_uint32),
        ("begin", c_uint32),
        ("end", c_uint32),
        ("scale", c_float),
        ("int8", c_int32),
    ]


class _Inputs(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("q", "qpos", "kpos", "table", "k", "v", "ks", "vs")]


class _Outputs(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("normalized", "m", "l", "visible")]


_oracle = None


def build(ref: bool = False) -> None:
    """Run oracle/Makefile (the C oracle; with ``ref`` also oracle/_ref)."""
    target = "all" if ref else "oracle"
    subprocess.run(["make", "-s", "-C", str(HERE), target, f"REF={REFERENCE_DIR}"], check=True)


def _load_oracle():
    global _oracle
    if _oracle is None:
        if not ORACLE_LIB.exists():
            build()
        lib = ctypes.CDLL(str(ORACLE_LIB))
        lib.kvbo_reference.restype = c_int
        lib.kvbo_reference.argtypes = [POINTER(_Shape), POINTER(_Inputs), POINTER(_Outputs), c_int]
        lib.kvbo_merge.restype = None
        lib.kvbo_merge.argtypes = [c_uint32, c_uint32, c_uint32] + [c_void_p] * 6
        lib.kvbo_append_kv.restype = c_int
        lib.kvbo_append_kv.argtypes = [c_uint32] * 5 + [c_void_p] * 7
        _oracle = lib
    return _oracle


def _np(x, dtype):
    if hasattr(x, "detach"):
        x = x.detach().cpu().numpy()
    return np.ascontiguousarray(np.asarray(x), dtype=dtype)


def shape_fields(shape) -> dict:
    names = ("rows", "q_heads", "kv_heads", "dim", "page_tokens", "pages", "tokens", "begin", "end", "scale", "int8")
    if isinstance(shape, dict):
        return {n: shape[n] for n in names}
    return {n: getattr(shape, n) for n in names}


def reference(shape, q, q_positions, k_positions, page_table, k, v, k_scales=None, v_scales=None, threads: int = 1):
    """FP64 oracle output: dict(normalized [rows,q_heads,dim], m, l, visible)."""
    f = shape_fields(shape)
    int8 = bool(f["int8"])
    arrs = [
        _np(q, np.float32),
        _np(q_positions, np.int64),
        _np(k_positions, np.int64),
        _np(page_table, np.int64).astype(np.uint32),
        _np(k, np.int8 if int8 else np.float32),
        _np(v, np.int8 if int8 else np.float32),
        _np(k_scales, np.float32) if int8 else np.zeros(1, np.float32),
        _np(v_scales, np.float32) if int8 else np.zeros(1, np.float32),
    ]
    rh = f["rows"] * f["q_heads"]
    out_n = np.zeros((f["rows"], f["q_heads"], f["dim"]), np.float64)
    out_m = np.zeros(rh, np.float64)
    out_l = np.zeros(rh, np.float64)
    vis = np.zeros(rh, np.uint8)
    s = _Shape(*(int(f[n]) for n, _ in _Shape._fields_[:9]), float(f["scale"]), int(int8))
    ins = _Inputs(*(a.ctypes.data for a in arrs))
    outs = _Outputs(out_n.ctypes.data, out_m.ctypes.data, out_l.ctypes.data, vis.ctypes.data)
    rc = _load_oracle().kvbo_reference(ctypes.byref(s), ctypes.byref(ins), ctypes.byref(outs), threads)
    if rc != 0:
        raise RuntimeError(f"oracle failed with status {rc}")
    return {
        "normalized": out_n,
        "m": out_m.reshape(f["rows"], f["q_heads"]),
        "l": out_l.reshape(f["rows"], f["q_heads"]),
        "visible": vis.reshape(f["rows"], f["q_heads"]).astype(bool),
    }


def reference_case(case, threads: int = 1):
    """Oracle of a kvbridge_b200.synth.SingleCase."""
    return reference(
        case.shape, case.q, case.q_positions, case.k_positions, case.page_table,
        case.k, case.v, case.k_scales, case.v_scales, threads=threads,
    )


def merge(m_parts, l_parts, n_parts):
    """FP64 log-sum-exp merge; m/l [parts, rh], n [parts, rh, dim]."""
    m_parts = _np(m_parts, np.float64)
    l_parts = _np(l_parts, np.float64)
    n_parts = _np(n_parts, np.float64)
    parts, rh = m_parts.shape
    dim = n_parts.shape[-1]
    m = np.zeros(rh)
    l = np.zeros(rh)
    n = np.zeros((rh, dim))
    _load_oracle().kvbo_merge(parts, rh, dim, m_parts.ctypes.data, l_parts.ctypes.data,
                              n_parts.ctypes.data, m.ctypes.data, l.ctypes.data, n.ctypes.data)
    return m, l, n


def make_reference_fixture(tokens: int, permute: bool = False) -> dict:
    """The reference's deterministic fixture (examples/attention_reference.h:19-48):
    rows 8, 24 q / 4 kv heads, dim 256, 32-token pages, scale 1/16, bf16-exact
    Q = ((i*7)%257 - 128)/1024, patterned int8 K/V and rational scales."""
    rows, qh, kvh, dim, P = 8, 24, 4, 256, 32
    pages = (tokens + 31) // 32
    shape = dict(rows=rows, q_heads=qh, kv_heads=kvh, dim=dim, page_tokens=P, pages=pages,
                 tokens=tokens, begin=0, end=tokens, scale=0.0625, int8=True)
    table = np.array([pages - 1 - p if permute else p for p in range(pages)], np.uint32)
    i = np.arange(rows * qh * dim)
    q = (((i * 7) % 257).astype(np.int64) - 128).astype(np.float32) / 1024.0
    qpos = np.array([tokens - rows + r for r in range(rows)], np.int64)
    kpos = np.arange(tokens, dtype=np.int64)
    slots = pages * kvh * P
    k = np.zeros(slots * dim, np.int8)
    v = np.zeros(slots * dim, np.int8)
    ks = np.ones(slots, np.float32)
    vs = np.ones(slots, np.float32)
    d = np.arange(dim)
    for t in range(tokens):
        p, slot = int(table[t // P]), t % P
        for h in range(kvh):
            si = (p * kvh + h) * P + slot
            ks[si] = np.float32((t + h) % 7 + 1) / np.float32(512.0)
            vs[si] = np.float32((t * 3 + h) % 5 + 1) / np.float32(512.0)
            k[si * dim + d] = (((t * 17 + h * 11 + d * 3) % 256) - 128).astype(np.int8)
            vidx = ((p * kvh + h) * dim + d) * P + slot
            v[vidx] = (((t * 7 + h * 13 + d * 5) % 256) - 128).astype(np.int8)
    return dict(shape=shape, q=q, q_positions=qpos, k_positions=kpos, page_table=table,
                k=k, v=v, k_scales=ks, v_scales=vs)


class RefOracle:
    """The reference's own FP64 oracle and shape layer (oracle/_ref)."""

    def __init__(self):
        if not REF_ORACLE_LIB.exists():
            raise FileNotFoundError(f"{REF_ORACLE_LIB} not built (needs the reference sources)")
        lib = ctypes.CDLL(str(REF_ORACLE_LIB))
        dims = POINTER(c_uint32)
        lib.kvbref_shape_error.restype = c_char_p
        lib.kvbref_shape_error.argtypes = [dims, c_float, c_int]
        lib.kvbref_sizes.restype = c_int
        lib.kvbref_sizes.argtypes = [dims, c_float, c_int, POINTER(c_uint64)]
        lib.kvbref_mma_supported.restype = c_int
        lib.kvbref_mma_supported.argtypes = [dims, c_float, c_int]
        lib.kvbref_prepare.restype = c_void_p
        lib.kvbref_prepare.argtypes = [dims, c_float] + [c_void_p] * 8
        lib.kvbref_run.restype = c_int
        lib.kvbref_run.argtypes = [c_void_p, c_int, POINTER(c_double)]
        lib.kvbref_result.restype = c_int
        lib.kvbref_result.argtypes = [c_void_p, c_void_p, c_void_p]
        lib.kvbref_free.restype = None
        lib.kvbref_free.argtypes = [c_void_p]
        self.lib = lib

    @staticmethod
    def available() -> bool:
        return REF_ORACLE_LIB.exists()

    @staticmethod
    def _dims(f):
        return (c_uint32 * 9)(*(int(f[n]) for n in ("rows", "q_heads", "kv_heads", "dim", "page_tokens",
                                                       "pages", "tokens", "begin", "end")))

    def shape_error(self, shape) -> Optional[str]:
        f = shape_fields(shape)
        msg = self.lib.kvbref_shape_error(self._dims(f), float(f["scale"]), int(bool(f["int8"])))
        return msg.decode() if msg else None

    def sizes(self, shape):
        """(split_count, scratch, scalar, numerator) or None if the reference throws."""
        f = shape_fields(shape)
        out = (c_uint64 * 4)()
        rc = self.lib.kvbref_sizes(self._dims(f), float(f["scale"]), int(bool(f["int8"])), out)
        return None if rc else tuple(int(x) for x in out)

    def mma_supported(self, shape) -> bool:
        f = shape_fields(shape)
        return bool(self.lib.kvbref_mma_supported(self._dims(f), float(f["scale"]), int(bool(f["int8"]))))

    def prepare(self, shape, q, q_positions, k_positions, page_table, k, v, k_scales, v_scales):
        f = shape_fields(shape)
        arrs = [_np(q, np.float32), _np(q_positions, np.int64), _np(k_positions, np.int64),
                _np(page_table, np.int64).astype(np.uint32), _np(k, np.int8), _np(v, np.int8),
                _np(k_scales, np.float32), _np(v_scales, np.float32)]
        h = self.lib.kvbref_prepare(self._dims(f), float(f["scale"]), *(a.ctypes.data for a in arrs))
        if not h:
            raise ValueError("reference rejected the shape")
        return _RefRun(self, h, f)


class _RefRun:
    def __init__(self, owner: RefOracle, handle, f):
        self.owner, self.handle, self.f = owner, handle, f

    def run(self, threads: int) -> float:
        secs = c_double()
        rc = self.owner.lib.kvbref_run(self.handle, threads, ctypes.byref(secs))
        if rc:
            raise RuntimeError("reference run failed")
        return secs.value

    def result(self):
        f = self.f
        n = np.zeros((f["rows"], f["q_heads"], f["dim"]), np.float64)
        vis = np.zeros((f["rows"], f["q_heads"]), np.uint8)
        rc = self.owner.lib.kvbref_result(self.handle, n.ctypes.data, vis.ctypes.data)
        if rc:
            raise RuntimeError("reference result unavailable (run first)")
        return {"normalized": n, "visible": vis.astype(bool)}

    def close(self):
        if self.handle:
            self.owner.lib.kvbref_free(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


class RefCuda:
    """The reference's own CUDA launchers (oracle/_ref/libkvbref_cuda.so)."""

    def __init__(self):
        if not REF_CUDA_LIB.exists():
            raise FileNotFoundError(f"{REF_CUDA_LIB} not built (needs the reference sources)")
        lib = ctypes.CDLL(str(REF_CUDA_LIB))
        for name in ("kvbref_cuda_launch_attention", "kvbref_cuda_launch_attention_mma"):
            fn = getattr(lib, name)
            fn.restype = c_int
            fn.argtypes = [POINTER(c_uint32), c_float, c_int, POINTER(c_void_p)] + [c_void_p] * 5
        lib.kvbref_cuda_preload_reference.restype = c_int
        lib.kvbref_cuda_preload_reference.argtypes = []
        self.lib = lib

    @staticmethod
    def available() -> bool:
        return REF_CUDA_LIB.exists()

    def launch(self, shape, ptrs, scratch, m, l, n, stream=0, mma=False) -> int:
        f = shape_fields(shape)
        dims = RefOracle._dims(f)
        p = (c_void_p * 8)(*ptrs)
        fn = self.lib.kvbref_cuda_launch_attention_mma if mma else self.lib.kvbref_cuda_launch_attention
        return fn(dims, float(f["scale"]), int(bool(f["int8"])), p, scratch, m, l, n, stream)


def append_kv(k_new, v_new, slots, k, v, k_scales, v_scales, pages: int, page_tokens: int) -> int:
    """Quantise and write rows into numpy pools in place (oracle/kvb_oracle.c
    kvbo_append_kv). k_new/v_new float32 [tokens, kv_heads, dim]; slots int64
    [tokens]; k int8 [pages, kv, P, D]; v int8 [pages, kv, D, P]; scales float32
    [pages, kv, P]. Returns the number of out-of-range slots skipped."""
    kn = np.ascontiguousarray(_np(k_new, np.float32))
    vn = np.ascontiguousarray(_np(v_new, np.float32))
    sl = np.ascontiguousarray(_np(slots, np.int64))
    for a in (k, v, k_scales, v_scales):
        assert isinstance(a, np.ndarray) and a.flags["C_CONTIGUOUS"]
    assert k.dtype == np.int8 and v.dtype == np.int8
    assert k_scales.dtype == np.float32 and v_scales.dtype == np.float32
    tokens, kv_heads, dim = kn.shape
    assert vn.shape == kn.shape and sl.shape == (tokens,)
    assert k.shape == (pages, kv_heads, page_tokens, dim) and v.shape == (pages, kv_heads, dim, page_tokens)
    assert k_scales.shape == (pages, kv_heads, page_tokens) and v_scales.shape == k_scales.shape
    ptr = lambda a: a.ctypes.data_as(c_void_p)  # noqa: E731
    return _load_oracle().kvbo_append_kv(tokens, kv_heads, dim, page_tokens, pages, ptr(kn), ptr(vn),
                                         ptr(sl), ptr(k), ptr(v), ptr(k_scales), ptr(v_scales))
