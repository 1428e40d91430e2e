"""Build recipe of the in-tree shared library ``kvbridge_b200/libkvbridge_b200.so``.

nvcc cross-compiles the sm_100a kernels without a GPU, so this runs both in
the CPU container and on a GPU box. The library links the CUDA runtime
statically and is linked with -Bsymbolic so its C++ entry points bind to
their own definitions even when another library exporting the same
``kvbridge::`` names is loaded in the process.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libkvbridge_b200.so"
BUILD_DIR = PKG / "_build"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["attention_shape.cpp", "attention.cu", "c_api.cpp"]
HEADERS = [
    "kvb_device.cuh",
    "kvb_schedule.h",
    "decode_tma.cuh",
    "decode_tc.cuh",
    "decode_f32.cuh",
    "decode_simt.cuh",
    "merge.cuh",
    "peer_merge.cuh",
    "append_kv.cuh",
    "launch_checks.h",
]


def _inputs() -> list[Path]:
    files = [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS]
    files += sorted(INCLUDE.rglob("*.h"))
    files.append(Path(__file__))
    return files


def needs_build() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    return any(f.stat().st_mtime > built for f in _inputs() if f.exists())


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}")


TRACE_LIB = PKG / "libkvbridge_b200_trace.so"
TRACE_BUILD_DIR = PKG / "_build_trace"


def build(force: bool = False, verbose_ptxas: bool = False, trace: bool = False) -> Path:
    """Compile the library if any input changed (or ``force``); return its path.
    ``trace`` builds the event-trace variant (-DKVB_TC_TRACE) beside it."""
    lib, build_dir = (TRACE_LIB, TRACE_BUILD_DIR) if trace else (LIB, BUILD_DIR)
    if not force and lib.exists() and not any(
            f.stat().st_mtime > lib.stat().st_mtime for f in _inputs() if f.exists()):
        return lib
    build_dir.mkdir(exist_ok=True)
    common = ["-std=c++17", "-O3", f"-I{INCLUDE}", f"-I{CSRC}", "-Xcompiler", "-fPIC"]
    if trace:
        common.append("-DKVB_TC_TRACE")
    objects = []
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmd = [NVCC, *common, "-c", str(CSRC / src), "-o", str(obj)]
        if src.endswith(".cu"):
            cmd[1:1] = [*ARCH, "-lineinfo", "--expt-relaxed-constexpr"]
            if verbose_ptxas:
                cmd.insert(1, "-Xptxas=-v")
        _run(cmd)
        objects.append(str(obj))
    tmp = lib.with_suffix(".so.tmp")
    _run([NVCC, *ARCH, "-shared", "-o", str(tmp), *objects, "-Xlinker", "-Bsymbolic"])
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    force = "--force" in sys.argv
    print(build(force=force, verbose_ptxas="--ptxas-v" in sys.argv, trace="--trace" in sys.argv))
