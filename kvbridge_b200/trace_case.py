"""Per-tile event timeline of the tcgen05 partial kernel (the event-trace
build of the library, -DKVB_TC_TRACE): ``python -m kvbridge_b200.trace_case
--case native``. Runs warm-up calls of a profile_case workload, then one
traced call, and prints for each 128-token tile the median over the first 16
CTAs of each event's time (microseconds after the CTA passed its setup
barrier, from SM clock stamps converted at --mhz) and of the spans between
them:

  copy   producer armed the tile's first stage      (kTraceCopyIssued)
  qk     MMA thread issued QK (its stages had landed) (kTraceQkIssued)
  sm_in  softmax warp 0 saw S ready                 (kTraceSoftmaxIn)
  sm_out softmax warp 0 published P                 (kTraceSoftmaxOut)
  pv     MMA thread issued PV                       (kTracePvIssued)
  f_in   fold warp 0 saw O ready                    (kTraceFoldIn)
  f_out  fold warp 0 released O                     (kTraceFoldOut)
  sm_ld  softmax warp 0 had S in registers          (kTraceSmLoaded)
  sm_red softmax warp 0 passed the column-max barrier (kTraceSmReduced)
  sm_par softmax warp 0 passed the parameter barrier (kTraceSmParams)
  p_seen MMA thread saw P from every softmax warp   (kTracePReadySeen)
  o_seen MMA thread saw O^T released by the fold   (kTraceOFreeSeen)
  v_seen MMA thread saw the tile's V landed         (kTraceVSeen)
  sm_st  softmax warp 0 finished its P stores (before its proxy fence) (kTraceSmStored)
"""
from __future__ import annotations

import argparse
import ctypes
import os
import statistics
import sys

CTAS, TILES, EVENTS = 16, 16, 15
NAMES = ["start", "qk", "sm_in", "sm_out", "pv", "f_in", "f_out", "copy", "sm_ld", "sm_red", "sm_par", "p_seen", "o_seen", "v_seen", "sm_st"]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--case", default="native")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--mhz", type=float, default=1965.0, help="SM clock used to convert cycles to microseconds")
    args = ap.parse_args(argv)
    os.environ["KVB_TRACE_LIBRARY"] = "1"
    import torch

    from . import _lib, api, build, profile_case

    build.build(trace=True)
    lib = _lib.load()
    api.set_decode_kernel(api.KERNEL_TCGEN05)
    call = profile_case.make_call(args.case, torch.device("cuda", 0))
    n = CTAS * TILES * EVENTS
    buf = (ctypes.c_ulonglong * n)()
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    _lib.check(lib.kvb_debug_read_tc_trace(buf, n))  # clears
    call()
    torch.cuda.synchronize()
    _lib.check(lib.kvb_debug_read_tc_trace(buf, n))
    if api.read_device_status() != 0:
        print("device status nonzero:", api.read_wait_failure(), file=sys.stderr)
        return 1
    stamps = [[[buf[(c * TILES + t) * EVENTS + e] for e in range(EVENTS)] for t in range(TILES)]
              for c in range(CTAS)]
    rows = []
    for t in range(TILES):
        ev = {}
        for e, name in enumerate(NAMES):
            vals = [(stamps[c][t][e] - stamps[c][0][0]) / args.mhz for c in range(CTAS)
                    if stamps[c][0][0] and stamps[c][t][e]]
            ev[name] = statistics.median(vals) if vals else None
        if ev["qk"] is None:
            break
        rows.append(ev)
    print(f"tcgen05 partial kernel timeline, case {args.case}: median over {CTAS} CTAs, "
          f"microseconds (SM cycles / {args.mhz:.0f} MHz) after each CTA's setup barrier")
    print("tile " + " ".join(f"{k:>7}" for k in NAMES[1:]) + "   softmax    fold  sm_out->pv  copy->qk")
    for t, ev in enumerate(rows):
        def f(x):
            return f"{x:7.2f}" if x is not None else "      -"

        def span(a, b):
            return f"{ev[b] - ev[a]:9.2f}" if ev[a] is not None and ev[b] is not None else "        -"

        print(f"{t:4d} " + " ".join(f(ev[k]) for k in NAMES[1:]) + "  " + span("sm_in", "sm_out") + " "
              + span("f_in", "f_out") + "  " + span("sm_out", "pv") + "  " + span("copy", "qk"))
    return 0


if __name__ == "__main__":
    sys.exit(main())
