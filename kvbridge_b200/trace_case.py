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
  p_g0..p_g2  softmax warp 0 finished the P digits of its column group 0, 1, 2
         (4 columns each; group 3 ends at sm_st) (kTracePGroup)

``--kernel warp`` prints instead the per-CTA timeline of the warp-level
partial kernel (decode_tma.cuh, CtaTraceEvent) for the last of
``--back-to-back`` calls (default 2) replayed from one CUDA graph, as in
bench.py, and the chain from the first call's partial
kernel through its merge to the second call's dependency wait: every traced CTA's events on one time axis (the global timer
at entry and exit aligns CTAs of different SMs; SM clock stamps place the
events in between, converted at the clock rate each CTA's own entry/exit
pair implies), the distribution over CTAs of each event and of the spans
start (entry to first stage landed), streaming (first stage landed to last
stage armed), drain (last stage armed to the last warp done; split at the
moment the last stage landed) and combine
(last warp done to partials written), and a histogram of CTA exit times.
"""
from __future__ import annotations

import argparse
import ctypes
import os
import statistics
import sys

CTAS, TILES, EVENTS = 16, 16, 18
NAMES = ["start", "qk", "sm_in", "sm_out", "pv", "f_in", "f_out", "copy", "sm_ld", "sm_red", "sm_par", "p_seen", "o_seen",
         "v_seen", "sm_st", "p_g0", "p_g1", "p_g2"]


# CtaTraceEvent of decode_tma.cuh.
CTA_MAX, CTA_EVENTS, MERGE_MAX, MERGE_EVENTS = 1024, 20, 1024, 5
(E_ENTRY_NS, E_ENTRY_CLK, E_SM, E_DEP, E_FIRST_COPY, E_LAST_COPY, E_FIRST_STAGE, E_WARP0,
 E_PARTIAL, E_EXIT_NS, E_STAGES, E_LAST_STAGE, E_FIRST_ENTRY_NS, E_FIRST_EXIT_NS, E_PROD_WAIT,
 E_CONS_WAIT) = (0, 1, 2, 3, 4, 5, 6, 7, 11, 12, 13, 14, 16, 17, 18, 19)


def _pct(vals, q):
    v = sorted(vals)
    return v[min(len(v) - 1, int(round(q * (len(v) - 1))))]


def cta_timeline(args, torch, _lib, api, profile_case) -> int:
    lib = _lib.load()
    api.set_decode_kernel(api.KERNEL_WARP_MMA)
    call = profile_case.make_call(args.case, torch.device("cuda", 0))
    n = CTA_MAX * CTA_EVENTS
    buf = (ctypes.c_ulonglong * n)()
    mbuf = (ctypes.c_ulonglong * (MERGE_MAX * MERGE_EVENTS))()
    # The traced calls replay from a CUDA graph, as in bench.py, so that the
    # host's launch rate does not set the gaps between them.
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            call()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(args.back_to_back):
            call()
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    _lib.check(lib.kvb_debug_read_cta_trace(buf, n))  # clears
    _lib.check(lib.kvb_debug_read_merge_trace(mbuf, MERGE_MAX * MERGE_EVENTS))
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    _lib.check(lib.kvb_debug_read_cta_trace(buf, n))
    _lib.check(lib.kvb_debug_read_merge_trace(mbuf, MERGE_MAX * MERGE_EVENTS))
    if api.read_device_status() != 0:
        print("device status nonzero:", api.read_wait_failure(), file=sys.stderr)
        return 1
    rows = [[buf[c * CTA_EVENTS + e] for e in range(CTA_EVENTS)] for c in range(CTA_MAX)]
    rows = [r for r in rows if r[E_ENTRY_NS] and r[E_EXIT_NS] and r[E_PARTIAL]]
    if not rows:
        print("no CTA was traced", file=sys.stderr)
        return 1
    # Clock rate per CTA from its entry/exit pair (cycles per ns = GHz).
    ghz = statistics.median((r[E_PARTIAL] - r[E_ENTRY_CLK]) / max(1, r[E_EXIT_NS] - r[E_ENTRY_NS]) for r in rows)
    entries = sorted({r[E_ENTRY_NS] for r in rows})
    steps = [b - a for a, b in zip(entries, entries[1:]) if b > a]
    t0 = min(r[E_ENTRY_NS] for r in rows)

    def at(r, e):  # microseconds after the launch's first CTA entry
        if e == E_ENTRY_NS:
            return (r[E_ENTRY_NS] - t0) / 1e3
        if not r[e]:
            return None
        return (r[E_ENTRY_NS] - t0) / 1e3 + (r[e] - r[E_ENTRY_CLK]) / ghz / 1e3

    events = [("entry", E_ENTRY_NS), ("dependency wait passed", E_DEP), ("first stage armed", E_FIRST_COPY),
              ("first stage landed", E_FIRST_STAGE), ("last stage armed", E_LAST_COPY),
              ("last stage landed", E_LAST_STAGE)]
    table = []
    for name, e in events:
        table.append((name, [at(r, e) for r in rows if at(r, e) is not None]))
    first_done = [min(at(r, E_WARP0 + w) for w in range(4) if r[E_WARP0 + w]) for r in rows]
    last_done = [max(at(r, E_WARP0 + w) for w in range(4) if r[E_WARP0 + w]) for r in rows]
    table.append(("first warp done", first_done))
    table.append(("last warp done", last_done))
    table.append(("partials written (exit)", [at(r, E_PARTIAL) for r in rows]))
    stages = [r[E_STAGES] for r in rows]
    print(f"warp-level partial kernel, case {args.case}: last of {args.back_to_back} back-to-back calls, "
          f"{len(rows)} CTAs on {len({r[E_SM] for r in rows})} SMs, {statistics.median(stages):.0f} stages "
          f"a CTA (min {min(stages)}, max {max(stages)}); SM clock {ghz * 1e3:.0f} MHz from the CTAs' "
          f"own entry/exit pairs; global timer step {min(steps) if steps else 0} ns")
    print("microseconds after the first CTA's entry, over CTAs:")
    print(f"{'event':28s} {'min':>7s} {'p10':>7s} {'median':>7s} {'p90':>7s} {'max':>7s}")
    for name, vals in table:
        print(f"{name:28s} " + " ".join(f"{_pct(vals, q):7.2f}" for q in (0, 0.1, 0.5, 0.9, 1.0)))
    spans = [
        ("start: entry -> first landed", [at(r, E_FIRST_STAGE) - at(r, E_ENTRY_NS) for r in rows if r[E_FIRST_STAGE]]),
        ("streaming: landed -> last armed", [at(r, E_LAST_COPY) - at(r, E_FIRST_STAGE) for r in rows
                                             if r[E_FIRST_STAGE] and r[E_LAST_COPY]]),
        ("drain: last armed -> last warp", [d - at(r, E_LAST_COPY) for r, d in zip(rows, last_done) if r[E_LAST_COPY]]),
        ("  last stage's copy", [at(r, E_LAST_STAGE) - at(r, E_LAST_COPY) for r in rows
                                 if r[E_LAST_STAGE] and r[E_LAST_COPY]]),
        ("  last landed -> last warp", [d - at(r, E_LAST_STAGE) for r, d in zip(rows, last_done) if r[E_LAST_STAGE]]),
        ("warp spread: first -> last warp", [b - a for a, b in zip(first_done, last_done)]),
        ("combine: last warp -> written", [at(r, E_PARTIAL) - d for r, d in zip(rows, last_done)]),
    ]
    print(f"{'span (per CTA)':32s} {'min':>7s} {'median':>7s} {'p90':>7s} {'max':>7s}")
    for name, vals in spans:
        print(f"{name:32s} " + " ".join(f"{_pct(vals, q):7.2f}" for q in (0, 0.5, 0.9, 1.0)))
    life = [(r[E_PARTIAL] - r[E_ENTRY_CLK]) for r in rows]
    pw = [r[E_PROD_WAIT] / max(1, x) for r, x in zip(rows, life)]
    cw = [r[E_CONS_WAIT] / max(1, x) for r, x in zip(rows, life)]
    print(f"producer waiting for free slots: median {100 * statistics.median(pw):.0f} % of the CTA's "
          f"lifetime (p10 {100 * _pct(pw, 0.1):.0f}, p90 {100 * _pct(pw, 0.9):.0f}); consumer warp 0 "
          f"waiting for data: median {100 * statistics.median(cw):.0f} % (p10 {100 * _pct(cw, 0.1):.0f}, "
          f"p90 {100 * _pct(cw, 0.9):.0f})")
    exits = [at(r, E_PARTIAL) for r in rows]
    lo = int(min(exits))
    hist = [0] * (int(max(exits)) - lo + 1)
    for x in exits:
        hist[int(x) - lo] += 1
    print("CTA exits per microsecond: " + ", ".join(f"{lo + i}: {c}" for i, c in enumerate(hist) if c))

    # The chain between calls: the first call's partial kernel, its merge, and
    # the next call's partial kernel, on the global timer.
    merges = [[mbuf[c * MERGE_EVENTS + e] for e in range(MERGE_EVENTS)] for c in range(MERGE_MAX)]
    merges = [m for m in merges if all(m)]
    first_exits = [r[E_FIRST_EXIT_NS] for r in rows if r[E_FIRST_EXIT_NS]]
    if args.back_to_back >= 2 and merges and first_exits:
        z = max(first_exits)

        def span_us(vals):
            return f"{(min(vals) - z) / 1e3:7.2f} .. {(max(vals) - z) / 1e3:7.2f}"

        deps = [t0 + at(r, E_DEP) * 1e3 for r in rows if r[E_DEP]]
        print("call 1 -> its merge -> call 2 (global timer, microseconds after call 1's last partial CTA exit):")
        print(f"  call 1 partial CTAs exited       {span_us(first_exits)}")
        print(f"  call 1 merge CTAs entered        {span_us([m[0] for m in merges])}")
        print(f"  call 1 merge dependency passed   {span_us([m[1] for m in merges])}")
        print(f"  call 1 merge first loads used    {span_us([m[3] for m in merges])}")
        print(f"  call 1 merge warps folded        {span_us([m[4] for m in merges])}")
        print(f"  call 1 merge CTAs exited         {span_us([m[2] for m in merges])}")
        if args.back_to_back == 2:
            print(f"  call 2 partial CTAs entered      {span_us([r[E_ENTRY_NS] for r in rows])}")
            print(f"  call 2 dependency wait passed    {span_us(deps)}")
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--case", default="native")
    ap.add_argument("--kernel", choices=["tcgen05", "warp"], default="tcgen05")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--back-to-back", type=int, default=2, help="warp: calls issued before the read")
    ap.add_argument("--mhz", type=float, default=1965.0, help="tcgen05: SM clock used to convert cycles to microseconds")
    args = ap.parse_args(argv)
    os.environ["KVB_TRACE_LIBRARY"] = "1"
    import torch

    from . import _lib, api, build, profile_case

    build.build(trace=True)
    if args.kernel == "warp":
        return cta_timeline(args, torch, _lib, api, profile_case)
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
