"""Helpers shared by the GPU tests: run the library on a synthetic case and
compare with the FP64 oracle."""
from __future__ import annotations

import numpy as np
import torch

import kvbridge_b200 as kvb
from kvbridge_b200 import synth
from kvbridge_b200.api import Shape

# Acceptance tolerances of this path against the FP64 oracle: max-abs 2e-3
# and rel-L2 1e-3. They apply as stated to the fp32 n/l the kernels compute.
# The fp16 output also carries its own rounding (half an fp16 ulp of the
# value, 2^-9 at |out| in [4, 8) and more above; the outlier configuration
# reaches |out| ~ 32), so its max-abs bound is 2e-3 plus that half ulp.
MAX_ABS = 2e-3
REL_L2 = 1e-3


def to_device(case: synth.SingleCase, device) -> synth.SingleCase:
    return synth.SingleCase(
        case.shape,
        *(getattr(case, f).to(device) for f in ("q", "q_positions", "k_positions", "page_table", "k", "v", "k_scales", "v_scales")),
    )


def outputs_for(shape: kvb.Shape, device):
    scratch = torch.full((kvb.scratch_elements(shape),), float("nan"), device=device)
    rh = kvb.output_scalar_elements(shape)
    m = torch.full((rh,), float("nan"), device=device)
    l = torch.full((rh,), float("nan"), device=device)
    n = torch.full((kvb.output_numerator_elements(shape),), float("nan"), device=device)
    return scratch, m, l, n


def run_single(case: synth.SingleCase, partitions: int = 0, fp16_out: bool = True, api: str = "ex"):
    """Runs one call; returns dict of host tensors (m, l, n, out, scratch)."""
    device = case.q.device
    scratch, m, l, n = outputs_for(case.shape, device)
    out = torch.full((kvb.output_numerator_elements(case.shape),), float("nan"), device=device,
                     dtype=torch.float16) if fp16_out else None
    inp = case.device_input()
    if api == "ex":
        kvb.launch_attention_ex(case.shape, inp, scratch, m, l, n, partitions=partitions, out_f16=out)
    elif api == "ref":
        kvb.launch_attention(case.shape, inp, scratch, m, l, n)
    elif api == "mma":
        kvb.launch_attention_mma(case.shape, inp, scratch, m, l, n)
    torch.cuda.synchronize()
    res = {"m": m.cpu(), "l": l.cpu(), "n": n.cpu(), "scratch": scratch}
    if out is not None:
        res["out"] = out.cpu()
    return res


def normalized(res, shape) -> np.ndarray:
    n = res["n"].double().numpy().reshape(shape.rows, shape.q_heads, shape.dim)
    l = res["l"].double().numpy().reshape(shape.rows, shape.q_heads, 1)
    return np.where(l > 0, n / np.where(l > 0, l, 1.0), 0.0)


def errors(actual: np.ndarray, expected: np.ndarray):
    diff = actual.astype(np.float64) - expected
    max_abs = float(np.max(np.abs(diff))) if diff.size else 0.0
    denom = float(np.linalg.norm(expected))
    rel_l2 = float(np.linalg.norm(diff) / denom) if denom > 0 else float(np.linalg.norm(diff))
    return max_abs, rel_l2


def check_against_oracle(res, shape, ref, label=""):
    """Asserts n/l (fp32) and the fp16 output against the oracle; checks the
    empty-row convention (m=-inf, l=0, n=0) row by row."""
    vis = ref["visible"]
    m = res["m"].numpy().reshape(shape.rows, shape.q_heads)
    l = res["l"].numpy().reshape(shape.rows, shape.q_heads)
    n = res["n"].numpy().reshape(shape.rows, shape.q_heads, shape.dim)
    assert np.array_equal(l > 0, vis), f"{label}: visibility differs"
    assert np.all(np.isneginf(m[~vis])), f"{label}: empty rows must have m=-inf"
    assert np.all(n[~vis] == 0), f"{label}: empty rows must have n=0"
    assert np.all(np.isfinite(m[vis])) and np.all(np.isfinite(n)), f"{label}: non-finite output"
    got = normalized(res, shape)
    ma, rl = errors(got, ref["normalized"])
    assert ma <= MAX_ABS and rl <= REL_L2, f"{label}: n/l max_abs={ma:.3e} rel_l2={rl:.3e}"
    if vis.any():
        # m is the max logit and l the softmax denominator of the same row.
        assert np.allclose(m[vis], ref["m"][vis], rtol=1e-5, atol=1e-5), f"{label}: m differs"
        assert np.allclose(l[vis], ref["l"][vis], rtol=2e-3, atol=0), f"{label}: l differs"
    if "out" in res:
        out = res["out"].double().numpy().reshape(shape.rows, shape.q_heads, shape.dim)
        expect = ref["normalized"]
        half_ulp = np.spacing(np.abs(expect).astype(np.float16)).astype(np.float64) / 2
        excess = np.abs(out - expect) - half_ulp
        ma16 = float(excess.max()) if excess.size else 0.0
        _, rl16 = errors(out, expect)
        assert ma16 <= MAX_ABS and rl16 <= REL_L2, f"{label}: fp16 out max_abs-halfulp={ma16:.3e} rel_l2={rl16:.3e}"
    return ma, rl


def report(label: str, **values) -> None:
    """Records an achieved-error line: printed, and appended as JSON to the
    file named by $KVB_PARITY_REPORT when that is set."""
    import json
    import os

    line = {"case": label, **{k: (float(v) if isinstance(v, (int, float, np.floating)) else v)
                              for k, v in values.items()}}
    print(f"[parity] {json.dumps(line)}")
    path = os.environ.get("KVB_PARITY_REPORT")
    if path:
        with open(path, "a") as fh:
            fh.write(json.dumps(line) + "\n")


def host_pool(bc):
    """The batched case's K/V pool and scales as numpy arrays (copied once)."""
    return tuple(getattr(bc, f).cpu().numpy() for f in ("k", "v", "k_scales", "v_scales"))


def check_batched(bc, m, l, n, out=None, label="batched", threads=None, out_bf16=None, pool=None):
    """Every sequence of a batched call against the FP64 oracle (n/l, m, l,
    the fp16 output and optionally the bf16 output). Returns the worst
    (max_abs, rel_l2) of n/l over the batch."""
    import os

    import oracle

    threads = threads or os.cpu_count() or 8
    k, v, ks, vs = pool if pool is not None else host_pool(bc)
    s = bc.shape
    H, D, P = s.q_heads, s.dim, s.page_tokens
    m, l, n = m.cpu(), l.cpu(), n.cpu()
    out = out.cpu() if out is not None else None
    out_bf16 = out_bf16.cpu() if out_bf16 is not None else None
    table_all = bc.block_table.cpu()
    q_all = bc.q.cpu()
    worst = (0.0, 0.0)
    for b, length in enumerate(bc.lens):
        sl = slice(b * H, (b + 1) * H)
        if length == 0:
            assert torch.all(l[sl] == 0) and torch.all(torch.isneginf(m[sl])), f"{label}: seq {b} not empty"
            continue
        npg = (length + P - 1) // P
        table = torch.zeros(s.pages, dtype=torch.int64)
        table[:npg] = table_all[b, :npg].to(torch.int64)
        shape = Shape(1, H, s.kv_heads, D, P, s.pages, length, 0, length, s.scale, True)
        ref = oracle.reference(shape, q_all[b], torch.tensor([length - 1]), torch.arange(length), table,
                               k, v, ks, vs, threads=threads)
        res = {"m": m[sl], "l": l[sl], "n": n[b * H * D:(b + 1) * H * D]}
        if out is not None:
            res["out"] = out[b * H * D:(b + 1) * H * D]
        ma, rl = check_against_oracle(res, shape, ref, f"{label} seq {b}")
        if out_bf16 is not None:
            check_bf16(out_bf16[b * H * D:(b + 1) * H * D], shape, ref, f"{label} seq {b} bf16")
        worst = (max(worst[0], ma), max(worst[1], rl))
    return worst


def check_bf16(out_bf16, shape, ref, label=""):
    """bf16 output n/l against the oracle: max-abs 2e-3 beyond half a bf16
    ulp of the value (bf16 keeps 8 significant bits), rel-L2 within 1e-3 plus
    the bf16 rounding (2^-9 relative)."""
    got = out_bf16.float().double().numpy().reshape(shape.rows, shape.q_heads, shape.dim)
    expect = ref["normalized"]
    mag = np.abs(expect)
    # half an ulp of bf16 at |x|: 2^(floor(log2|x|) - 8)
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(mag > 0, mag, 1.0)))
    half_ulp = np.where(mag > 0, np.exp2(e - 8), 0.0)
    excess = np.abs(got - expect) - half_ulp
    ma = float(excess.max()) if excess.size else 0.0
    _, rl = errors(got, expect)
    assert ma <= MAX_ABS and rl <= REL_L2 + 2.0 ** -9, f"{label}: bf16 max_abs-halfulp={ma:.3e} rel_l2={rl:.3e}"
    return ma, rl
