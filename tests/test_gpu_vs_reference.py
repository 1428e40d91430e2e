"""Speed against the reference's own CUDA kernels on the same B200, built from
its sources for sm_100a (oracle/_ref/libkvbref_cuda.so: the SIMT launcher,
reference src/attention_shared.cu:339, and the MMA launcher,
src/attention_mma.cu:33). Same device inputs, same stream, back-to-back calls
over four resident KV layers. Ours must match the FP64 oracle within the path
tolerance and the reference kernel must agree with ours within 1e-2 relative
L2 (its MMA kernel rounds Q and K to bf16, src/partial_attention_mma.cuh);
then ours must be the faster. Run with -s to see the timings."""
from __future__ import annotations

import pytest
import torch

import kvbridge_b200 as kvb
import oracle
from kvbridge_b200 import synth
from kvb_testutil import check_against_oracle, errors, normalized

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not oracle.RefCuda.available(), reason="reference CUDA build absent"),
]

CASES = [
    # BASELINE cfg2 through the reference's SIMT launcher (its MMA launcher
    # rejects this shape by contract).
    ("cfg2-64K", dict(rows=1, q_heads=32, kv_heads=8, dim=128, page_tokens=64, tokens=65536), False),
    # The reference MMA kernel's native shape: 8 query rows, 24/4 heads,
    # dim 256, 32-token pages, 32K tokens.
    ("native-8x6-d256", dict(rows=8, q_heads=24, kv_heads=4, dim=256, page_tokens=32, tokens=32768), True),
]


def _per_call_us(fn, iters):
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(iters):
        fn(i)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e3 / iters


@pytest.mark.parametrize("name,kw,mma", CASES, ids=[c[0] for c in CASES])
def test_faster_than_reference_kernels(cuda_device, name, kw, mma):
    rows, tokens = kw["rows"], kw["tokens"]
    qpos = [tokens - rows + r for r in range(rows)] if rows > 1 else None
    layers = [synth.make_single(seed=70 + i, device=cuda_device, q_positions=qpos, **kw) for i in range(4)]
    shape = layers[0].shape
    ref = oracle.RefCuda()
    rh = kvb.output_scalar_elements(shape)
    bufs = {k: torch.empty(rh if k in ("m", "l") else (kvb.scratch_elements(shape) if k == "scratch" else
                                                          kvb.output_numerator_elements(shape)), device=cuda_device)
            for k in ("scratch", "m", "l", "n")}
    inputs = [c.device_input() for c in layers]
    ptrs = [[t.data_ptr() for t in (c.q, c.q_positions, c.k_positions, c.page_table, c.k, c.v, c.k_scales,
                                   c.v_scales)] for c in layers]
    launch = kvb.launch_attention_mma if mma else kvb.launch_attention

    def ours(i):
        launch(shape, inputs[i % 4], bufs["scratch"], bufs["m"], bufs["l"], bufs["n"],
               stream=torch.cuda.current_stream())

    def theirs(i):
        rc = ref.launch(shape, ptrs[i % 4], bufs["scratch"].data_ptr(), bufs["m"].data_ptr(), bufs["l"].data_ptr(),
                        bufs["n"].data_ptr(), torch.cuda.current_stream().cuda_stream, mma=mma)
        assert rc == 0

    # Layer 0: ours against the FP64 oracle, theirs against ours.
    ours(0)
    torch.cuda.synchronize()
    mine = {k: bufs[k].cpu() for k in ("m", "l", "n")}
    check_against_oracle(mine, shape, oracle.reference_case(layers[0], threads=16), name)
    theirs(0)
    torch.cuda.synchronize()
    other = {k: bufs[k].cpu() for k in ("m", "l", "n")}
    _, rl = errors(normalized(other, shape), normalized(mine, shape).astype("float64"))
    assert rl <= 1e-2, rl

    t_ours = _per_call_us(ours, 40)
    t_ref = _per_call_us(theirs, 40)
    assert kvb.read_device_status() == 0
    gbs = layers[0].kv_bytes() / 1e3
    print(f"\n{name}: ours {t_ours:.1f} us ({gbs / t_ours:.0f} GB/s effective KV), reference "
          f"{'MMA' if mma else 'SIMT'} kernel {t_ref:.1f} us ({gbs / t_ref:.0f} GB/s): {t_ref / t_ours:.1f}x")
    assert t_ours < t_ref
