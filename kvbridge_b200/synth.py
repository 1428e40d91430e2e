"""Seeded synthetic decode-attention inputs in the kvbridge memory formats.

Stands in for real KV caches (no checkpoints or datasets are involved): the
value distributions follow the benchmark configurations of this path -
queries are fp16 N(0,1) values stored as fp32, K and V are fp32 N(0,1)
quantised per (token, kv head) by absmax to int8 (``scale = absmax / 127``,
``code = rint(x / scale)`` clamped to +-127), optionally with a fraction of
10x outlier tokens, and logical pages map to physical pages through a seeded
random permutation. Generation runs in torch on any device, seeded with a
``torch.Generator`` of that device.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from .api import BatchInput, BatchShape, DeviceInput, Shape

STAGE_TOKENS = 64


@dataclass
class SingleCase:
    """One decode call of the reference interface (rows of one sequence)."""

    shape: Shape
    q: torch.Tensor  # f32 [rows, q_heads, dim]
    q_positions: torch.Tensor  # i64 [rows]
    k_positions: torch.Tensor  # i64 [tokens]
    page_table: torch.Tensor  # i32 [pages] (uint32 values < 2^31)
    k: torch.Tensor  # i8 [pages, kv_heads, page_tokens, dim]
    v: torch.Tensor  # i8 [pages, kv_heads, dim, page_tokens]
    k_scales: torch.Tensor  # f32 [pages, kv_heads, page_tokens]
    v_scales: torch.Tensor

    def device_input(self) -> DeviceInput:
        return DeviceInput(
            self.q,
            self.q_positions,
            self.k_positions,
            self.page_table,
            self.k,
            self.v,
            self.k_scales,
            self.v_scales,
        )

    def kv_bytes(self) -> int:
        """Algorithmic KV bytes of one call: int8 K+V plus fp32 K/V scales per
        attended token and KV head."""
        s = self.shape
        per_token = s.kv_heads * (2 * s.dim + 8)
        return (s.end - s.begin) * per_token


@dataclass
class BatchCase:
    shape: BatchShape
    q: torch.Tensor  # f32 [batch, q_heads, dim]
    seq_lens: torch.Tensor  # i32 [batch]
    block_table: torch.Tensor  # i32 [batch, table_stride]
    k: torch.Tensor
    v: torch.Tensor
    k_scales: torch.Tensor
    v_scales: torch.Tensor
    lens: list

    def batch_input(self) -> BatchInput:
        return BatchInput(
            self.q, self.seq_lens, self.block_table, self.k, self.v, self.k_scales, self.v_scales
        )

    def kv_bytes(self) -> int:
        s = self.shape
        return sum(self.lens) * s.kv_heads * (2 * s.dim + 8)


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def quantize_kv(x: torch.Tensor):
    """Symmetric absmax int8 quantisation over the last dim: (codes, scales)."""
    absmax = x.abs().amax(dim=-1)
    scale = absmax / 127.0
    safe = torch.where(scale > 0, scale, torch.ones_like(scale))
    codes = torch.round(x / safe.unsqueeze(-1)).clamp_(-127, 127).to(torch.int8)
    return codes, scale.to(torch.float32)


def make_kv_pool(
    pages: int,
    kv_heads: int,
    page_tokens: int,
    dim: int,
    gen: torch.Generator,
    device,
    outlier_frac: float = 0.0,
    chunk_pages: int = 4096,
):
    """Quantised K [pages, kv, P, D], V [pages, kv, D, P] and their scales."""
    k = torch.empty((pages, kv_heads, page_tokens, dim), dtype=torch.int8, device=device)
    v = torch.empty((pages, kv_heads, dim, page_tokens), dtype=torch.int8, device=device)
    ks = torch.empty((pages, kv_heads, page_tokens), dtype=torch.float32, device=device)
    vs = torch.empty_like(ks)
    for p0 in range(0, pages, chunk_pages):
        p1 = min(pages, p0 + chunk_pages)
        for dst, sdst, transpose in ((k, ks, False), (v, vs, True)):
            x = torch.randn((p1 - p0, kv_heads, page_tokens, dim), generator=gen, device=device)
            if outlier_frac > 0:
                hit = torch.rand((p1 - p0, kv_heads, page_tokens), generator=gen, device=device)
                x = torch.where((hit < outlier_frac).unsqueeze(-1), x * 10.0, x)
            codes, scales = quantize_kv(x)
            dst[p0:p1] = codes.transpose(-1, -2) if transpose else codes
            sdst[p0:p1] = scales
    return k, v, ks, vs


def make_single(
    rows: int,
    q_heads: int,
    kv_heads: int,
    dim: int,
    page_tokens: int,
    tokens: int,
    seed: int,
    device="cpu",
    begin: int = 0,
    end: Optional[int] = None,
    outlier_frac: float = 0.0,
    spare_pages: int = 0,
    q_positions: Optional[Sequence[int]] = None,
    scale: Optional[float] = None,
) -> SingleCase:
    end = tokens if end is None else end
    gen = _gen(device, seed)
    needed = (tokens + page_tokens - 1) // page_tokens
    pages = needed + spare_pages
    table = torch.randperm(pages, generator=gen, device=device)[:needed].to(torch.int32)
    if needed < pages:  # the table covers the logical pages; the pool may be larger
        table = table.contiguous()
    k, v, ks, vs = make_kv_pool(pages, kv_heads, page_tokens, dim, gen, device, outlier_frac)
    q = torch.randn((rows, q_heads, dim), generator=gen, device=device).half().float()
    kpos = torch.arange(tokens, dtype=torch.int64, device=device)
    if q_positions is None:
        qpos = torch.full((rows,), tokens - 1, dtype=torch.int64, device=device)
    else:
        qpos = torch.tensor(list(q_positions), dtype=torch.int64, device=device)
    shape = Shape(
        rows,
        q_heads,
        kv_heads,
        dim,
        page_tokens,
        max(pages, needed),
        tokens,
        begin,
        end,
        1.0 / math.sqrt(dim) if scale is None else scale,
        True,
    )
    # A table shorter than `pages` is padded so page_table has `pages` entries.
    if table.numel() < shape.pages:
        pad = torch.zeros(shape.pages - table.numel(), dtype=torch.int32, device=device)
        table = torch.cat([table, pad])
    return SingleCase(shape, q, qpos, kpos, table, k, v, ks, vs)


def make_batched(
    q_heads: int,
    kv_heads: int,
    dim: int,
    page_tokens: int,
    seq_lens: Sequence[int],
    seed: int,
    device="cpu",
    outlier_frac: float = 0.0,
) -> BatchCase:
    gen = _gen(device, seed)
    lens = [int(x) for x in seq_lens]
    batch = len(lens)
    per_seq = [(n + page_tokens - 1) // page_tokens for n in lens]
    stride = max(1, max(per_seq))
    pages = max(1, sum(per_seq))
    perm = torch.randperm(pages, generator=gen, device=device).to(torch.int32)
    table = torch.zeros((batch, stride), dtype=torch.int32, device=device)
    off = 0
    for b, npg in enumerate(per_seq):
        table[b, :npg] = perm[off : off + npg]
        off += npg
    k, v, ks, vs = make_kv_pool(pages, kv_heads, page_tokens, dim, gen, device, outlier_frac)
    q = torch.randn((batch, q_heads, dim), generator=gen, device=device).half().float()
    shape = BatchShape(
        batch, q_heads, kv_heads, dim, page_tokens, pages, stride, max(lens), 1.0 / math.sqrt(dim)
    )
    sl = torch.tensor(lens, dtype=torch.int32, device=device)
    return BatchCase(shape, q, sl, table, k, v, ks, vs, lens)


def ragged_lengths(batch: int, lo: int, hi: int, seed: int) -> list:
    """Per-sequence context lengths drawn uniformly in [lo, hi] from `seed`."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return [int(x) for x in torch.randint(lo, hi + 1, (batch,), generator=g)]
