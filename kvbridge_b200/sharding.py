"""Multi-GPU partitioning of decode attention (host orchestration).

Two modes, one process per GPU over ``torch.distributed``:

* KV-head sharding: rank g owns KV heads [g*H/G, (g+1)*H/G) with their query
  heads, in its own reference-format pool. The heads are independent, so the
  attention itself needs no communication; outputs stay head-sharded (an
  optional all-gather assembles them).
* Sequence sharding: rank g owns a contiguous, page-aligned token range of
  every sequence. Each rank computes the (m, l, n) partial of its range
  (launch_attention_ex / launch_attention_batched over local pages); the
  partials are all-gathered and merged with merge_attention_shards, the same
  log-sum-exp algebra as the split-K merge (reference src/attention_shared.cu:
  295-335) with one "split" per rank.

The exchange and merge functions are parameters so the orchestration runs
unchanged on CPU ``gloo`` ranks in the tests. On GPUs that reach each other
over NVLink, ``PeerExchange`` replaces the all-gather and the merge with one
kernel that reads the other ranks' partials from their memory
(merge_attention_peers).
"""
from __future__ import annotations

from typing import Callable, List, Sequence, Tuple


def kv_head_range(kv_heads: int, world: int, rank: int) -> Tuple[int, int]:
    """KV heads [h0, h1) owned by `rank`; kv_heads must divide evenly."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if kv_heads % world:
        raise ValueError(f"{kv_heads} KV heads do not shard evenly over {world} ranks")
    per = kv_heads // world
    return rank * per, (rank + 1) * per


def sequence_ranges(tokens: int, page_tokens: int, world: int) -> List[Tuple[int, int]]:
    """Contiguous page-aligned token ranges covering [0, tokens), balanced to
    one page; ranks beyond the page count get empty ranges."""
    if world <= 0 or page_tokens <= 0 or tokens < 0:
        raise ValueError("world and page_tokens must be positive")
    pages = -(-tokens // page_tokens)
    out = []
    for r in range(world):
        p0 = pages * r // world
        p1 = pages * (r + 1) // world
        out.append((min(tokens, p0 * page_tokens), min(tokens, p1 * page_tokens)))
    return out


def local_pages(ranges: Sequence[Tuple[int, int]], rank: int, page_tokens: int) -> Tuple[int, int]:
    """Logical pages [p0, p1) stored by `rank` for its token range."""
    b, e = ranges[rank]
    if e <= b:
        return b // page_tokens, b // page_tokens
    return b // page_tokens, -(-e // page_tokens)


def all_gather_partials(m, l, n, group=None):
    """Stacks every rank's (m, l, n) partial: [G, ...] tensors, rank-major."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    out = []
    for t in (m, l, n):
        t = t.contiguous()
        buf = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        if t.device.type == "cuda":
            dist.all_gather_into_tensor(buf, t, group=group)
        else:
            dist.all_gather(list(buf.unbind(0)), t, group=group)
        out.append(buf)
    return tuple(out)


def all_gather_packed(buf, group=None):
    """One all-gather of every rank's packed partial buffer [m | l | n]:
    returns [G, buf.numel()], rank-major. On GPU this is a single NCCL
    collective; merge_attention_shards_ex reads the result in place with
    shard_stride = buf.numel()."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    flat = buf.contiguous().view(-1)
    out = torch.empty((world, flat.numel()), dtype=flat.dtype, device=flat.device)
    if flat.device.type == "cuda":
        dist.all_gather_into_tensor(out, flat, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), flat, group=group)
    return out


def packed_views(buf, row_heads: int, dim: int):
    """(m, l, n) views of a packed partial buffer [m (rh) | l (rh) | n (rh*dim)]."""
    return buf[:row_heads], buf[row_heads:2 * row_heads], buf[2 * row_heads:2 * row_heads + row_heads * dim]


def sequence_sharded_decode(
    local_partial: Callable[[], Tuple["object", "object", "object"]],
    merge: Callable[["object", "object", "object"], "object"],
    group=None,
    exchange: Callable = all_gather_partials,
):
    """Computes this rank's partial, exchanges partials, merges them.

    local_partial() -> (m, l, n) of the rank's range; merge(m_parts, l_parts,
    n_parts) -> merged result. Every rank takes the same collective steps."""
    m, l, n = local_partial()
    mp, lp, np_ = exchange(m, l, n, group)
    return merge(mp, lp, np_)


def gpu_packed_shard_merge(rh: int, dim: int, device, out_f16: bool = True):
    """merge() of the packed exchange: gathered [G, rh * (dim + 2)] from
    all_gather_packed is merged in place (merge_attention_shards_ex with
    shard_stride = rh * (dim + 2)) into preallocated outputs."""
    import torch

    from . import api

    m = torch.empty(rh, device=device)
    l = torch.empty(rh, device=device)
    n = torch.empty(rh * dim, device=device)
    out = torch.empty(rh * dim, dtype=torch.float16, device=device) if out_f16 else None

    def merge(gathered):
        shards = gathered.shape[0]
        api.merge_attention_shards_ex(shards, rh, dim, gathered, gathered[:, rh:], gathered[:, 2 * rh:],
                                      rh * (dim + 2), m, l, n, out_f16=out)
        return m, l, n, out

    return merge


def gpu_shard_merge(rh: int, dim: int, out_f16: bool = True):
    """merge() for sequence_sharded_decode on GPU tensors: the library's
    merge_attention_shards kernel (log-sum-exp over the ranks' partials)."""
    import torch

    from . import api

    def merge(mp, lp, np_):
        shards = mp.shape[0]
        dev = mp.device
        m = torch.empty(rh, device=dev)
        l = torch.empty(rh, device=dev)
        n = torch.empty(rh * dim, device=dev)
        out = torch.empty(rh * dim, dtype=torch.float16, device=dev) if out_f16 else None
        api.merge_attention_shards(shards, rh, dim, mp, lp, np_, m, l, n, out)
        return m, l, n, out

    return merge


class PeerExchange:
    """Sequence-shard exchange over NVLink peer memory for one process group:
    every rank allocates a peer buffer (``api.peer_buffer_alloc``), the CUDA IPC
    handles are all-gathered once, and each rank maps the others' buffers.
    Per call: ``slot()`` gives the address of this call's slot (packed
    [m | l | n] floats) for the local decode to write its partials into, and
    ``merge(...)`` launches the kernel that publishes the slot, waits for the
    other ranks' and merges them all into m, l, n (and an fp16 / bf16 output).
    Every rank must make the same sequence of calls; the epoch (call number)
    advances in ``slot()``. ``close()`` unmaps and frees the buffers."""

    def __init__(self, row_heads: int, dim: int, group=None):
        import torch.distributed as dist

        from . import api

        self._api = api
        self.row_heads, self.dim = row_heads, dim
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.own, handle = api.peer_buffer_alloc(api.peer_buffer_bytes(row_heads, dim))
        handles: list = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.buffers = [self.own if r == self.rank else api.peer_buffer_open(h) for r, h in enumerate(handles)]
        # Every rank has mapped every buffer (and the zeroed flags are in
        # place) before any rank publishes into another's.
        dist.barrier(group=group)
        self.epoch = 0

    def slot(self):
        """Starts the next call; returns (m, l, n) addresses of its slot."""
        if not self.buffers:
            raise RuntimeError("the exchange is closed")
        self.epoch += 1
        base = self._api.peer_slot(self.own, self.epoch, self.row_heads, self.dim)
        return base, base + 4 * self.row_heads, base + 8 * self.row_heads

    def merge(self, m, l, n, out_f16=None, out_bf16=None, stream=None) -> None:
        self._api.merge_attention_peers(self.buffers, self.rank, self.epoch, self.row_heads, self.dim, m, l, n,
                                        out_f16, out_bf16, stream)

    def close(self) -> None:
        """Releases the mappings and the buffer (once; later calls do
        nothing); every rank's kernels that read them must have finished
        (synchronize, then a barrier)."""
        if not self.buffers:
            return
        for r, b in enumerate(self.buffers):
            if r != self.rank:
                self._api.peer_buffer_close(b)
        self._api.peer_buffer_free(self.own)
        self.buffers = []
        self.own = 0
