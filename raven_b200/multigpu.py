"""Multi-GPU plumbing for batched search: one process per GPU.

The reference runs `GraphSearcher::batch_search` (src/graph/vamana.rs:1983-2095)
as a rayon map over the queries of one in-memory graph; it has no multi-node
or multi-GPU layer. Two layouts map that onto several B200s:

* Replicated index, query partition (collections that fit one GPU). Every rank
  holds the whole index and searches its own contiguous slice of the queries.
  No collective on the data path; the only collectives are the timing barrier
  and the max-over-ranks reduction (`max_over_ranks`).
* Sharded collection (collections too large for one GPU). The base vectors
  are split into `n_shards` contiguous shards, shard s holding global ids
  [s * shard_size, (s + 1) * shard_size), each with its own graph and codes.
  Shard s lives on rank s % world. Every rank searches every query on each of
  its shards; the per-shard top-k lists (f32 distance, shard-local id, count)
  are exchanged by one all-gather and merged per query on the GPU by
  `raven_merge_topk_gathered_device`, ties ordered by (distance, shard, rank in the
  shard's list). Searching each shard exactly as the reference searches one
  graph and merging by that rule gives the same ids as running the reference
  on every shard and merging its outputs on the host.

The search kernel writes each shard's lists (ids, distances, counts) into one
block of the rank's send buffer, one all-gather moves every rank's blocks, and
the merge kernel reads the gathered buffer where it lies (shard s is block
(s % world) * per_rank + s // world). The exchange works on NCCL (CUDA
tensors) and gloo (CPU tensors, used by the CPU tests of this module).
"""
from __future__ import annotations

import ctypes as C
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib as L


def query_slice(nq: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous rows [lo, hi) of an nq-query batch searched by `rank`; the
    first nq % world ranks take one row more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    base, extra = divmod(nq, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shards_of_rank(n_shards: int, world: int, rank: int) -> List[int]:
    """Shards held by `rank`: s with s % world == rank, ascending."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    return list(range(rank, n_shards, world))


def max_over_ranks(x: float, device: Optional[torch.device] = None, group=None) -> float:
    """Max of a per-rank scalar (device time of the timed region) over all
    ranks; the identity without an initialised process group."""
    if not (dist.is_available() and dist.is_initialized()):
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def block_words(nq: int, k: int) -> int:
    """32-bit words of one shard's lists in the exchange layout: ids u32
    [nq][k], distances f32 [nq][k], counts u32 [nq], end to end."""
    return nq * (2 * k + 1)


def per_rank(n_shards: int, world: int) -> int:
    """Shard blocks every rank sends (ranks holding fewer pad with unused blocks)."""
    return -(-n_shards // world)


def gathered_block(shard: int, world: int, per: int) -> int:
    """Block index of `shard` in the all-gathered buffer: rank shard % world,
    slot shard // world there."""
    return (shard % world) * per + shard // world


def block_views(buf: torch.Tensor, j: int, nq: int, k: int):
    """(ids, dists, counts) views of block j of a flat int32 buffer: ids
    [nq, k] int32 (u32 bit patterns), dists [nq, k] f32, counts [nq] int32."""
    w = block_words(nq, k)
    b = buf[j * w:(j + 1) * w]
    return (b[:nq * k].view(nq, k), b[nq * k:2 * nq * k].view(torch.float32).view(nq, k), b[2 * nq * k:])


def exchange_blocks(send: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather every rank's send buffer (its shard blocks) into one flat
    buffer, rank-major. NCCL on CUDA tensors; gloo (CPU tests) gathers a list."""
    world = dist.get_world_size(group)
    recv = send.new_empty(world * send.numel())
    if send.is_cuda:
        dist.all_gather_into_tensor(recv, send, group=group)
    else:
        parts = list(recv.chunk(world))
        dist.all_gather(parts, send, group=group)
    return recv


def read_gathered(recv: torch.Tensor, n_shards: int, world: int, nq: int, k: int):
    """Host-side view of a gathered buffer in shard order: ids [S, nq, k]
    (uint32), dists [S, nq, k], counts [S, nq] as numpy arrays."""
    import numpy as np

    per = per_rank(n_shards, world)
    a = recv.cpu().numpy()
    w = block_words(nq, k)
    ids = np.zeros((n_shards, nq, k), np.uint32)
    ds = np.zeros((n_shards, nq, k), np.float32)
    cs = np.zeros((n_shards, nq), np.uint32)
    for s in range(n_shards):
        b = a[gathered_block(s, world, per) * w:][:w]
        ids[s] = b[:nq * k].view(np.uint32).reshape(nq, k)
        ds[s] = b[nq * k:2 * nq * k].view(np.float32).reshape(nq, k)
        cs[s] = b[2 * nq * k:].view(np.uint32)
    return ids, ds, cs


class ShardedCollection:
    """Per-shard device indexes of this rank and the search-exchange-merge step.

    `shards` maps shard number -> DeviceIndex for the shards this rank holds
    (exactly `shards_of_rank(n_shards, world, rank)`); every shard but the last
    covers `shard_size` global ids.

    A step writes each local shard's top-k lists straight into this rank's
    send buffer (one block per shard, the layout of `block_views`), gathers
    every rank's buffer with one all-gather, and merges the gathered blocks
    in place with raven_merge_topk_gathered_device: no packing or reordering
    copies. The buffers are kept per (nq, k) and reused, so the tensors a step
    returns are valid until the next step with the same shape.
    """

    def __init__(self, shards: Dict[int, "object"], n_shards: int, shard_size: int, group=None):
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        want = shards_of_rank(n_shards, world, rank)
        if sorted(shards) != want:
            raise ValueError(f"rank {rank} must hold shards {want}, got {sorted(shards)}")
        self.shards = shards
        self.order = want
        self.n_shards = n_shards
        self.shard_size = shard_size
        self.group = group
        self.world = world
        self.per = per_rank(n_shards, world)
        self._bufs = {}

    def _buffers(self, nq: int, k: int, dev, stream):
        key = (nq, k, str(dev))
        if key not in self._bufs:
            with torch.cuda.stream(stream):
                send = torch.zeros(self.per * block_words(nq, k), dtype=torch.int32, device=dev)
                recv = torch.zeros(self.world * send.numel(), dtype=torch.int32, device=dev) if self.world > 1 else send
                out = (torch.zeros((nq, k), dtype=torch.int32, device=dev),
                       torch.zeros((nq, k), dtype=torch.float32, device=dev),
                       torch.zeros(nq, dtype=torch.int32, device=dev))
            self._bufs[key] = (send, recv, out)
        return self._bufs[key]

    def _exchange_merge(self, send, recv, out, nq: int, k: int, stream, marks=None):
        lib = L.load()
        if self.world > 1:
            with torch.cuda.stream(stream):
                dist.all_gather_into_tensor(recv, send, group=self.group)
        if marks is not None:
            marks[1].record(stream)
        L.check(lib.raven_merge_topk_gathered_device(recv.data_ptr(), self.n_shards, self.world, self.per, nq, k,
                                                     self.shard_size, out[0].data_ptr(), out[1].data_ptr(),
                                                     out[2].data_ptr(), stream.cuda_stream))
        return out

    def search(self, d_queries: torch.Tensor, params: L.SearchParams, stream: torch.cuda.Stream, marks=None):
        """Every query on every shard, then exchange and merge. Returns device
        tensors (ids [nq, k] int32 view of global u32 ids, dists [nq, k],
        counts [nq]); queued on `stream`. `marks`: two CUDA events recorded
        after the searches and after the exchange (for the step's breakdown)."""
        lib = L.load()
        nq, k = d_queries.shape[0], params.k
        send, recv, out = self._buffers(nq, k, d_queries.device, stream)
        for j, s in enumerate(self.order):
            ids, ds, cnt = block_views(send, j, nq, k)
            o = L.SearchOutputs(ids=C.cast(ids.data_ptr(), L.u32p), dists=C.cast(ds.data_ptr(), L.f32p),
                                counts=C.cast(cnt.data_ptr(), L.u32p))
            L.check(lib.raven_search_batch_device(self.shards[s]._h, d_queries.data_ptr(), nq, C.byref(params),
                                                  C.byref(o), stream.cuda_stream))
        if marks is not None:
            marks[0].record(stream)
        return self._exchange_merge(send, recv, out, nq, k, stream, marks)

    def gathered(self, nq: int, k: int, device) -> torch.Tensor:
        """The gathered buffer of the last step with this shape (every shard's
        lists, block (s % world) * per + s // world)."""
        return self._bufs[(nq, k, str(device))][1]

    def exact(self, d_queries: torch.Tensor, k: int, stream: torch.cuda.Stream):
        """The exact top-k of the whole collection: the exact kNN of every local
        shard (raven_knn_exact_device), exchanged and merged the same way."""
        lib = L.load()
        nq = d_queries.shape[0]
        send, recv, out = self._buffers(nq, k, d_queries.device, stream)
        for j, s in enumerate(self.order):
            ids, ds, cnt = block_views(send, j, nq, k)
            L.check(lib.raven_knn_exact_device(self.shards[s]._h, d_queries.data_ptr(), nq, k, ids.data_ptr(),
                                               ds.data_ptr(), stream.cuda_stream))
            with torch.cuda.stream(stream):
                cnt.fill_(k)
        return self._exchange_merge(send, recv, out, nq, k, stream)
