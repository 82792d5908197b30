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
  `raven_merge_topk_device`, ties ordered by (distance, shard, rank in the
  shard's list). Searching each shard exactly as the reference searches one
  graph and merging by that rule gives the same ids as running the reference
  on every shard and merging its outputs on the host.

The exchange packs a shard's lists into one int32 tensor [nq, 2k + 1]
(ids, distance bit patterns, count) so that a step needs one all-gather;
it works unchanged on NCCL (CUDA tensors) and gloo (CPU tensors, used by the
CPU tests of this module).
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


def pack_lists(ids: torch.Tensor, dists: torch.Tensor, counts: torch.Tensor) -> torch.Tensor:
    """[n, nq, k] ids (int32 view of u32), [n, nq, k] f32, [n, nq] counts ->
    [n, nq, 2k + 1] int32 (distances as bit patterns)."""
    if ids.shape != dists.shape or counts.shape != ids.shape[:2]:
        raise ValueError("ids, dists must be [n, nq, k] and counts [n, nq]")
    return torch.cat([ids.to(torch.int32), dists.contiguous().view(torch.int32),
                      counts.to(torch.int32).unsqueeze(-1)], dim=-1)


def unpack_lists(packed: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    ids = packed[..., :k].contiguous()
    dists = packed[..., k:2 * k].contiguous().view(torch.float32)
    counts = packed[..., 2 * k].contiguous()
    return ids, dists, counts


def exchange_shard_lists(local: torch.Tensor, n_shards: int, group=None) -> torch.Tensor:
    """All-gather the packed lists of this rank's shards ([len(shards_of_rank),
    nq, 2k + 1]) and return every shard's lists in shard order
    ([n_shards, nq, 2k + 1]). Ranks holding fewer shards pad their block, so
    every rank sends the same shape."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    mine = shards_of_rank(n_shards, world, rank)
    if local.shape[0] != len(mine):
        raise ValueError(f"rank {rank} holds {len(mine)} shards, got lists for {local.shape[0]}")
    per = -(-n_shards // world)
    block = local.new_zeros((per,) + tuple(local.shape[1:]))
    block[:local.shape[0]] = local
    gathered = [torch.empty_like(block) for _ in range(world)]
    dist.all_gather(gathered, block, group=group)
    return torch.stack([gathered[s % world][s // world] for s in range(n_shards)])


class ShardedCollection:
    """Per-shard device indexes of this rank and the search-exchange-merge step.

    `shards` maps shard number -> DeviceIndex for the shards this rank holds
    (exactly `shards_of_rank(n_shards, world, rank)`); every shard but the last
    covers `shard_size` global ids.
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

    def search(self, d_queries: torch.Tensor, params: L.SearchParams, stream: torch.cuda.Stream):
        """Every query on every shard, then exchange and merge. Returns device
        tensors (ids [nq, k] int32 view of global u32 ids, dists [nq, k],
        counts [nq]); queued on `stream`."""
        lib = L.load()
        nq, k = d_queries.shape[0], params.k
        dev = d_queries.device
        with torch.cuda.stream(stream):  # every allocation and fill is ordered on the launch stream
            ids = torch.zeros((len(self.order), nq, k), dtype=torch.int32, device=dev)
            ds = torch.zeros((len(self.order), nq, k), dtype=torch.float32, device=dev)
            cnt = torch.zeros((len(self.order), nq), dtype=torch.int32, device=dev)
        for j, s in enumerate(self.order):
            out = L.SearchOutputs(ids=C.cast(ids[j].data_ptr(), L.u32p), dists=C.cast(ds[j].data_ptr(), L.f32p),
                                  counts=C.cast(cnt[j].data_ptr(), L.u32p))
            L.check(lib.raven_search_batch_device(self.shards[s]._h, d_queries.data_ptr(), nq, C.byref(params),
                                                  C.byref(out), stream.cuda_stream))
        with torch.cuda.stream(stream):
            packed = pack_lists(ids, ds, cnt)
            if self.world > 1:
                packed = exchange_shard_lists(packed, self.n_shards, self.group)
            all_i, all_d, all_c = unpack_lists(packed, k)
            out_i = torch.zeros((nq, k), dtype=torch.int32, device=dev)
            out_d = torch.zeros((nq, k), dtype=torch.float32, device=dev)
            out_c = torch.zeros(nq, dtype=torch.int32, device=dev)
        L.check(lib.raven_merge_topk_device(all_i.data_ptr(), all_d.data_ptr(), all_c.data_ptr(), self.n_shards, nq, k,
                                            self.shard_size, out_i.data_ptr(), out_d.data_ptr(), out_c.data_ptr(),
                                            stream.cuda_stream))
        return out_i, out_d, out_c
