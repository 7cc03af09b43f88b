"""Multi-GPU layouts of the sampler, one process per GPU.

Row split (the weak-scaling layout): rank g samples its own contiguous range of
rows with its own rng states.  Rows are independent in sample_token
(src/sample.cpp:32-102), so there is no communication and every id equals the
single-GPU id.

Vocab shard (the tensor-parallel lm_head layout): rank g holds columns
[offset_g, offset_g + n_g) of every row.  Each rank selects its local
candidates into blocks (zs_shard_partials: local top-K keys with global ids,
local max, local sum-exp).  The global top-K is a subset of the union of the
local top-Ks, so merging a row's blocks from every rank gives the single-GPU
shortlist, draw and rng state.  Two exchanges:

  * row-owner (VocabShardedSampler, the default): rank o owns rows
    owner_rows(o); every rank sends o the byte spans of its block area that
    hold o's rows (grouped point-to-point sends), o merges only its rows, and
    the owners' ids and rng states are all-gathered.  Per rank: about 1/G of the
    blocks received, B/G rows merged, 12 bytes per row gathered.
  * all-gather (VocabShardedSampler(..., owner=False)): every rank receives
    every block area and merges every row.
"""

from __future__ import annotations

from typing import Optional, Tuple


def row_range(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """(first row, row count) of `rank`: contiguous, sizes differ by at most 1."""
    if world <= 0 or not 0 <= rank < world or batch < 0:
        raise ValueError("bad row split")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def vocab_range(n_vocab: int, world: int, rank: int) -> Tuple[int, int]:
    """(vocab offset, column count) of `rank`: equal contiguous slices, the last
    rank also takes the remainder."""
    if world <= 0 or not 0 <= rank < world or n_vocab <= 0:
        raise ValueError("bad vocab split")
    per = n_vocab // world
    lo = rank * per
    hi = n_vocab if rank == world - 1 else lo + per
    return lo, hi - lo


def all_gather_blocks(recv, send, group=None) -> None:
    """recv[g * len(send):(g + 1) * len(send)] = rank g's send, for every rank g.
    One collective, the same call on every rank."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    n = send.numel()
    if recv.numel() != world * n:
        raise ValueError("recv must hold world_size blocks of send's size")
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(recv, send, group=group)
    else:
        dist.all_gather(list(recv.view(world, n).unbind(0)), send, group=group)


class VocabShardedSampler:
    """Vocab-sharded sample_token over a process group (NCCL on GPUs)."""

    def __init__(self, sampler, group=None, owner: bool = True):
        import torch.distributed as dist
        self.sampler = sampler
        self.group = group
        self.owner = owner
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._key = None
        self._slots = None
        self._ids = None
        self._states = None

    def _buffers(self, batch: int, nbytes: int):
        import torch
        R = (batch + self.world - 1) // self.world
        if self._key != (batch, nbytes):
            dev = self.sampler.device
            self._slots = torch.empty(self.world * nbytes, dtype=torch.uint8, device=dev)
            self._ids = torch.empty(self.world * R, dtype=torch.int32, device=dev)
            self._states = torch.empty(self.world * R, dtype=torch.int64, device=dev)
            self._key = (batch, nbytes)
        return self._slots, self._ids, self._states, R

    def sample(self, logits_local, vocab_offset: int, n_vocab_total: int, params, rng_state,
               out=None, history=None, history_len=None, stream=None):
        """logits_local: CUDA float32 [B, n_local], this rank's columns of every row.
        rng_state: CUDA int64 [B], identical on every rank (advanced identically).
        Returns the ids (CUDA int32 [B]), identical on every rank."""
        import torch
        from .sampler import Sampler
        B = logits_local.shape[0]
        G, rank = self.world, self.rank
        nbytes = Sampler.shard_partial_bytes(B, n_vocab_total, G, params)
        slots, ids_pad, st_pad, R = self._buffers(B, nbytes)
        mine = slots[rank * nbytes:(rank + 1) * nbytes]
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=self.sampler.device)
        self.sampler.shard_partials(logits_local, vocab_offset, n_vocab_total, G, params, mine,
                                    history, history_len, stream=stream)
        if not self.owner:
            all_gather_blocks(slots, mine.clone(), self.group)
            return self.sampler.shard_merge(slots, G, B, n_vocab_total, params, rng_state,
                                            out=out, stream=stream).ids
        # 1. blocks of each owner's rows to that owner
        spans = [Sampler.shard_row_spans(B, n_vocab_total, G, params,
                                         *Sampler.shard_owner_rows(B, G, o)) for o in range(G)]
        exchange_owner_blocks(slots, nbytes, spans, self.group)
        # 2. the owner merges its rows into [G][R] arrays: the caller's own when
        #    B = G * R, padded copies otherwise
        r0, n = Sampler.shard_owner_rows(B, G, rank)
        needs_rng = rng_state is not None
        direct = G * R == B
        ids_buf = out if direct else ids_pad
        st_buf = rng_state if direct else st_pad
        if needs_rng and not direct:
            st_pad[:B].copy_(rng_state)
        self.sampler.shard_merge(slots, G, B, n_vocab_total, params,
                                 st_buf if needs_rng else None, out=ids_buf, stream=stream,
                                 rows=(r0, n))
        # 3. every owner's ids and rng states to every rank
        _all_gather_own(ids_buf, R, rank, self.group)
        if needs_rng:
            _all_gather_own(st_buf, R, rank, self.group)
        if not direct:
            if needs_rng:
                rng_state.copy_(st_pad[:B])
            out.copy_(ids_pad[:B])
        return out


def exchange_owner_blocks(slots, nbytes: int, spans, group=None) -> None:
    """Row-owner exchange of partial block areas.  slots: [world * nbytes] bytes, this
    rank's area at slot `rank`; spans[o]: the (offset, length) ranges of an area that
    the merge of owner o's rows reads.  Afterwards slot g of this rank holds rank g's
    bytes at every range of spans[rank].  One batch of point-to-point operations, the
    same calls on every rank."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    mine = slots[rank * nbytes:(rank + 1) * nbytes]
    ops = []
    for peer in range(world):
        if peer == rank:
            continue
        for off, ln in spans[peer]:
            ops.append(dist.P2POp(dist.isend, mine[off:off + ln], peer, group))
        base = peer * nbytes
        for off, ln in spans[rank]:
            ops.append(dist.P2POp(dist.irecv, slots[base + off:base + off + ln], peer, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


def _all_gather_own(buf, R: int, rank: int, group=None) -> None:
    """buf[g * R:(g + 1) * R] = rank g's own entries, for every rank g (in place on
    NCCL)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    own = buf[rank * R:(rank + 1) * R]
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(buf, own, group=group)
    else:
        parts = [buf[g * R:(g + 1) * R].clone() for g in range(world)]
        dist.all_gather(parts, own.clone(), group=group)
        for g in range(world):
            buf[g * R:(g + 1) * R].copy_(parts[g])
