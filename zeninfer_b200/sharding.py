"""Multi-GPU layouts of the sampler, one process per GPU.

Row split (the weak-scaling layout): rank g samples its own contiguous range of
rows with its own rng states.  Rows are independent in sample_token
(src/sample.cpp:32-102), so there is no communication and every id equals the
single-GPU id.

Vocab shard (the tensor-parallel lm_head layout): rank g holds columns
[offset_g, offset_g + n_g) of every row.  Each rank selects its local
candidates into one block per row and slice (zs_shard_partials: local top-K
keys with global ids, local max, local sum-exp); the blocks are all-gathered;
every rank merges the G blocks of each row (zs_shard_merge) and draws.  The
global top-K is a subset of the union of the local top-Ks, so the shortlist,
the draw and the rng states are the single-GPU ones on every rank.  The only
collective is that all-gather: about 8 * (K + slack) bytes per row and rank
against 4 * V / G bytes of logits read.
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

    def __init__(self, sampler, group=None):
        import torch.distributed as dist
        self.sampler = sampler
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._send = None
        self._recv = None

    def _buffers(self, nbytes: int):
        import torch
        if self._send is None or self._send.numel() != nbytes:
            dev = self.sampler.device
            self._send = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            self._recv = torch.empty(self.world * nbytes, dtype=torch.uint8, device=dev)
        return self._send, self._recv

    def sample(self, logits_local, vocab_offset: int, n_vocab_total: int, params, rng_state,
               out=None, history=None, history_len=None, stream=None):
        """logits_local: CUDA float32 [B, n_local], this rank's columns of every row.
        rng_state: CUDA int64 [B], identical on every rank (advanced identically).
        Returns the ids (CUDA int32 [B]), identical on every rank."""
        from .sampler import Sampler
        B = logits_local.shape[0]
        nbytes = Sampler.shard_partial_bytes(B, n_vocab_total, self.world, params)
        send, recv = self._buffers(nbytes)
        self.sampler.shard_partials(logits_local, vocab_offset, n_vocab_total, self.world,
                                    params, send, history, history_len, stream=stream)
        all_gather_blocks(recv, send, self.group)
        return self.sampler.shard_merge(recv, self.world, B, n_vocab_total, params, rng_state,
                                        out=out, stream=stream).ids
