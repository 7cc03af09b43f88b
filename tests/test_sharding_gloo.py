"""The vocab-sharded exchange on CPU: two gloo ranks, world size 2.

Each rank takes its vocab_range of every row, selects its local top-K as
candidate keys (value descending, id ascending; the key order the kernels
use), packs them into one block per row, and the blocks go through
sharding.all_gather_blocks -- the collective the GPU path uses.  Merging the
gathered blocks must give the global shortlist of the restatement on every
rank.  A second test drops one rank before the collective: the survivor gets
an error from the short process-group timeout instead of waiting forever.

The row-owner exchange (sharding.exchange_owner_blocks and the ids/states
all-gather) runs on world sizes 2 and 3 with the library's own block spans
(zs_shard_row_spans, host arithmetic only): every owner must end up with each
rank's bytes at exactly the spans of its rows.
"""

import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest

ROWS, V, K = 6, 5003, 40   # V not divisible by 2: the last rank takes the remainder


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _keys(vals, ids):
    u = vals.astype(np.float32).view(np.uint32).astype(np.uint64)
    u = np.where(vals == 0, np.uint64(0), u)  # -0 == +0
    ordv = np.where(u & np.uint64(0x80000000), ~u & np.uint64(0xFFFFFFFF), u | np.uint64(0x80000000))
    ordv = np.where(np.isnan(vals), np.uint64(0), ordv)
    return (ordv << np.uint64(32)) | (~ids.astype(np.uint64) & np.uint64(0xFFFFFFFF))


def _rows():
    return np.random.default_rng(123).normal(0, 2, size=(ROWS, V)).astype(np.float32)


def _worker(rank, world, port, mode, q):
    try:
        import torch
        import torch.distributed as dist
        from zeninfer_b200 import sharding
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=10))
        if mode == "drop" and rank == 1:
            dist.destroy_process_group()
            q.put((rank, "left"))
            return
        x = _rows()
        lo, n = sharding.vocab_range(V, world, rank)
        blk_words = 2 + K  # header (count, pad) + keys, as uint64 words
        send = np.zeros((ROWS, blk_words), dtype=np.uint64)
        for r in range(ROWS):
            keys = _keys(x[r, lo:lo + n], np.arange(lo, lo + n))
            top = np.sort(keys)[::-1][:K]
            send[r, 0] = top.size
            send[r, 2:2 + top.size] = top
        send_t = torch.from_numpy(send.view(np.uint8).reshape(-1).copy())
        recv_t = torch.empty(world * send_t.numel(), dtype=torch.uint8)
        try:
            sharding.all_gather_blocks(recv_t, send_t)
        except Exception as e:  # the peer is gone: the collective must fail, not hang
            q.put((rank, "error:" + type(e).__name__))
            return
        recv = recv_t.numpy().view(np.uint64).reshape(world, ROWS, blk_words)
        shortlists = []
        for r in range(ROWS):
            allk = np.concatenate([recv[g, r, 2:2 + int(recv[g, r, 0])] for g in range(world)])
            top = np.sort(allk)[::-1][:K]
            shortlists.append((~(top & np.uint64(0xFFFFFFFF)) & np.uint64(0xFFFFFFFF))
                              .astype(np.int64).tolist())
        q.put((rank, shortlists))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "exception:" + traceback.format_exc()))


def _run(mode):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q), daemon=True) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=120) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return res


def test_vocab_shard_exchange_gives_global_shortlist():
    import oracle
    from zeninfer_b200 import SamplingParams, rng_seed
    res = _run("ok")
    for r in (0, 1):
        assert not isinstance(res[r], str), res[r]
    assert res[0] == res[1]
    x = _rows()
    st = np.array([rng_seed(i + 1) for i in range(ROWS)], dtype=np.uint64)
    _, _, cid, _, _ = oracle.oracle_sample(x, SamplingParams(temp=1.0, top_k=K), st, cand_ld=K)
    assert [list(map(int, row)) for row in cid] == res[0]


def test_dropped_rank_fails_the_collective():
    res = _run("drop")
    assert res[1] == "left"
    assert isinstance(res[0], str) and res[0].startswith("error:"), res[0]


def _owner_worker(rank, world, port, batch, q):
    try:
        import torch
        import torch.distributed as dist
        from zeninfer_b200 import Sampler, SamplingParams, sharding
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=20))
        out = {}
        for name, p in (("k50", SamplingParams(temp=0.7, top_k=50, top_p=0.9)),
                        ("k1500", SamplingParams(temp=1.0, top_k=1500))):
            nbytes = Sampler.shard_partial_bytes(batch, 151936, world, p)
            spans = [Sampler.shard_row_spans(batch, 151936, world, p,
                                             *Sampler.shard_owner_rows(batch, world, o))
                     for o in range(world)]
            pattern = lambda g: ((torch.arange(nbytes, dtype=torch.int64) * 7 + g * 31) % 251
                                 ).to(torch.uint8)
            slots = torch.zeros(world * nbytes, dtype=torch.uint8)
            slots[rank * nbytes:(rank + 1) * nbytes] = pattern(rank)
            sharding.exchange_owner_blocks(slots, nbytes, spans)
            ok = True
            for g in range(world):
                want = pattern(g)
                for off, ln in spans[rank]:
                    got = slots[g * nbytes + off:g * nbytes + off + ln]
                    ok = ok and bool(torch.equal(got, want[off:off + ln]))
            # the owners' results to every rank: rows r0..r0+n written by their owner only
            R = (batch + world - 1) // world
            ids = torch.full((world * R,), -1, dtype=torch.int32)
            r0, n = Sampler.shard_owner_rows(batch, world, rank)
            assert r0 == rank * R or n == 0
            ids[r0:r0 + n] = torch.arange(r0, r0 + n, dtype=torch.int32) * 10 + rank
            sharding._all_gather_own(ids, R, rank)
            want_ids = [r * 10 + min(r // R, world - 1) for r in range(batch)]
            out[name] = (ok, ids[:batch].tolist() == want_ids, len(spans[rank]))
        q.put((rank, out))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "exception:" + traceback.format_exc()))


@pytest.mark.parametrize("world,batch", [(2, 4096), (2, 5), (3, 7)])
def test_row_owner_exchange(world, batch):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_owner_worker, args=(r, world, port, batch, q), daemon=True)
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=120) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert not isinstance(res[r], str), res[r]
        for name, (spans_ok, ids_ok, nspans) in res[r].items():
            assert spans_ok and ids_ok, (r, name, spans_ok, ids_ok, nspans)
