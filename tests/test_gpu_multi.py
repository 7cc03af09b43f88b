"""Two GPUs, one process each: the vocab-sharded sampler over NCCL gives every
rank the single-GPU ids and rng states,

  * through the package's torch.distributed path (VocabShardedSampler): the
    row-owner exchange (grouped sends of each owner's block spans, the owner's
    merge, an all-gather of ids and states) and the all-gather route, on a batch
    that divides by the world size and on one that does not;
  * through the C ABI's own zs_sample_sharded (an NCCL communicator created with
    the process's libnccl): the row-owner route, and with row info the route that
    merges every row on every rank.

Then one rank stops taking part (it never makes its next zs_sample_sharded
call): the other rank's call must return ZS_ERR_NCCL within its collective
timeout, having aborted the communicator, and its handle must still sample
correctly.  The rank that stopped leaves only between steps, with nothing of its
own in flight; NVLS is off (NCCL_NVLS_ENABLE=0).  Skipped with fewer than two
GPUs."""

import ctypes as C
import os
import socket
import time
import traceback
from datetime import timedelta

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WORLD = 2
ZS_ERR_NCCL = 5


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class NcclUniqueId(C.Structure):
    _fields_ = [("internal", C.c_char * 128)]


def _worker(rank, port, q):
    try:
        import torch
        import torch.distributed as dist
        from zeninfer_b200 import Sampler, SamplingParams, states_to_tensor, tensor_to_states
        from zeninfer_b200 import sharding
        from zeninfer_b200 import workloads as W
        from zeninfer_b200._native import SamplerError
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD,
                                timeout=timedelta(seconds=30), device_id=dev)
        s = Sampler(rank)
        V = W.VOCAB
        x_all = torch.from_numpy(W.generate(5, 385, row0=900)).to(dev)
        lo, n = sharding.vocab_range(V, WORLD, rank)
        results = {}

        def single(x, p):
            st = states_to_tensor(W.WORKLOADS[5].row_states(0, x.shape[0]), dev)
            ids = s.sample(x, p, st, sync_check=True, row_info=True)
            return ids.ids.cpu().numpy(), tensor_to_states(st), ids.row_info

        def same(a_ids, a_st, b_ids, b_st):
            return (bool(np.array_equal(a_ids, b_ids.cpu().numpy())),
                    bool(np.array_equal(a_st, tensor_to_states(b_st))))

        for name, p in (("k50", SamplingParams(temp=0.7, top_k=50, top_p=0.9)),
                        ("greedy", SamplingParams()),
                        ("k256", SamplingParams(temp=1.0, top_p=0.95)),
                        ("k1024", SamplingParams(temp=0.8, top_k=1024))):
            for rows in ((384, 385) if name == "k50" else (384,)):
                x = x_all[:rows]
                one_ids, one_st, _ = single(x, p)
                for owner in (True, False):
                    st_sh = states_to_tensor(W.WORKLOADS[5].row_states(0, rows), dev)
                    sh = sharding.VocabShardedSampler(s, owner=owner).sample(
                        x[:, lo:lo + n].contiguous(), lo, V, p, st_sh)
                    torch.cuda.synchronize()
                    s.check_device_status()
                    results[f"torch_{name}_{rows}_{'owner' if owner else 'gather'}"] = \
                        same(one_ids, one_st, sh, st_sh)
        # the C ABI's own NCCL path: a communicator from this process's libnccl
        nccl = C.CDLL("libnccl.so.2")
        uid = NcclUniqueId()
        if rank == 0:
            assert nccl.ncclGetUniqueId(C.byref(uid)) == 0
        # the raw 128 bytes (a c_char array's value would stop at the first NUL)
        obj = [C.string_at(C.addressof(uid), C.sizeof(uid)) if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        C.memmove(C.addressof(uid), obj[0], C.sizeof(uid))
        comm = C.c_void_p()
        assert nccl.ncclCommInitRank(C.byref(comm), WORLD, uid, rank) == 0
        p = SamplingParams(temp=0.7, top_k=50, top_p=0.9)
        for rows in (384, 385):
            x = x_all[:rows]
            one_ids, one_st, one_info = single(x, p)
            xl = x[:, lo:lo + n].contiguous()
            st_c = states_to_tensor(W.WORKLOADS[5].row_states(0, rows), dev)
            ids_c = s.sample_sharded(xl, lo, V, WORLD, p, st_c, comm.value)
            torch.cuda.synchronize()
            s.check_device_status()
            results[f"c_abi_owner_{rows}"] = same(one_ids, one_st, ids_c, st_c)
            st_c = states_to_tensor(W.WORKLOADS[5].row_states(0, rows), dev)
            ids_c, info = s.sample_sharded(xl, lo, V, WORLD, p, st_c, comm.value, row_info=True)
            torch.cuda.synchronize()
            ok_ids, ok_st = same(one_ids, one_st, ids_c, st_c)
            results[f"c_abi_full_{rows}"] = (ok_ids and bool(np.array_equal(info["m"],
                                                                              one_info["m"])),
                                             ok_st)
        # A rank stops taking part: rank 1 skips the next step.  Rank 0's call must
        # come back with ZS_ERR_NCCL inside its timeout, not wait for good.
        x = x_all[:384]
        one_ids, one_st, _ = single(x, p)
        xl = x[:, lo:lo + n].contiguous()
        if rank == 0:
            s.set_collective_timeout(2000)
            st_c = states_to_tensor(W.WORKLOADS[5].row_states(0, 384), dev)
            t0 = time.monotonic()
            status = 0
            try:
                s.sample_sharded(xl, lo, V, WORLD, p, st_c, comm.value)
            except SamplerError as e:
                status = e.status
            dt = time.monotonic() - t0
            torch.cuda.synchronize()
            # the handle still samples correctly after the abort
            after_ids, after_st, _ = single(x, p)
            results["dropout"] = (status == ZS_ERR_NCCL and dt < 20.0,
                                  bool(np.array_equal(after_ids, one_ids) and
                                       np.array_equal(after_st, one_st)))
            results["dropout_seconds"] = dt
        dist.barrier()  # rank 1 waits here until rank 0's call has returned
        if rank == 1:
            nccl.ncclCommAbort(comm)  # local: its peer has already aborted
        else:
            pass  # rank 0's communicator was aborted (and freed) by zs_sample_sharded
        s.close()
        dist.destroy_process_group()
        q.put((rank, results))
    except Exception:
        q.put((rank, "exception:" + traceback.format_exc()))


@pytest.mark.skipif(_gpus() < WORLD, reason="needs two GPUs")
def test_vocab_shard_two_gpus():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q), daemon=True) for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=240) for _ in procs)
    finally:  # never leave a rank behind, whatever happened
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(WORLD):
        assert not isinstance(res[r], str), res[r]
        for name, val in res[r].items():
            if name.endswith("_seconds"):
                continue
            ids_ok, st_ok = val
            assert ids_ok and st_ok, (r, name, ids_ok, st_ok, res[r].get("dropout_seconds"))
    assert "dropout" in res[0]
