"""Two GPUs, one process each: the vocab-sharded sampler over NCCL gives every
rank the single-GPU ids and rng states, through the package's all-gather path
(torch.distributed) and through the C ABI's own zs_sample_sharded (an NCCL
communicator created with the process's libnccl).  Skipped with fewer than two
GPUs."""

import ctypes as C
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WORLD = 2


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
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD,
                                timeout=timedelta(seconds=30), device_id=dev)
        s = Sampler(rank)
        rows, V = 384, W.VOCAB
        x = torch.from_numpy(W.generate(5, rows, row0=900)).to(dev)
        lo, n = sharding.vocab_range(V, WORLD, rank)
        results = {}
        for name, p in (("k50", SamplingParams(temp=0.7, top_k=50, top_p=0.9)),
                        ("greedy", SamplingParams()),
                        ("k256", SamplingParams(temp=1.0, top_p=0.95)),
                        ("k1024", SamplingParams(temp=0.8, top_k=1024))):
            st0 = W.WORKLOADS[5].row_states(0, rows)
            st_one = states_to_tensor(st0, dev)
            one = s.sample(x, p, st_one, sync_check=True).ids.cpu().numpy()
            st_sh = states_to_tensor(st0, dev)
            sh = sharding.VocabShardedSampler(s).sample(x[:, lo:lo + n].contiguous(), lo, V, p,
                                                        st_sh)
            torch.cuda.synchronize()
            s.check_device_status()
            results[name] = (bool(np.array_equal(one, sh.cpu().numpy())),
                             bool(np.array_equal(tensor_to_states(st_one), tensor_to_states(st_sh))))
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
        st0 = W.WORKLOADS[5].row_states(0, rows)
        st_one = states_to_tensor(st0, dev)
        one = s.sample(x, p, st_one, sync_check=True).ids.cpu().numpy()
        st_c = states_to_tensor(st0, dev)
        ids_c = s.sample_sharded(x[:, lo:lo + n].contiguous(), lo, V, WORLD, p, st_c, comm.value)
        torch.cuda.synchronize()
        s.check_device_status()
        results["c_abi"] = (bool(np.array_equal(one, ids_c.cpu().numpy())),
                            bool(np.array_equal(tensor_to_states(st_one), tensor_to_states(st_c))))
        nccl.ncclCommDestroy(comm)
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
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in range(WORLD):
        assert not isinstance(res[r], str), res[r]
        for name, (ids_ok, st_ok) in res[r].items():
            assert ids_ok and st_ok, (r, name, ids_ok, st_ok)
