"""Multi-rank logic of the two decode partitionings, on CPU with gloo ranks
(world size 2 and 4): head/request partitions and the KV-head all-gather
reassembly, with the oracle as each rank's local attention. The same classes
run on NCCL with the sm_100a kernel on GPUs (tests/test_sharding_gpu.py)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import REPO


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partitions(pkg):
    from lean_infer_b200 import sharding as S

    shards = [S.kv_head_shard(r, 4, 8, 16) for r in range(4)]
    assert [(s.kv_lo, s.kv_hi, s.q_lo, s.q_hi) for s in shards] == [(0, 2, 0, 4), (2, 4, 4, 8), (4, 6, 8, 12),
                                                                    (6, 8, 12, 16)]
    one = S.kv_head_shard(3, 8, 8, 16)
    assert (one.num_kv_heads, one.num_q_heads, one.q_lo) == (1, 2, 6)
    with pytest.raises(ValueError):
        S.kv_head_shard(0, 3, 8, 16)
    reqs = [S.request_shard(r, 3, 1024) for r in range(3)]
    assert sum(len(x) for x in reqs) == 1024 and reqs[0].stop == reqs[1].start and reqs[-1].stop == 1024


def _worker(rank, world, port, q, k_cache, v_cache, bt, seqlens, out_q):
    import sys

    sys.path.insert(0, str(REPO))
    import __graft_entry__

    __graft_entry__.load_package()
    import torch.distributed as dist
    from lean_infer_b200 import sharding as S
    from oracle import paged_attention as opa

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = S.kv_head_shard(rank, world, 8, 16)
        kc, vc = S.shard_pool(k_cache, v_cache, sh)

        def local(qq, kk, vv, sl, b):
            return opa.paged_decode(qq, kk, vv, b, sl).to(qq.dtype)

        dec = S.KVHeadShardedDecode(sh, local_attn=local)
        out = dec(q[:, :, sh.q_lo:sh.q_hi].contiguous(), kc, vc, seqlens, bt)
        if rank == 0:
            out_q.put(out)
        # rank 0 hosts the rendezvous store: no rank may still be talking to
        # it when rank 0 tears its process group down
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_kv_head_sharded_decode_gloo(pkg, world):
    """Sharded + gathered output == the unsharded oracle."""
    from lean_infer_b200 import workloads as W
    from oracle import paged_attention as opa

    w = W.decode_batch(6, 1, 700, num_blocks=None, seed=70)
    q = w.q.float()
    kc, vc = w.k_cache.float(), w.v_cache.float()
    ref = opa.paged_decode(q, kc, vc, w.block_table, w.cache_seqlens)
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, kc, vc, w.block_table, w.cache_seqlens, out_q))
             for r in range(world)]
    for p in procs:
        p.start()
    out = out_q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)


def _dead_rank_worker(rank, world, port, res_q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, before the collective
    t = torch.ones(4)
    try:
        dist.all_gather_into_tensor(torch.empty(8), t)
        res_q.put("completed")
    except Exception as e:  # the short process-group timeout ends the collective with an error
        res_q.put(type(e).__name__)


def test_rank_loss_ends_collective_with_error(pkg):
    """A rank that leaves between steps makes the others' next all-gather fail
    with an error after the process-group timeout, instead of hanging."""
    ctx = mp.get_context("spawn")
    res_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, 2, port, res_q)) for r in range(2)]
    for p in procs:
        p.start()
    res = res_q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res != "completed"
