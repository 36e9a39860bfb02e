"""KV-head-sharded decode on 2 GPUs over NCCL: each rank runs the sm_100a
decode kernel on its kv heads and the outputs are all-gathered; the result
must match the fp32 oracle over all heads. Skipped with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import REPO

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_q):
    import datetime
    import sys

    sys.path.insert(0, str(REPO))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import __graft_entry__

    pkg = __graft_entry__.load_package()
    import torch.distributed as dist
    from lean_infer_b200 import sharding as S
    from lean_infer_b200 import workloads as W

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        w = W.decode_batch(40, 1, 3000, num_blocks=None, seed=90)  # same requests on every rank (CPU, seeded)
        sh = S.kv_head_shard(rank, world, 8, 16)
        kc, vc = S.shard_pool(w.k_cache, w.v_cache, sh)
        dec = S.KVHeadShardedDecode(sh)
        out = dec(w.q[:, :, sh.q_lo:sh.q_hi].contiguous().to(dev), kc.to(dev), vc.to(dev),
                  w.cache_seqlens.to(dev), w.block_table.to(dev))
        torch.cuda.synchronize()
        pkg.check_device_errors(rank)
        if rank == 0:
            out_q.put(out.cpu())
    finally:
        dist.destroy_process_group()


def test_kv_head_sharded_decode_nccl(pkg):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from lean_infer_b200 import workloads as W
    from oracle import paged_attention as opa

    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    out = out_q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    w = W.decode_batch(40, 1, 3000, num_blocks=None, seed=90)
    ref = opa.paged_decode(w.q, w.k_cache, w.v_cache, w.block_table, w.cache_seqlens)
    assert (out.float() - ref).abs().max().item() <= TOL


def _nvlink_worker(rank, world, port, out_q):
    import datetime
    import sys

    sys.path.insert(0, str(REPO))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import __graft_entry__

    pkg = __graft_entry__.load_package()
    import torch.distributed as dist
    from lean_infer_b200 import sharding as S
    from lean_infer_b200 import workloads as W

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        sh = S.kv_head_shard(rank, world, 8, 16)
        fused = S.NVLinkAllGatherDecode(sh, max_batch=64)
        outs = []
        for call, seed in enumerate((91, 92, 93)):  # three calls in a row, alternating slots
            w = W.decode_batch(40 + call, 1, 3000, num_blocks=None, seed=seed)
            kc, vc = S.shard_pool(w.k_cache, w.v_cache, sh)
            o = fused(w.q[:, :, sh.q_lo:sh.q_hi].contiguous().to(dev), kc.to(dev), vc.to(dev),
                      w.cache_seqlens.to(dev), w.block_table.to(dev), slot=call % 2)
            outs.append(o.cpu().clone() if rank == 0 else None)
        torch.cuda.synchronize()
        pkg.check_device_errors(rank)
        if rank == 0:
            out_q.put(outs)
        fused.close()
    finally:
        dist.destroy_process_group()


def test_kv_head_sharded_decode_nvlink_allgather(pkg):
    """The all-gather fused into the decode kernels (peer stores + epochs)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from lean_infer_b200 import workloads as W
    from oracle import paged_attention as opa

    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nvlink_worker, args=(r, 2, port, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    outs = out_q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for call, seed in enumerate((91, 92, 93)):
        w = W.decode_batch(40 + call, 1, 3000, num_blocks=None, seed=seed)
        ref = opa.paged_decode(w.q, w.k_cache, w.v_cache, w.block_table, w.cache_seqlens)
        assert (outs[call].float() - ref).abs().max().item() <= TOL, call
