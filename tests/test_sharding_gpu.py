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


def _barrier_call(lib, bufs, world, rank, err, dev):
    import ctypes

    sig = (ctypes.c_void_p * world)(*[b.data_ptr() for b in bufs])
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    return lib.la_p2p_barrier(sig, world, rank, ctypes.c_void_p(err.data_ptr()), stream)


def test_p2p_barrier_reports_a_peer_that_never_arrives(pkg, cuda_dev):
    """Rank 0 of a 2-rank gather waits for an epoch that nothing publishes
    (the peer skipped its barrier): the bounded wait runs out, the kernel
    returns with LA_DEVERR_WAIT_TIMEOUT in the error word, the host raises on
    check_device_errors, and the context stays usable. One GPU: both ranks'
    signal words are plain buffers on this device and nothing runs as rank 1."""
    import time

    from lean_infer_b200 import _lib
    from lean_infer_b200 import flash_attn_interface as fai

    lib = _lib.load()
    assert lib.la_init(cuda_dev.index) == 0
    bufs = [torch.zeros(64, dtype=torch.int32, device=cuda_dev) for _ in range(2)]
    err = fai.error_word(cuda_dev.index)
    pkg.check_device_errors(cuda_dev.index)  # start from a clear word
    t0 = time.perf_counter()
    assert _barrier_call(lib, bufs, 2, 0, err, cuda_dev) == 0
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(err.item()) == 1  # LA_DEVERR_WAIT_TIMEOUT
    with pytest.raises(_lib.LeanAttnError, match="bounded wait timed out"):
        pkg.check_device_errors(cuda_dev.index)
    assert waited >= 1.0  # it waited for its bound, it did not return early
    # rank 0 published epoch 1 into both ranks' words
    assert int(bufs[0][0].item()) == 1 and int(bufs[1][0].item()) == 1 and int(bufs[0][2].item()) == 1
    # the peer now publishes its epoch 1 (as its own barrier would): the next
    # wait of rank 0 is for epoch 2, so publish that too and the call passes
    bufs[0][1] = 2
    assert _barrier_call(lib, bufs, 2, 0, err, cuda_dev) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    pkg.check_device_errors(cuda_dev.index)


def _oproj_worker(rank, world, port, out_q):
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
        wo = (torch.randn(1024, 2048, generator=torch.Generator().manual_seed(5)) / 2048 ** 0.5).to(torch.bfloat16)
        wo = wo.to(dev)
        res = []
        for call, seed in enumerate((94, 95, 96)):  # three layers in a row, alternating slots
            w = W.decode_batch(40 + 7 * call, 1, 3000, num_blocks=None, seed=seed)
            kc, vc = S.shard_pool(w.k_cache, w.v_cache, sh)
            y = fused.attention_o_proj(w.q[:, :, sh.q_lo:sh.q_hi].contiguous().to(dev), kc.to(dev), vc.to(dev),
                                       w.cache_seqlens.to(dev), w.block_table.to(dev), wo, slot=call % 2)
            g = fused.local[call % 2][:y.shape[0]].clone()
            res.append((y.cpu(), g.cpu()))
        torch.cuda.synchronize()
        pkg.check_device_errors(rank)
        out_q.put((rank, res))
        fused.close()
    finally:
        dist.destroy_process_group()


def test_kv_head_sharded_o_proj_fused_with_the_gather(pkg):
    """Row f4: decode on each rank's heads, the all-gather stores fused into
    it, and o_proj on tcgen05 consuming the peers' heads as they land (no
    barrier). y must be bit-identical on both ranks, equal the fp32 product
    of the gathered heads to one bf16 rounding, and match the fp32 oracle
    (attention over all heads, then o_proj)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from lean_infer_b200 import workloads as W
    from oracle import paged_attention as opa

    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_oproj_worker, args=(r, 2, port, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(out_q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    wo = (torch.randn(1024, 2048, generator=torch.Generator().manual_seed(5)) / 2048 ** 0.5).to(torch.bfloat16)
    for call, seed in enumerate((94, 95, 96)):
        y0, g0 = got[0][call]
        y1, _ = got[1][call]
        assert torch.equal(y0, y1), call
        B = y0.shape[0]
        exact = g0.view(B, 2048).float() @ wo.float().T
        assert torch.all((y0.float() - exact).abs() <= 2 ** -8 * exact.abs() + 1e-6), call
        w = W.decode_batch(40 + 7 * call, 1, 3000, num_blocks=None, seed=seed)
        o_ref = opa.paged_decode(w.q, w.k_cache, w.v_cache, w.block_table, w.cache_seqlens)
        assert (g0.float() - o_ref[:, 0]).abs().max().item() <= TOL
        y_ref = o_ref.view(B, 2048) @ wo.float().T
        assert (y0.float() - y_ref).abs().max().item() <= TOL * y_ref.abs().max().item() + 1e-3
