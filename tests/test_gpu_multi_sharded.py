"""Sequence-sharded decode over NCCL: one process per GPU (2-4 GPUs when the
box has them, skipped otherwise), with the selection from exchanged
statistics and with the score-row all-gather, over NCCL and (statistics
exchange) over peer-mapped memory.  Every rank must return the output the
single-GPU step computes on rank 0's device."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

Hq, Hkv, D, BS, S = 32, 8, 128, 16, (1 << 18) + 77
KW = dict(avg_budget=64, k_min=2, k_max=512)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(dev):
    g = torch.Generator(device=dev).manual_seed(9)
    q = torch.randn((Hq, D), device=dev, generator=g).to(torch.bfloat16)
    K = torch.randn((Hkv, S, D), device=dev, generator=g).to(torch.bfloat16)
    V = torch.randn((Hkv, S, D), device=dev, generator=g).to(torch.bfloat16)
    return q, K, V


def _rank(rank, world, port, results, selection, comm_kind):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta
    import torch.distributed as dist
    from adakv_b200.sharded import PeerGroup, ShardedDecoder, TorchGroup, shard_range
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        q, K, V = _inputs(dev)
        nb = -(-S // BS)
        lo, n = shard_range(nb, world, rank)
        t0, t1 = lo * BS, min(S, (lo + n) * BS)
        comm = PeerGroup() if comm_kind == "peer" else TorchGroup()
        dec = ShardedDecoder(K[:, t0:t1].contiguous(), V[:, t0:t1].contiguous(), S, Hq, BS,
                             comm, selection=selection, **KW)
        del K, V
        out = dec.step(q)
        out2 = dec.step(q)  # a second step reuses every buffer
        torch.cuda.synchronize(dev)
        same = bool(torch.equal(out, out2))
        if comm_kind == "peer":
            same = same and not comm.timed_out()
        outs = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(outs, out)
        if rank == 0:
            from adakv_b200.batch import BatchedDecoder
            q, K, V = _inputs(dev)
            ref = BatchedDecoder(1, Hq, Hkv, D, BS, S, torch.bfloat16, dev, **KW)
            ref.load(K[None], V[None], [S])
            r = ref.step(q[None])[0].float()
            errs = [float((o.float() - r).abs().max()) for o in outs]
            results.put((errs, same))
        dist.barrier()
        if comm_kind == "peer":
            comm.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("selection,comm_kind", [("stats", "nccl"), ("rows", "nccl"),
                                                 ("stats", "peer")])
def test_sharded_decode_over_nccl(selection, comm_kind):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 or more GPUs")
    world = min(4, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, results, selection, comm_kind))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert [p.exitcode for p in procs] == [0] * world
    errs, same = results.get(timeout=10)
    assert same
    assert max(errs) < 2e-2, errs
