"""Batch sharding and the final gather, on CPU with gloo (world size 2 and 3),
including a rank that fails: the others see the failure through a short
process-group timeout instead of hanging."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from uplift_b200.sharding import SlotGather, gather_to_rank0, shard, shard_bounds


def test_shard_bounds_cover_in_order():
    for n in (0, 1, 5, 8, 64, 67):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, fail_rank, q):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        full = torch.arange(n * 3, dtype=torch.float32).reshape(n, 3)
        local = shard(full, rank, world) * 2.0          # per-rank "compute"
        if rank == fail_rank:
            raise RuntimeError("injected failure before the gather")
        got = gather_to_rank0(local, n)
        # channels_last images travel as their NHWC storage
        imgs = torch.arange(n * 4 * 3 * 5, dtype=torch.float32).reshape(n, 4, 3, 5)
        imgs = imgs.contiguous(memory_format=torch.channels_last)
        got_cl = gather_to_rank0(shard(imgs, rank, world) + 1.0, n)
        if rank == 0:
            q.put(("ok", torch.equal(got, full * 2.0) and torch.equal(got_cl, imgs + 1.0)
                   and got_cl.is_contiguous(memory_format=torch.channels_last)))
        else:
            q.put(("ok", got is None and got_cl is None))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put(("err", f"rank {rank}: {type(e).__name__}"))
    finally:
        dist.destroy_process_group()


def _run(world, n, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


@pytest.mark.parametrize("world,n", [(2, 8), (2, 7), (3, 5)])
def test_gather_to_rank0_gloo(world, n):
    res = _run(world, n)
    assert all(kind == "ok" and flag for kind, flag in res), res


def test_failed_rank_is_detected_by_timeout():
    res = _run(2, 8, fail_rank=1)
    kinds = sorted(kind for kind, _ in res)
    assert kinds == ["err", "err"], res  # the failing rank and the one left waiting both end


def test_slot_gather_rejects_host_and_mixed_slots():
    """SlotGather (the copy-engine gather over CUDA IPC) validates its slots
    before touching a device: host tensors and slots of different shapes are
    refused."""
    with pytest.raises(ValueError, match="CUDA tensors"):
        SlotGather([torch.zeros(2, 3), torch.zeros(2, 3)], None, [0, 2], None, 1, 2, None)
    with pytest.raises(ValueError, match="one shape"):
        SlotGather([torch.zeros(2, 3), torch.zeros(4, 3)], None, [0, 2], None, 1, 2, None)
