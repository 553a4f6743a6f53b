"""Batch sharding across GPUs (one process per GPU).

The Local Attender and the upsampler are independent per image, so the only
parallelism is splitting the image batch into contiguous shards; nothing is
exchanged while computing.  `gather_to_rank0` is the optional final gather of
the per-rank outputs to rank 0 (torch.distributed gather: NCCL over NVLink
on GPUs, gloo on CPUs); the other ranks never receive or hold the full
batch.  `SlotGather` does the same for a stream of micro-batches on the copy
engines (CUDA IPC on one node), overlapped with the computation of the next
micro-batch.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


def shard_bounds(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [lo, hi) slice of n items for `rank`; the first n % world
    ranks get one extra item."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's slice of a batch-first tensor."""
    lo, hi = shard_bounds(t.shape[0], rank, world)
    return t[lo:hi]


def _dense_view(t: torch.Tensor) -> tuple[torch.Tensor, bool]:
    """A contiguous view of a dense tensor, without a copy: a channels_last
    4-D tensor is viewed as NHWC.  Returns (view, was_channels_last)."""
    if t.dim() == 4 and not t.is_contiguous() and t.is_contiguous(memory_format=torch.channels_last):
        return t.permute(0, 2, 3, 1), True
    return t.contiguous(), False


def gather_to_rank0(local: torch.Tensor, n_total: int, group: Optional[dist.ProcessGroup] = None):
    """Concatenate every rank's batch slice on rank 0 in rank order.

    All ranks must call it (it is a collective): a gather to rank 0
    (NCCL over NVLink on GPUs, gloo on CPUs), so only rank 0 receives and
    holds the full batch.  Shards may differ by one item: every rank pads to
    the largest shard for the equal-size gather and rank 0 trims.
    Channels_last tensors travel as their NHWC storage (no layout copy) and
    come back channels_last.  Returns the full batch on rank 0 and None
    elsewhere."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    sizes = [shard_bounds(n_total, r, world) for r in range(world)]
    biggest = max(hi - lo for lo, hi in sizes)
    if local.shape[0] != sizes[rank][1] - sizes[rank][0]:
        raise ValueError(f"rank {rank} holds {local.shape[0]} items, expected {sizes[rank][1] - sizes[rank][0]}")
    if local.shape[0] != biggest:
        padded = torch.zeros_like(local[:1]).expand((biggest,) + tuple(local.shape[1:])).clone(
            memory_format=torch.preserve_format)
        padded[:local.shape[0]] = local
        local = padded
    src, cl = _dense_view(local)
    dst = dist.get_global_rank(group, 0) if group is not None else 0
    if rank != 0:
        dist.gather(src, gather_list=None, dst=dst, group=group)
        return None
    out = torch.empty((world * biggest,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device,
                      memory_format=torch.channels_last if cl else torch.contiguous_format)
    parts = [_dense_view(out[r * biggest:(r + 1) * biggest])[0] for r in range(world)]
    dist.gather(src, gather_list=parts, dst=dst, group=group)
    keep = [out[r * biggest:r * biggest + (hi - lo)] for r, (lo, hi) in enumerate(sizes)]
    return keep[0] if world == 1 else torch.cat(keep, dim=0)


class SlotGather:
    """Streaming gather of fixed per-rank output slots to rank 0 on the copy
    engines (one process per GPU on one node).

    Every rank writes its micro-batch outputs into a few fixed device slots
    (e.g. the outputs of CUDA graphs replayed in turn); rank 0 maps each
    peer's slots once (CUDA IPC, into its own device's context with peer
    access, so its copy engines read them over NVLink) and copies each
    micro-batch into `out`, its [global batch, ...] tensor, with
    cudaMemcpyAsync on one stream per peer, while the ranks compute the next
    micro-batch.  Interprocess events order the two sides: a rank's `ready`
    event (recorded after it wrote a slot) before rank 0 copies it, rank 0's
    `done` event (recorded after the copy) before the rank writes that slot
    again.  A key in `store` per event and micro-batch makes each event
    recorded before the other process waits on it (a stream wait takes the
    event's latest record), so no kernel ever waits on another process.

    Use on every rank, in the same order:

        g = SlotGather(slots, out, offsets, store, rank, world, stream)
        for each micro-batch j:
            g.before_write(j)     # stream waits until slot j % n_slots is free
            ... write the outputs of micro-batch j into slots[j % n_slots] on stream ...
            g.after_write(j, i)   # i: the micro-batch's place in this rank's shard;
                                  # rank 0 enqueues every rank's copies of it
        g.join()                  # rank 0: the stream waits for the copies
        g.close()                 # after a device synchronisation, on every rank

    `offsets[r]` is the index in `out` (dim 0) of rank r's first item; rank
    r's micro-batch j lands at offsets[r] + j * slot_items.  Only rank 0
    holds `out` (None elsewhere).  The micro-batch index j counts across
    calls (keep increasing it), so that slot reuse is ordered across passes.
    """

    def __init__(self, slots, out, offsets, store, rank: int, world: int, stream: torch.cuda.Stream):
        import pickle
        from cuda.bindings import driver as drv
        from cuda.bindings import runtime as rt
        self._rt, self._store, self.rank, self.world, self.stream = rt, store, rank, world, stream
        self.slots = list(slots)
        if len({(t.shape, t.dtype) for t in self.slots}) != 1 or not all(t.is_cuda for t in self.slots):
            raise ValueError("slots must be CUDA tensors of one shape and dtype")
        if any(not (t.is_contiguous() or t.is_contiguous(memory_format=torch.channels_last)) for t in self.slots):
            raise ValueError("slots must be dense")
        self.n_slots = len(self.slots)
        self.items = self.slots[0].shape[0]
        self.nbytes = self.slots[0].numel() * self.slots[0].element_size()
        self.offsets = list(offsets)
        self.out = out
        dev = self.slots[0].device
        self.ready = [torch.cuda.Event(interprocess=True) for _ in range(self.n_slots)]
        self._opened = []

        def ok(res, what):
            if res[0] not in (rt.cudaError_t.cudaSuccess, drv.CUresult.CUDA_SUCCESS):
                raise RuntimeError(f"{what}: {res[0]}")
            return res[1:] if len(res) > 2 else (res[1] if len(res) == 2 else None)

        if rank != 0:
            handles = []
            for t in self.slots:  # (IPC handle of the slot's allocation, offset in it)
                base, _ = ok(drv.cuMemGetAddressRange(t.data_ptr()), "cuMemGetAddressRange")
                h = ok(rt.cudaIpcGetMemHandle(int(base)), "cudaIpcGetMemHandle")
                handles.append((bytes(h.reserved), t.data_ptr() - int(base)))
            store.set(f"sg:h{rank}", pickle.dumps((handles, [e.ipc_handle() for e in self.ready])))
            self.peer_done = [torch.cuda.Event.from_ipc_handle(dev, h)
                              for h in pickle.loads(store.get(f"sg:dh{rank}"))]
            return
        if out is None or not out.is_cuda:
            raise ValueError("rank 0 needs its CUDA output tensor")
        self.done = [[torch.cuda.Event(interprocess=True) for _ in range(self.n_slots)] for _ in range(world)]
        self.peer_ptrs, self.peer_ready, self.copy_streams = [None], [None], [None]
        for r in range(1, world):
            handles, evh = pickle.loads(store.get(f"sg:h{r}"))
            mapped, ptrs = {}, []
            for hb, off in handles:
                if hb not in mapped:  # slots sharing an allocation share one mapping
                    h = rt.cudaIpcMemHandle_t()
                    h.reserved = hb
                    mapped[hb] = int(ok(rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess),
                                        "cudaIpcOpenMemHandle"))
                    self._opened.append(mapped[hb])
                ptrs.append(mapped[hb] + off)
            self.peer_ptrs.append(ptrs)
            self.peer_ready.append([torch.cuda.Event.from_ipc_handle(dev, h) for h in evh])
            self.copy_streams.append(torch.cuda.Stream(dev))
            store.set(f"sg:dh{r}", pickle.dumps([e.ipc_handle() for e in self.done[r]]))
        self.copy_streams[0] = torch.cuda.Stream(dev)

    def _copy(self, dst: torch.Tensor, src_ptr: int, stream: torch.cuda.Stream):
        rt = self._rt
        err, = rt.cudaMemcpyAsync(dst.data_ptr(), src_ptr, self.nbytes, rt.cudaMemcpyKind.cudaMemcpyDefault,
                                  rt.cudaStream_t(stream.cuda_stream))
        if err != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"cudaMemcpyAsync: {err}")

    def before_write(self, j: int):
        """Make the stream wait until slot j % n_slots has been copied out."""
        if j < self.n_slots:
            return
        sl = j % self.n_slots
        if self.rank != 0:
            key = f"sg:d{self.rank}:{j - self.n_slots}"
            self._store.wait([key])
            self._store.delete_key(key)  # one key per event record: the store stays small
            self.stream.wait_event(self.peer_done[sl])
        else:
            self.stream.wait_event(self.done[0][sl])

    def after_write(self, j: int, index: int):
        """Slot j % n_slots holds this rank's micro-batch `index` (its position
        in the rank's shard, in micro-batches); on rank 0 also enqueue every
        rank's copy of it."""
        sl = j % self.n_slots
        self.ready[sl].record(self.stream)
        if self.rank != 0:
            self._store.set(f"sg:r{self.rank}:{j}", b"1")
            return
        cs = self.copy_streams[0]
        cs.wait_event(self.ready[sl])
        lo = self.offsets[0] + index * self.items
        self._copy(self.out[lo:lo + self.items], self.slots[sl].data_ptr(), cs)
        self.done[0][sl].record(cs)
        for r in range(1, self.world):
            self._store.wait([f"sg:r{r}:{j}"])
            self._store.delete_key(f"sg:r{r}:{j}")
            cs = self.copy_streams[r]
            cs.wait_event(self.peer_ready[r][sl])
            lo = self.offsets[r] + index * self.items
            self._copy(self.out[lo:lo + self.items], self.peer_ptrs[r][sl], cs)
            self.done[r][sl].record(cs)
            self._store.set(f"sg:d{r}:{j}", b"1")

    def join(self):
        """Rank 0: make the stream wait for every copy enqueued so far."""
        if self.rank == 0:
            for cs in self.copy_streams:
                self.stream.wait_stream(cs)

    def close(self):
        """Rank 0 unmaps the peers' slots; call on every rank after a device
        synchronisation, and free the slots only after every rank returned
        (e.g. after a barrier)."""
        for base in self._opened:
            self._rt.cudaIpcCloseMemHandle(base)
        self._opened = []
