"""K/V broadcast on the copy engines, between the GPUs of one node.

NCCL's collectives are kernels: while the persistent attention kernel holds
every SM, a broadcast enqueued beside it cannot start, so query-row sharding
(``shard.attention_by_rows``) pays for the broadcast of the next call's K and
V on top of this call's kernel. A device-to-device copy that reads another
GPU's memory runs on the copy engines instead and overlaps the kernel.

``KVBroadcast`` keeps a ring of ``depth`` K/V buffer pairs on every rank,
mapped into the neighbouring ranks' address spaces with CUDA IPC
(``cudaIpcGetMemHandle`` / ``cudaIpcOpenMemHandle``, opened on the rank's
own device with lazy peer access). The ranks form a tree rooted at the
source (by default every other rank is the source's child); each rank pulls
a call's K and V from its parent's ring into its own with one
``cudaMemcpyAsync`` each on a copy stream: the data crosses NVLink once per
rank, into local memory, and the kernel reads it from there.

Ordering across processes uses inter-process CUDA events plus per-rank call
counters in host shared memory (``Board``). A rank records an event and only
then publishes the call's index; a rank that needs that event waits for the
index on the host before it enqueues the wait on the event, so it never
waits on an older recording of the same event. Per call i (buffer pair b =
i % depth), with "have" the event a rank records once its pair b holds call
i:

* source, ``source(i)``: the host waits until every child has published
  "have i - depth", the current stream waits for their events: pair b may
  be rewritten. The caller writes call i's K and V into the returned pair.
* source, ``start(i)``: records "have" on the current stream and publishes i.
* other ranks, ``start(i)``: wait until the parent has published i; the
  copy stream waits for the parent's "have", for the children's "have" of
  call i - depth and for this rank's own last use of pair b (``release``),
  pulls K and V, records "have" and publishes i.
* every rank, ``wait(i)``: the current stream waits for call i's K/V;
  returns the pair. ``release(i)`` after enqueuing the kernels that read it.

``RowGather`` does the reverse for the output: every rank pushes its block
of query rows into the other ranks' output rings.

Host waits carry a time limit, so a rank that died leaves the others with an
error instead of a hang. No kernel of this module waits on another GPU, and
nothing here uses multicast. All ranks must be on one node (CUDA IPC and the
shared-memory board both need it).
"""

from __future__ import annotations

import time
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

# Board channels of KVBroadcast and RowGather
_HAVE = 0
_FREED, _PUSHED = 0, 1


def _rt():
    try:
        from cuda.bindings import driver, runtime
    except ImportError as e:  # pragma: no cover - cuda-python ships with the image
        raise RuntimeError(f"copy-engine transport needs cuda-python: {e}") from e
    return runtime, driver


def _check(res, what: str):
    """Raises on a non-zero status; returns the call's outputs (None, one, or a tuple)."""
    if not isinstance(res, tuple):
        res = (res,)
    err, out = res[0], res[1:]
    if int(err) != 0:
        raise RuntimeError(f"{what} failed: {err}")
    if not out:
        return None
    return out[0] if len(out) == 1 else out


def export_tensor(t: torch.Tensor) -> Tuple[bytes, int]:
    """(IPC handle of the allocation holding t, byte offset of t in it)."""
    rt, drv = _rt()
    ptr = t.data_ptr()
    base, _size = _check(drv.cuMemGetAddressRange(ptr), "cuMemGetAddressRange")
    handle = _check(rt.cudaIpcGetMemHandle(int(base)), "cudaIpcGetMemHandle")
    return bytes(handle.reserved), ptr - int(base)


def open_handle(handle: bytes) -> int:
    """Maps another process's allocation into this device's address space."""
    rt, _ = _rt()
    h = rt.cudaIpcMemHandle_t()
    h.reserved = handle
    return int(_check(rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle"))


def close_handle(base: int) -> None:
    rt, _ = _rt()
    rt.cudaIpcCloseMemHandle(base)


def copy_async(dst: int, src: int, nbytes: int, stream: int) -> None:
    """cudaMemcpyAsync device to device (a peer source runs on a copy engine)."""
    rt, _ = _rt()
    _check(rt.cudaMemcpyAsync(dst, src, nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice, stream),
           "cudaMemcpyAsync")


class _IpcEvent:
    """An inter-process CUDA event (no timing), created here or opened from a handle."""

    def __init__(self, handle: Optional[bytes] = None):
        rt, _ = _rt()
        self._rt = rt
        if handle is None:
            flags = rt.cudaEventInterprocess | rt.cudaEventDisableTiming
            self.ev = _check(rt.cudaEventCreateWithFlags(flags), "cudaEventCreateWithFlags")
            self.handle = bytes(_check(rt.cudaIpcGetEventHandle(self.ev), "cudaIpcGetEventHandle").reserved)
        else:
            h = rt.cudaIpcEventHandle_t()
            h.reserved = handle
            self.ev = _check(rt.cudaIpcOpenEventHandle(h), "cudaIpcOpenEventHandle")
            self.handle = handle

    def record(self, stream: int) -> None:
        _check(self._rt.cudaEventRecord(self.ev, stream), "cudaEventRecord")

    def wait_on(self, stream: int) -> None:
        _check(self._rt.cudaStreamWaitEvent(stream, self.ev, 0), "cudaStreamWaitEvent")

    def destroy(self) -> None:
        self._rt.cudaEventDestroy(self.ev)


class Board:
    """Per-rank, per-channel monotonic counters in host shared memory, for
    ranks on one node: ``publish(ch, i)`` sets this rank's counter of channel
    ch to i + 1 (calls are published in increasing order), ``wait(ch, ranks,
    i)`` returns once every listed rank has published call i. A round trip is
    a few microseconds, against tens for a key in the process group's store,
    which matters at several handshakes per call and call times of a tenth of
    a millisecond. A wait gives up with TimeoutError after `timeout_s`, so a
    rank that died leaves the others with an error instead of a hang.
    Construction is collective over `group` (rank 0 creates the segment and
    removes its name once every rank has mapped it)."""

    def __init__(self, channels: int, group=None, timeout_s: float = 120.0):
        import numpy as np
        from multiprocessing import resource_tracker, shared_memory

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.timeout_s = timeout_s
        size = 8 * channels * self.world
        shm = shared_memory.SharedMemory(create=True, size=size) if self.rank == 0 else None
        names: list = [None] * self.world
        dist.all_gather_object(names, shm.name if shm is not None else None, group=group)
        if shm is None:
            shm = shared_memory.SharedMemory(name=names[0])
            # the creator owns the segment; this process must not unlink it at exit
            resource_tracker.unregister(shm._name, "shared_memory")  # noqa: SLF001
        self._shm = shm
        self.arr = np.ndarray((channels, self.world), dtype=np.int64, buffer=shm.buf)
        if self.rank == 0:
            self.arr[:] = 0
        dist.barrier(group=group)
        if self.rank == 0:
            shm.unlink()  # every rank has it mapped; the name is no longer needed

    def publish(self, ch: int, i: int) -> None:
        self.arr[ch, self.rank] = i + 1

    def wait(self, ch: int, ranks, i: int) -> None:
        row = self.arr[ch]
        need = i + 1
        pending = [r for r in ranks if row[r] < need]
        if not pending:
            return
        deadline = time.monotonic() + self.timeout_s
        n = 0
        while pending:
            pending = [r for r in pending if row[r] < need]
            n += 1
            if n > 32:
                time.sleep(0)
            if (n & 1023) == 0 and time.monotonic() > deadline:
                raise TimeoutError(f"rank(s) {pending} did not publish call {i} on channel {ch} "
                                   f"within {self.timeout_s} s")

    def close(self) -> None:
        self.arr = None
        self._shm.close()


class KVBroadcast:
    """K and V of every call from rank `src` to all ranks of `group`, pulled
    on the copy engines (see the module docstring).

    The ranks form a tree rooted at `src` with `fanout` children per rank
    (default: every other rank is a child of the source). A rank pulls each
    call's K and V from its parent's ring into its own, and its children
    pull from it once it has them, so the source serves `fanout` pulls per
    call instead of world - 1. One inter-process event per ring pair and
    rank ("have": recorded once the pair holds the call) serves both
    directions: the children wait on it before pulling, the parent before
    refilling the pair with call i + depth; one board channel publishes it.

    shape, dtype: one K (or V) tensor. depth: buffer pairs in the ring (2
    lets call i + 1's transfer run during call i's kernel). Construction is
    collective over `group` (an exchange of IPC handles)."""

    def __init__(self, shape, dtype=torch.float16, src: int = 0, group=None, depth: int = 2,
                 device: Optional[torch.device] = None, fanout: Optional[int] = None):
        if depth < 2:
            raise ValueError("depth must be >= 2")
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.src, self.depth, self.group = src, depth, group
        self.is_source = self.rank == src
        self.fanout = max(1, self.world - 1 if fanout is None else int(fanout))
        pos = (self.rank - src) % self.world
        self.parent = None if pos == 0 else (src + (pos - 1) // self.fanout) % self.world
        self.children: List[int] = [(src + c) % self.world
                                    for c in range(pos * self.fanout + 1, pos * self.fanout + self.fanout + 1)
                                    if c < self.world]
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        ring = torch.empty((depth, 2) + tuple(shape), dtype=dtype, device=self.device)
        self.k = [ring[b, 0] for b in range(depth)]
        self.v = [ring[b, 1] for b in range(depth)]
        self.nbytes = self.k[0].numel() * self.k[0].element_size()
        # calls issued so far: call indices run on across uses, every rank alike
        self.calls = 0
        self._sourced = -1
        self.copy_stream = torch.cuda.Stream(self.device)
        self.board = Board(1, group)  # channel HAVE: this rank's ring holds call i
        self._mapped: dict = {}
        self._events: List[_IpcEvent] = []
        with torch.cuda.device(self.device):
            self.have = [self._event() for _ in range(depth)]
            if not self.is_source:
                self.released = [torch.cuda.Event() for _ in range(depth)]
                self.arrived = [torch.cuda.Event() for _ in range(depth)]
            handle, off = export_tensor(ring)
            payload = {"ring": (handle, off), "have": [e.handle for e in self.have]}
            payloads: list = [None] * self.world
            dist.all_gather_object(payloads, payload, group=group)
            self.child_have = {c: [self._event(h) for h in payloads[c]["have"]] for c in self.children}
            if self.parent is not None:
                handle, off = payloads[self.parent]["ring"]
                if handle not in self._mapped:
                    self._mapped[handle] = open_handle(handle)
                base = self._mapped[handle] + off
                pair = 2 * self.nbytes
                self.parent_k = [base + b * pair for b in range(depth)]
                self.parent_v = [base + b * pair + self.nbytes for b in range(depth)]
                self.parent_have = [self._event(h) for h in payloads[self.parent]["have"]]

    def _event(self, handle: Optional[bytes] = None) -> _IpcEvent:
        e = _IpcEvent(handle)
        self._events.append(e)
        return e

    def _children_done(self, i: int, stream: int) -> None:
        """`stream` waits until every child has pulled call i - depth out of
        pair b (so the pair may take call i)."""
        if i >= self.depth and self.children:
            b = i % self.depth
            self.board.wait(_HAVE, self.children, i - self.depth)
            for c in self.children:
                self.child_have[c][b].wait_on(stream)

    def source(self, i: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Source rank: the pair to write call i's K and V into, once every
        child has pulled what the pair held before (the current stream waits
        for that)."""
        if not self.is_source:
            raise RuntimeError("source() is for the source rank")
        b = i % self.depth
        self._sourced = i
        self._children_done(i, torch.cuda.current_stream(self.device).cuda_stream)
        return self.k[b], self.v[b]

    def start(self, i: int) -> None:
        """Source: call i's K/V are complete once the current stream reaches
        this point. Other ranks: enqueue the pull of call i's K/V from the
        parent."""
        b = i % self.depth
        if self.is_source:
            if self._sourced != i:  # the pair must be free of call i - depth's pulls first
                self.source(i)
            self.have[b].record(torch.cuda.current_stream(self.device).cuda_stream)
            self.board.publish(_HAVE, i)
            return
        self.board.wait(_HAVE, [self.parent], i)
        cs = self.copy_stream.cuda_stream
        self.parent_have[b].wait_on(cs)
        self._children_done(i, cs)
        if i >= self.depth:
            self.copy_stream.wait_event(self.released[b])
        copy_async(self.k[b].data_ptr(), self.parent_k[b], self.nbytes, cs)
        copy_async(self.v[b].data_ptr(), self.parent_v[b], self.nbytes, cs)
        self.have[b].record(cs)
        self.board.publish(_HAVE, i)
        self.arrived[b].record(self.copy_stream)

    def wait(self, i: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """The current stream waits for call i's K/V; returns them."""
        b = i % self.depth
        if not self.is_source:
            torch.cuda.current_stream(self.device).wait_event(self.arrived[b])
        return self.k[b], self.v[b]

    def release(self, i: int) -> None:
        """Call after enqueuing the last kernel that reads call i's K/V."""
        if not self.is_source:
            self.released[i % self.depth].record(torch.cuda.current_stream(self.device))

    def close(self) -> None:
        """Collective: every rank's copies are done before any buffer or
        mapping goes away."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for e in self._events:
            e.destroy()
        self._events = []
        for base in self._mapped.values():
            close_handle(base)
        self._mapped = {}
        self.board.close()


class RowGather:
    """Every call's output assembled on every rank by the copy engines: each
    rank pushes its block of query rows into the other ranks' output rings
    (CUDA IPC) right after its kernel has written them, instead of an NCCL
    all-gather (a kernel, which would have to wait for free SMs).

    out_shape: [B, H, Sq, D] with B * H == 1 (a rank's row block is then one
    contiguous range); rows: (start, stop) of every rank's block. Per call i
    (ring slot b = i % depth):

    * ``begin(i)``: this rank's slot b may be written by the other ranks
      (recorded on the current stream, so after whatever consumed call
      i - depth's output), and this rank's own push of call i - depth has
      read its rows (the current stream waits);
    * the kernel writes this rank's rows of ``out(i)`` (``rows_out(i)``);
    * ``push(i)``: after that kernel, the copy stream waits for every other
      rank's "begin i", then copies the rows into their slot b;
    * ``complete(i)``: the current stream waits for every other rank's push
      of call i: ``out(i)`` then holds the whole output until call i + depth
      begins; or ``ack(i)`` when nobody reads call i's output: the host
      only waits until every other rank has enqueued its push of call i.

    One of the two must run for call i before ``begin(i + depth)``: a rank
    re-records its "begin" and "pushed" events only after every other rank
    has enqueued its wait on the previous recording. Construction is
    collective over `group`."""

    def __init__(self, out_shape, rows, dtype=torch.float16, group=None, depth: int = 2,
                 device: Optional[torch.device] = None):
        B, H, Sq, D = out_shape
        if B * H != 1:
            raise ValueError("RowGather needs B * H == 1 (contiguous row blocks)")
        if depth < 2:
            raise ValueError("depth must be >= 2")
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.depth, self.group = depth, group
        self.peers = [r for r in range(self.world) if r != self.rank]
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.ring = torch.empty((depth,) + tuple(out_shape), dtype=dtype, device=self.device)
        self.row_bytes = D * self.ring.element_size()
        self.slot_bytes = Sq * self.row_bytes
        self.start_row, self.stop_row = rows[self.rank]
        self.copy_stream = torch.cuda.Stream(self.device)
        self.calls = 0
        self.board = Board(2, group)  # channels FREED, PUSHED
        self._mapped: dict = {}
        self._events: List[_IpcEvent] = []
        with torch.cuda.device(self.device):
            self.pushed = [self._event() for _ in range(depth)]
            self.freed = [self._event() for _ in range(depth)]
            self.push_read = [torch.cuda.Event() for _ in range(depth)]
            self.written = [torch.cuda.Event() for _ in range(depth)]
            handle, off = export_tensor(self.ring)
            payload = {"ring": (handle, off), "pushed": [e.handle for e in self.pushed],
                       "freed": [e.handle for e in self.freed]}
            payloads: list = [None] * self.world
            dist.all_gather_object(payloads, payload, group=group)
            self.peer_ring, self.peer_pushed, self.peer_freed = {}, {}, {}
            for p in self.peers:
                h, o = payloads[p]["ring"]
                if h not in self._mapped:
                    self._mapped[h] = open_handle(h)
                self.peer_ring[p] = self._mapped[h] + o
                self.peer_pushed[p] = [self._event(x) for x in payloads[p]["pushed"]]
                self.peer_freed[p] = [self._event(x) for x in payloads[p]["freed"]]

    def _event(self, handle: Optional[bytes] = None) -> _IpcEvent:
        e = _IpcEvent(handle)
        self._events.append(e)
        return e

    def out(self, i: int) -> torch.Tensor:
        return self.ring[i % self.depth]

    def rows_out(self, i: int) -> torch.Tensor:
        return self.ring[i % self.depth][:, :, self.start_row:self.stop_row]

    def begin(self, i: int) -> None:
        b = i % self.depth
        cur = torch.cuda.current_stream(self.device)
        if i >= self.depth:
            cur.wait_event(self.push_read[b])
        self.freed[b].record(cur.cuda_stream)
        self.board.publish(_FREED, i)

    def push(self, i: int) -> None:
        b = i % self.depth
        cur = torch.cuda.current_stream(self.device)
        self.written[b].record(cur)
        self.copy_stream.wait_event(self.written[b])
        cs = self.copy_stream.cuda_stream
        nbytes = (self.stop_row - self.start_row) * self.row_bytes
        if self.peers and nbytes > 0:
            self.board.wait(_FREED, self.peers, i)
            src = self.rows_out(i).data_ptr()
            off = b * self.slot_bytes + self.start_row * self.row_bytes
            for p in self.peers:
                self.peer_freed[p][b].wait_on(cs)
                copy_async(self.peer_ring[p] + off, src, nbytes, cs)
        self.push_read[b].record(self.copy_stream)
        self.pushed[b].record(cs)
        self.board.publish(_PUSHED, i)

    def ack(self, i: int) -> None:
        if self.peers:
            self.board.wait(_PUSHED, self.peers, i)

    def complete(self, i: int) -> torch.Tensor:
        b = i % self.depth
        self.ack(i)
        cur = torch.cuda.current_stream(self.device).cuda_stream
        for p in self.peers:
            self.peer_pushed[p][b].wait_on(cur)
        return self.out(i)

    def close(self) -> None:
        """Collective: every rank's copies are done before any buffer or
        mapping goes away."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for e in self._events:
            e.destroy()
        self._events = []
        for base in self._mapped.values():
            close_handle(base)
        self._mapped = {}
        self.board.close()
