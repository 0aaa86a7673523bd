"""Attention on tensors that live in host memory, with the PCIe copies overlapped.

The operator itself (``gfx906_b200.attn``) takes CUDA tensors, like the
reference's ``attn.cpp``. A caller whose q, k, v are in host memory otherwise
pays upload, compute and download one after the other. ``attn_host`` cuts the
(batch x head) units into contiguous blocks and runs, on three CUDA streams,
the upload of block i+1, the attention of block i and the download of block
i-1 at the same time (PCIe moves data in both directions at once). Every byte
of q, k, v and o still crosses the bus on every call.

Blocks are contiguous in the flattened b * H + h index, so each block's q, k,
v and o are single contiguous ranges of the [B, H, S, D] tensors.

The device copies live in two persistent buffer sets per device, used by
alternate calls. Events order each set's reuse (the uploads of call n + 2 wait
for the kernels of call n, its kernels for the downloads of call n), so back
to back calls allocate nothing and the uploads of one call follow those of the
previous call on the link without waiting for its kernels or downloads. The
kernels run on a third stream of the library's, so the next call's kernels do
not wait for this call's downloads either; only the caller's stream does.
"""

from __future__ import annotations

import threading

import torch

__all__ = ["attn_host"]

_streams = {}
_streams_lock = threading.Lock()
_pools = {}  # device index -> _Pool
# Buffer sets larger than this are allocated per call instead of kept.
_POOL_MAX_BYTES = 2 << 30


def _side_streams(device: torch.device):
    """Upload, download and kernel streams of a device, created on first use."""
    key = device.index
    with _streams_lock:
        trio = _streams.get(key)
        if trio is None:
            trio = tuple(torch.cuda.Stream(device=device) for _ in range(3))
            _streams[key] = trio
    return trio


class _BufferSet:
    """Device copies of q, k, v and o for one call, and the events that say
    when the previous call using them no longer needs them."""

    def __init__(self, units, Sq, Skv, D, dev):
        self.q = torch.empty((units, Sq, D), dtype=torch.float16, device=dev)
        self.k = torch.empty((units, Skv, D), dtype=torch.float16, device=dev)
        self.v = torch.empty((units, Skv, D), dtype=torch.float16, device=dev)
        self.o = torch.empty((units, Sq, D), dtype=torch.float16, device=dev)
        self.kernels_done = None   # compute-stream event after the last kernel reading q, k, v
        self.download_done = None  # download-stream event after the last copy out of o

    def release(self, streams):
        # the side streams may still use these buffers: the caching allocator
        # must not hand them out before those streams get past this point
        for t in (self.q, self.k, self.v, self.o):
            for st in streams:
                t.record_stream(st)


class _Pool:
    def __init__(self, key, dev):
        self.key = key
        self.sets = [_BufferSet(*key[1:], dev), _BufferSet(*key[1:], dev)]
        self.next = 0
        self.lock = threading.Lock()  # one call enqueues on a device at a time
        self.retired = False

    def retire(self, streams):
        # called with self.lock held, when another shape replaces this pool
        self.retired = True
        for bs in self.sets:
            bs.release(streams)


def attn_host(q, k, v, scale, out=None, device=None, blocks=None, non_blocking=False):
    """O = softmax(scale * q @ k^T) @ v for fp16 [B,H,S,D] tensors in host memory.

    q: [B, H, Sq, D]; k, v: [B, H, Skv, D]; all fp16 CPU tensors, contiguous.
    Pinned memory (``tensor.pin_memory()``) is what lets the copies overlap the
    kernel; pageable tensors work but their copies serialise.
    out: optional [B, H, Sq, D] fp16 CPU tensor for the result (allocated
    pinned when None). device: the CUDA device (default: the current one).
    blocks: number of (batch x head) blocks (default min(B*H, 4); for D = 512
    fewer, so that every block still fills the GPU).
    non_blocking: when False the call returns with ``out`` filled; when True it
    returns at once and the current CUDA stream is made to wait for the last
    download, so ``out`` is valid once that stream has been synchronised.
    q, k and v must hold their final values when the call is made: the
    uploads do not wait for work queued on the current stream (a
    ``non_blocking`` device-to-host copy into them must be synchronised
    first).
    """
    from . import _module_or_raise

    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.is_cuda:
            raise ValueError(f"attn_host: {name} must be a host tensor (use gfx906_b200.attn for CUDA tensors)")
        if t.dim() != 4 or t.dtype != torch.float16 or not t.is_contiguous():
            raise ValueError(f"attn_host: {name} must be a contiguous fp16 [B,H,S,D] tensor")
    B, H, Sq, D = q.shape
    if k.shape[:2] != (B, H) or v.shape != k.shape or k.shape[3] != D:
        raise ValueError("attn_host: k and v must be [B, H, Skv, D] matching q")
    if not torch.cuda.is_available():
        raise RuntimeError("attn_host: CUDA is not available")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    elif out.shape != q.shape or out.dtype != q.dtype or out.is_cuda or not out.is_contiguous():
        raise ValueError("attn_host: out must be a contiguous fp16 host tensor shaped like q")
    units = B * H
    if units == 0 or Sq == 0:
        return out
    Skv = k.shape[2]
    # Default 4 blocks: measured on B200 with back-to-back C2 calls, 1-4
    # blocks run at the PCIe copy floor (1.54 ms per call, the same pipeline
    # with no kernel 1.48-1.59 ms) and 8 blocks, 32 copies per call, at 1.71.
    nb = max(1, min(units, 4 if blocks is None else int(blocks)))
    if blocks is None:
        # at least 8 MiB of copies per block: below that, launch and copy
        # latencies cost more than the overlap saves
        moved = 2 * D * units * (2 * Sq + 2 * Skv)
        nb = max(1, min(nb, moved // (8 << 20)))
    if blocks is None and D == 512:
        # The D=512 kernel runs one CTA per (128-row query tile, head-dim half)
        # and does not split key ranges: a block must bring about 1.5 waves of
        # CTAs of its own, or cutting it up costs more kernel time than the
        # overlap saves.
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        ctas_per_unit = 2 * ((Sq + 127) // 128)
        min_units = -(-(3 * sms) // (2 * ctas_per_unit))
        nb = max(1, min(nb, units // max(1, min_units)))
    qf, kf, vf, of = (t.view(units, -1, D) for t in (q, k, v, out))
    mod = _module_or_raise()  # the strict operator: raises if the native code is missing

    with torch.cuda.device(dev):
        caller = torch.cuda.current_stream(dev)
        # Kernels run on a stream of their own, not the caller's: the caller's
        # stream waits for this call's last download, and on it the next
        # call's kernels would wait for that download too.
        up, down, compute = _side_streams(dev)
        key = (dev.index, units, Sq, Skv, D)
        if 2 * D * units * (2 * Sq + 2 * Skv) > _POOL_MAX_BYTES:
            pool, lock = None, threading.Lock()
        else:
            with _streams_lock:
                pool = _pools.get(dev.index)
                if pool is None or pool.key != key:
                    if pool is not None:
                        with pool.lock:
                            pool.retire((down, compute))
                    # allocated on the upload stream, their first user: the
                    # caching allocator only orders reuse on the allocating stream
                    with torch.cuda.stream(up):
                        pool = _Pool(key, dev)
                    _pools[dev.index] = pool
            lock = pool.lock
        with lock:
            if pool is not None and pool.retired:  # replaced by another thread meanwhile
                pool = None
            if pool is None:
                with torch.cuda.stream(up):
                    bs = _BufferSet(units, Sq, Skv, D, dev)
            else:
                bs = pool.sets[pool.next]
                pool.next ^= 1
                if bs.kernels_done is not None:
                    up.wait_event(bs.kernels_done)
                if bs.download_done is not None:
                    compute.wait_event(bs.download_done)
            done = None
            for i in range(nb):
                lo, hi = units * i // nb, units * (i + 1) // nb
                if hi == lo:
                    continue
                with torch.cuda.stream(up):
                    bs.q[lo:hi].copy_(qf[lo:hi], non_blocking=True)
                    bs.k[lo:hi].copy_(kf[lo:hi], non_blocking=True)
                    bs.v[lo:hi].copy_(vf[lo:hi], non_blocking=True)
                    uploaded = torch.cuda.Event()
                    uploaded.record(up)
                compute.wait_event(uploaded)
                with torch.cuda.stream(compute):
                    mod.attn_out(bs.q[lo:hi].unsqueeze(0), bs.k[lo:hi].unsqueeze(0), bs.v[lo:hi].unsqueeze(0),
                                 scale, bs.o[lo:hi].unsqueeze(0))
                computed = torch.cuda.Event()
                computed.record(compute)
                with torch.cuda.stream(down):
                    down.wait_event(computed)
                    of[lo:hi].copy_(bs.o[lo:hi], non_blocking=True)
                    done = torch.cuda.Event()
                    done.record(down)
            bs.kernels_done = torch.cuda.Event()
            bs.kernels_done.record(compute)
            bs.download_done = done
            if pool is None:
                bs.release((down, compute))
            caller.wait_event(done)
    if not non_blocking:
        done.synchronize()
    return out
