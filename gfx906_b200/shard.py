"""Multi-GPU partitioning of the attention forward (one process per GPU).

The path partitions without any exchange on the data path: every
(batch, head, query-row block) is independent given its K and V. Two layouts,
as the north star of this build describes them:

* ``"heads"``: the B*H (batch x head) units are cut into contiguous blocks,
  one per rank; each rank holds and computes only its own units.
* ``"rows"``: for few heads with very long sequences (e.g. B=1, H=1,
  S=131072), the query rows are cut into contiguous blocks of whole 256-row
  kernel query blocks, one per rank, and K/V -- held by one source rank -- are
  replicated to every rank with one NCCL broadcast each before the kernel runs.

``attention_sharded`` picks between the two for q, k, v held on every rank:
(batch x head) blocks while every rank gets at least one unit, query-row
blocks otherwise (C4's 4 heads on 8 GPUs).

Optionally the output blocks are all-gathered. Collectives happen only before
and after the local kernel call (``torch.distributed`` over NCCL on GPUs; the
same code runs over gloo on CPU in the tests). The local compute is
``gfx906_b200.attn`` (the sm_100a kernel); tests inject a CPU stand-in.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

ROW_ALIGN = 256  # query rows per kernel CTA unit: row shards stay whole units


@dataclass(frozen=True)
class Shard:
    """A contiguous [start, stop) block of units (heads or query rows)."""

    start: int
    stop: int

    @property
    def size(self) -> int:
        return self.stop - self.start


def split_even(n: int, world: int, rank: int, align: int = 1) -> Shard:
    """Rank's block of n items cut into `world` near-equal blocks of whole `align` groups."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    groups = (n + align - 1) // align
    lo = groups * rank // world
    hi = groups * (rank + 1) // world
    return Shard(min(n, lo * align), min(n, hi * align))


def head_shard(B: int, H: int, rank: int, world: int) -> Shard:
    """Rank's block of the flattened (batch x head) index b * H + h."""
    return split_even(B * H, world, rank)


def row_shard(Sq: int, rank: int, world: int) -> Shard:
    """Rank's block of query rows, in whole 256-row kernel units."""
    return split_even(Sq, world, rank, ROW_ALIGN)


def _default_attn():
    import gfx906_b200

    return gfx906_b200.attn


def _group_world(group):
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0  # a single process: no collectives
    return dist.get_world_size(group), dist.get_rank(group)


def _gather_dim(local: torch.Tensor, counts, dim: int, group, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """All-gather the ranks' blocks along `dim` (block r has counts[r] entries).

    Equal blocks (the usual case: C5's rows on 1/2/4/8 GPUs, C2's heads) go
    through one ``all_gather_into_tensor`` straight into the output when `dim`
    is the outermost dimension that is not 1, with no staging copies.
    Otherwise the blocks are padded to the largest, gathered, and
    concatenated. `out`, when given, receives the result (its shape must be
    the gathered shape)."""
    world = len(counts)
    full = list(local.shape)
    full[dim] = sum(counts)
    if out is not None and list(out.shape) != full:
        raise ValueError(f"out has shape {tuple(out.shape)}, the gathered shape is {tuple(full)}")
    outer = 1
    for n in local.shape[:dim]:
        outer *= n
    if len(set(counts)) == 1 and outer == 1 and local.is_contiguous():
        dst = out if out is not None and out.is_contiguous() else local.new_empty(full)
        dist.all_gather_into_tensor(dst.view(-1), local.view(-1), group=group)
        if out is not None and dst is not out:
            out.copy_(dst)
            return out
        return dst
    biggest = max(counts)
    pad = list(local.shape)
    pad[dim] = biggest
    buf = local.new_zeros(pad)
    buf.narrow(dim, 0, local.shape[dim]).copy_(local)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    res = torch.cat([p.narrow(dim, 0, c) for p, c in zip(parts, counts)], dim=dim)
    if out is not None:
        out.copy_(res)
        return out
    return res


def attention_by_heads(q, k, v, scale, group=None, gather=True,
                       local_attn: Optional[Callable] = None):
    """Each rank computes its block of (batch x head) units; q/k/v are full
    [B,H,S,D] tensors present on every rank (only the rank's slice is read).
    Returns the full output if `gather`, else this rank's [units, Sq, D] block."""
    attn = local_attn or _default_attn()
    world, rank = _group_world(group)
    B, H, Sq, D = q.shape
    sh = head_shard(B, H, rank, world)
    qf = q.reshape(B * H, Sq, D)[sh.start:sh.stop]
    kf = k.reshape(B * H, k.shape[2], D)[sh.start:sh.stop]
    vf = v.reshape(B * H, v.shape[2], D)[sh.start:sh.stop]
    out = attn(qf.unsqueeze(0), kf.unsqueeze(0), vf.unsqueeze(0), scale).squeeze(0)
    if not gather:
        return out
    if world == 1:
        return out.reshape(B, H, Sq, D)
    counts = [head_shard(B, H, r, world).size for r in range(world)]
    return _gather_dim(out, counts, 0, group).reshape(B, H, Sq, D)


def attention_by_rows(q_rows, k, v, scale, Sq: int, src: Optional[int] = 0, group=None, gather=True,
                      local_attn: Optional[Callable] = None, out: Optional[torch.Tensor] = None):
    """Query-row sharding with K/V replicated from rank `src`.

    q_rows: this rank's query rows [B, H, rows, D] (its `row_shard` of Sq).
    k, v: full [B, H, Skv, D] on rank `src`; on other ranks tensors of the
    same shape and dtype that receive the broadcast. src=None: every rank
    already holds k and v (no broadcast).
    Returns the full [B, H, Sq, D] output if `gather` (written into `out` when
    given), else this rank's rows.
    """
    attn = local_attn or _default_attn()
    world, rank = _group_world(group)
    sh = row_shard(Sq, rank, world)
    if q_rows.shape[2] != sh.size:
        raise ValueError(f"rank {rank} holds {q_rows.shape[2]} query rows, its shard is {sh.size}")
    if world > 1 and src is not None:
        dist.broadcast(k, src=src, group=group)
        dist.broadcast(v, src=src, group=group)
    local = attn(q_rows, k, v, scale) if sh.size > 0 else q_rows.new_zeros(q_rows.shape)
    if not gather or world == 1:
        if out is not None and gather:
            out.copy_(local)
            return out
        return local
    counts = [row_shard(Sq, r, world).size for r in range(world)]
    return _gather_dim(local, counts, 2, group, out=out)


def broadcast_kv(k, v, src: int = 0, group=None, async_op: bool = False):
    """Replicate K and V from rank `src` (one NCCL broadcast each).

    With async_op the broadcasts are enqueued on the collective stream after
    the work already issued on the current stream, and a list of two work
    handles is returned; `wait()` on them makes the current stream wait. A
    caller can so broadcast the next call's K/V while this call's kernel runs
    (the kernel reads other buffers)."""
    world, _ = _group_world(group)
    if world == 1:
        return []
    wk = dist.broadcast(k, src=src, group=group, async_op=async_op)
    wv = dist.broadcast(v, src=src, group=group, async_op=async_op)
    return [wk, wv] if async_op else []


def gather_rows(local, Sq: int, out: torch.Tensor, group=None, async_op: bool = False):
    """All-gather the ranks' query-row blocks of O into `out` ([B, H, Sq, D]).

    Equal blocks with B * H == 1 (C5 on 1/2/4/8 GPUs) go through one
    all_gather_into_tensor straight into `out`; with async_op its work
    handle is returned (None otherwise, or when the gather had to run
    synchronously through the padded path)."""
    world, rank = _group_world(group)
    if world == 1:
        out.copy_(local)
        return None
    counts = [row_shard(Sq, r, world).size for r in range(world)]
    outer = local.shape[0] * local.shape[1]
    if async_op and len(set(counts)) == 1 and outer == 1 and local.is_contiguous() and out.is_contiguous():
        return dist.all_gather_into_tensor(out.view(-1), local.view(-1), group=group, async_op=True)
    _gather_dim(local, counts, 2, group, out=out)
    return None


def _device_sms(t: torch.Tensor) -> int:
    return torch.cuda.get_device_properties(t.device).multi_processor_count


def attention_by_rows_pipelined(calls, Sq: int, src: int = 0, group=None, reserve_sms: int = 16,
                                local_attn: Optional[Callable] = None):
    """A sequence of query-row sharded calls with their collectives overlapped.

    calls: iterable of (q_rows, k, v, scale, out) as for attention_by_rows
    (k, v full on rank `src`, receive buffers elsewhere; out the gathered
    [B, H, Sq, D] output). Call i + 1's K/V broadcast and call i's output
    gather run on the collective stream while call i's kernel runs, so
    consecutive calls must not share k, v or out buffers (alternating two
    sets is enough: a broadcast into a set is enqueued after the kernel that
    last read it). The kernel is capped at the device's SMs minus
    `reserve_sms`, which the NCCL kernels use meanwhile (a persistent kernel
    on every SM would hold them off until it ends). Measured on two B200s:
    with 16 SMs left over the broadcast and the gather of C5 at S=32768 hide
    behind the kernel (0.209 ms per call against 0.255 in sequence; the cap
    costs the kernel ~11%), with 8 they do not fit and mostly serialise. It
    pays where the collectives take more than the cap costs: at S=131072 on
    two GPUs they are 4% of the kernel and the plain sequence is faster.
    Returns the outputs, all written once the current stream reaches this
    point.
    """
    import contextlib

    calls = list(calls)
    if not calls:
        return []
    attn = local_attn or _default_attn()
    world, rank = _group_world(group)
    sh = row_shard(Sq, rank, world)
    limit = contextlib.nullcontext()
    if local_attn is None and reserve_sms > 0 and calls[0][0].is_cuda:
        import gfx906_b200

        limit = gfx906_b200.sm_limit(max(2, _device_sms(calls[0][0]) - reserve_sms))
    outs = []
    with limit:
        pending = broadcast_kv(calls[0][1], calls[0][2], src=src, group=group, async_op=True)
        gathers = []
        for i, (q_rows, k, v, scale, out) in enumerate(calls):
            if q_rows.shape[2] != sh.size:
                raise ValueError(f"rank {rank} holds {q_rows.shape[2]} query rows, its shard is {sh.size}")
            for w in pending:
                w.wait()
            pending = []
            if i + 1 < len(calls):
                pending = broadcast_kv(calls[i + 1][1], calls[i + 1][2], src=src, group=group, async_op=True)
            local = attn(q_rows, k, v, scale) if sh.size > 0 else q_rows.new_zeros(q_rows.shape)
            gathers.append(gather_rows(local, Sq, out, group=group, async_op=True))
            outs.append(out)
        for w in gathers:
            if w is not None:
                w.wait()
    return outs


def attention_by_rows_copy_engine(q_rows_list, bc, scale, Sq: int, outs=None, group=None, fill=None, rg=None,
                                  consume=None, local_attn: Optional[Callable] = None):
    """A sequence of query-row sharded calls with K/V moved on the copy engines.

    bc: a ``peer.KVBroadcast`` over `group` (its source rank holds K/V). Call
    i's K and V reach every rank through bc's ring while call i - 1's kernel
    runs: the transfer needs no SM, so the kernel keeps every SM. On the
    source rank ``fill(i, k, v)`` writes call i's K/V into the ring pair (None:
    the pairs already hold them).

    Output, without `rg`: each call's rows are all-gathered (NCCL) into
    ``outs[i]`` after its kernel; returns outs. With `rg` (a
    ``peer.RowGather``; B * H == 1): the kernel writes this rank's rows into
    rg's ring and they are pushed to the other ranks on the copy engines;
    ``consume(i, out)`` gets call i's whole output once the current stream
    has waited for it (valid until call i + rg.depth begins); without
    `consume` only the last call's output is completed; returns it.
    """
    n = len(q_rows_list)
    if n == 0:
        return outs
    world, rank = _group_world(group)
    sh = row_shard(Sq, rank, world)
    for q_rows in q_rows_list:
        if q_rows.shape[2] != sh.size:
            raise ValueError(f"rank {rank} holds {q_rows.shape[2]} query rows, its shard is {sh.size}")
    if rg is not None:
        if local_attn is not None:
            raise ValueError("rg writes through the operator's attn_out; local_attn is not supported with it")
        import gfx906_b200

        attn_out = gfx906_b200._module_or_raise().attn_out
        j0 = rg.calls
        rg.calls += n
    else:
        attn = local_attn or _default_attn()
    i0 = bc.calls  # the rings' call indices continue from earlier uses
    bc.calls += n

    def begin(i):
        if bc.is_source:
            k, v = bc.source(i0 + i)
            if fill is not None:
                fill(i, k, v)
        bc.start(i0 + i)

    last = None
    begin(0)
    for i in range(n):
        k, v = bc.wait(i0 + i)
        if i + 1 < n:
            begin(i + 1)
        if rg is None:
            local = attn(q_rows_list[i], k, v, scale) if sh.size > 0 else q_rows_list[i].new_zeros(
                q_rows_list[i].shape)
            bc.release(i0 + i)
            gather_rows(local, Sq, outs[i], group=group)
            continue
        j = j0 + i
        rg.begin(j)
        if sh.size > 0:
            attn_out(q_rows_list[i], k, v, scale, rg.rows_out(j))
        bc.release(i0 + i)
        rg.push(j)
        if consume is not None:
            consume(i, rg.complete(j))
        elif i + 1 == n:
            last = rg.complete(j)
        else:
            rg.ack(j)
    return outs if rg is None else last


def choose_partition(B: int, H: int, world: int) -> str:
    """"heads" while every rank gets at least one (batch x head) unit, else "rows"."""
    return "heads" if B * H >= world else "rows"


def attention_sharded(q, k, v, scale, group=None, gather=True, partition: str = "auto",
                      local_attn: Optional[Callable] = None):
    """q, k, v: full [B, H, S, D] tensors on every rank. Each rank computes its
    block of (batch x head) units, or -- with fewer units than ranks, or
    partition="rows" -- its block of whole 256-row query blocks against the
    full K/V it already holds (no broadcast). Returns the full output if
    `gather`, else this rank's block ([units, Sq, D] or [B, H, rows, D])."""
    world, rank = _group_world(group)
    B, H, Sq, _ = q.shape
    if partition == "auto":
        partition = choose_partition(B, H, world)
    if partition == "heads":
        return attention_by_heads(q, k, v, scale, group=group, gather=gather, local_attn=local_attn)
    if partition != "rows":
        raise ValueError(f"unknown partition {partition!r}")
    sh = row_shard(Sq, rank, world)
    return attention_by_rows(q[:, :, sh.start:sh.stop].contiguous(), k, v, scale, Sq, src=None, group=group,
                             gather=gather, local_attn=local_attn)
