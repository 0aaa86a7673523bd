"""Multi-rank partitioning logic on CPU: world_size 2 and 3 over gloo.

The local attention is the CPU oracle standing in for the GPU kernel (the
kernel itself is covered by the gpu-marked tests); what is checked here is
the partition, the K/V broadcast and the output gather.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gfx906_b200 import shard
from gfx906_b200.configs import make_qkv


def oracle_attn(q, k, v, scale):
    from oracle.sdpa_math import sdpa_math_fp32

    return sdpa_math_fp32(q, k, v, scale).to(q.dtype)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_split_even_covers_everything_once():
    for n in (0, 1, 7, 256, 1000, 4096, 131072):
        for world in (1, 2, 3, 4, 8):
            for align in (1, 256):
                parts = [shard.split_even(n, world, r, align) for r in range(world)]
                assert parts[0].start == 0 and parts[-1].stop == n
                for a, b in zip(parts, parts[1:]):
                    assert a.stop == b.start
                for p in parts[:-1]:
                    assert p.size % align == 0
    assert shard.row_shard(131072, 3, 8) == shard.Shard(49152, 65536)
    assert shard.head_shard(1, 24, 7, 8) == shard.Shard(21, 24)
    with pytest.raises(ValueError):
        shard.split_even(10, 2, 2)


def _worker(rank, world, port, mode, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        if mode == "pipelined":
            _pipelined(rank, world, result_q)
            return
        if mode == "copy_engine":
            _copy_engine(rank, world, result_q)
            return
        B, H, Sq, Skv, D = {"heads": (2, 3, 300, 257, 64), "rows": (1, 1, 1100, 700, 64),
                            "rows_eq": (1, 1, 256 * world * 2, 700, 64), "rows_bh": (2, 3, 512 * world, 300, 32),
                            "auto": (1, 2, 800, 300, 32)}[mode]
        q, k, v = make_qkv(B, H, Sq, Skv, D, seed=7)
        scale = D ** -0.5
        if mode == "heads":
            out = shard.attention_by_heads(q, k, v, scale, local_attn=oracle_attn)
        elif mode == "auto":  # 2 units: heads on 2 ranks, query rows on 3
            out = shard.attention_sharded(q, k, v, scale, local_attn=oracle_attn)
        else:
            sh = shard.row_shard(Sq, rank, world)
            q_rows = q[:, :, sh.start:sh.stop].contiguous()
            if rank != 0:  # only rank 0 holds K/V; the others receive them
                k, v = torch.zeros_like(k), torch.zeros_like(v)
            # equal shards gather straight into a preallocated output
            dst = torch.full_like(q, float("nan")) if mode != "rows" else None
            out = shard.attention_by_rows(q_rows, k, v, scale, Sq, src=0, local_attn=oracle_attn, out=dst)
            if dst is not None:
                assert out is dst
        if rank == 0:
            q, k, v = make_qkv(B, H, Sq, Skv, D, seed=7)
            ref = oracle_attn(q, k, v, scale)
            result_q.put(float((out.float() - ref.float()).abs().max()))
    finally:
        dist.destroy_process_group()


class _FakeKV:
    """Stand-in for peer.KVBroadcast on CPU: the same call protocol (source,
    start, wait, release, running call indices), the transfer a gloo
    broadcast inside start()."""

    def __init__(self, shape, src=0, depth=2):
        self.is_source = dist.get_rank() == src
        self.src, self.depth, self.calls = src, depth, 0
        self.k = [torch.zeros(shape, dtype=torch.float16) for _ in range(depth)]
        self.v = [torch.zeros(shape, dtype=torch.float16) for _ in range(depth)]
        self.log = []

    def source(self, i):
        self.log.append(("source", i))
        return self.k[i % self.depth], self.v[i % self.depth]

    def start(self, i):
        self.log.append(("start", i))
        dist.broadcast(self.k[i % self.depth], src=self.src)
        dist.broadcast(self.v[i % self.depth], src=self.src)

    def wait(self, i):
        self.log.append(("wait", i))
        return self.k[i % self.depth], self.v[i % self.depth]

    def release(self, i):
        self.log.append(("release", i))


def _copy_engine(rank, world, result_q):
    """attention_by_rows_copy_engine over a fake broadcaster, used twice: the
    outputs equal the unsharded results, call i + 1 is started before call
    i's kernel, and call indices run on across uses."""
    Sq, Skv, D = 256 * world * 2, 300, 64
    scale = D ** -0.5
    inputs = [make_qkv(1, 1, Sq, Skv, D, seed=40 + i) for i in range(3)]
    sh = shard.row_shard(Sq, rank, world)
    bc = _FakeKV((1, 1, Skv, D))

    def fill(i, k, v):
        k.copy_(inputs[i][1])
        v.copy_(inputs[i][2])

    err = 0.0
    for use in range(2):
        outs = [torch.full((1, 1, Sq, D), float("nan"), dtype=torch.float16) for _ in range(3)]
        shard.attention_by_rows_copy_engine([x[0][:, :, sh.start:sh.stop].contiguous() for x in inputs], bc, scale,
                                            Sq, outs, fill=fill, local_attn=oracle_attn)
        for (q, k, v), out in zip(inputs, outs):
            err = max(err, float((out.float() - oracle_attn(q, k, v, scale).float()).abs().max()))
    starts = [i for op, i in bc.log if op == "start"]
    assert starts == list(range(6)), starts
    # within a use, the next call's transfer is enqueued before this call's
    # kernel is released
    for i in (0, 1, 3, 4):
        assert bc.log.index(("start", i + 1)) < bc.log.index(("release", i))
    if rank == 0:
        result_q.put(err)


def _pipelined(rank, world, result_q):
    """Three calls through attention_by_rows_pipelined (the next call's K/V
    broadcast while this one computes, each output gathered asynchronously):
    every output must equal the unsharded result of its own inputs."""
    Sq, Skv, D = 256 * world * 2, 300, 64
    scale = D ** -0.5
    inputs = [make_qkv(1, 1, Sq, Skv, D, seed=20 + i) for i in range(3)]
    sh = shard.row_shard(Sq, rank, world)
    # receive buffers alternate between two sets on the ranks that receive
    kbuf = [torch.zeros(1, 1, Skv, D, dtype=torch.float16) for _ in range(2)]
    vbuf = [torch.zeros(1, 1, Skv, D, dtype=torch.float16) for _ in range(2)]
    outs = [torch.full((1, 1, Sq, D), float("nan"), dtype=torch.float16) for _ in range(3)]
    calls = []
    for i in range(3):
        q, k, v = inputs[i]
        if rank != 0:
            k, v = kbuf[i % 2], vbuf[i % 2]
        calls.append((q[:, :, sh.start:sh.stop].contiguous(), k, v, scale, outs[i]))
    got = shard.attention_by_rows_pipelined(calls, Sq, src=0, local_attn=oracle_attn)
    assert all(a is b for a, b in zip(got, outs))
    if rank == 0:
        err = 0.0
        for i in range(3):
            q, k, v = inputs[i]
            err = max(err, float((outs[i].float() - oracle_attn(q, k, v, scale).float()).abs().max()))
        result_q.put(err)


@pytest.mark.parametrize("mode,world", [("heads", 2), ("rows", 2), ("rows", 3), ("heads", 3), ("auto", 2),
                                        ("auto", 3), ("rows_eq", 2), ("rows_eq", 3), ("rows_bh", 2),
                                        ("pipelined", 2), ("pipelined", 3), ("copy_engine", 2),
                                        ("copy_engine", 3)])
def test_sharded_attention_matches_unsharded(mode, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_worker, args=(world, free_port(), mode, q), nprocs=world, start_method="spawn",
                       join=True)
    assert q.get(timeout=60) == 0.0  # same local computation per row / head: identical bits


def test_single_process_needs_no_process_group():
    q, k, v = make_qkv(1, 2, 300, 200, 64, seed=8)
    ref = oracle_attn(q, k, v, 0.125)
    assert torch.equal(shard.attention_by_heads(q, k, v, 0.125, local_attn=oracle_attn), ref)
    assert torch.equal(shard.attention_by_rows(q, k, v, 0.125, 300, local_attn=oracle_attn), ref)


def test_choose_partition():
    assert shard.choose_partition(1, 4, 8) == "rows"   # C4 on 8 GPUs
    assert shard.choose_partition(1, 24, 8) == "heads"  # C2 on 8 GPUs
    assert shard.choose_partition(1, 1, 1) == "heads"
    q, k, v = make_qkv(1, 2, 300, 200, 64, seed=8)
    ref = oracle_attn(q, k, v, 0.125)
    assert torch.equal(shard.attention_sharded(q, k, v, 0.125, partition="rows", local_attn=oracle_attn), ref)
    with pytest.raises(ValueError):
        shard.attention_sharded(q, k, v, 0.125, partition="cols", local_attn=oracle_attn)
