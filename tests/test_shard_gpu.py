"""Sharded attention over NCCL on 2+ GPUs of one box (skipped with fewer GPUs).

Each rank runs the sm_100a kernel on its shard; the gathered result must equal
a single-GPU call on the full problem (same kernel, same rows: identical bits
for the row layout, whose per-row work does not depend on the shard).
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    import datetime

    import gfx906_b200
    from gfx906_b200 import shard
    from gfx906_b200.configs import make_qkv

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        errs = []
        # rows: one head, long sequence, K/V only on rank 0
        Sq, Skv, D = 4096 + 300, 8192, 64
        q, k, v = make_qkv(1, 1, Sq, Skv, D, seed=3)
        sh = shard.row_shard(Sq, rank, world)
        q_rows = q[:, :, sh.start:sh.stop].contiguous().cuda()
        kd, vd = (k.cuda(), v.cuda()) if rank == 0 else (torch.zeros_like(k).cuda(), torch.zeros_like(v).cuda())
        out = shard.attention_by_rows(q_rows, kd, vd, D ** -0.5, Sq, src=0)
        full = gfx906_b200.attn(q.cuda(), k.cuda(), v.cuda(), D ** -0.5)
        errs.append(float((out.float() - full.float()).abs().max()))
        # heads: (batch x head) blocks
        q, k, v = make_qkv(2, 5, 1000, 777, 128, seed=4)
        out = shard.attention_by_heads(q.cuda(), k.cuda(), v.cuda(), 128 ** -0.5)
        full = gfx906_b200.attn(q.cuda(), k.cuda(), v.cuda(), 128 ** -0.5)
        errs.append(float((out.float() - full.float()).abs().max()))
        # auto: 2 heads of D=512 on `world` ranks -> query-row blocks when world > 2
        q, k, v = make_qkv(1, 2, 1024, 640, 512, seed=5)
        out = shard.attention_sharded(q.cuda(), k.cuda(), v.cuda(), 512 ** -0.5)
        full = gfx906_b200.attn(q.cuda(), k.cuda(), v.cuda(), 512 ** -0.5)
        errs.append(float((out.float() - full.float()).abs().max()))
        # pipelined: 3 calls, K/V of the next broadcast and O gathered beside
        # the kernel, which leaves 16 SMs to NCCL (a different split, so the
        # tolerance, not identical bits)
        Sq, Skv, D = 2048 * world, 4096, 64
        ins = [make_qkv(1, 1, Sq, Skv, D, seed=30 + i) for i in range(3)]
        sh = shard.row_shard(Sq, rank, world)
        kb = [torch.zeros(1, 1, Skv, D, dtype=torch.float16, device="cuda") for _ in range(2)]
        vb = [torch.zeros(1, 1, Skv, D, dtype=torch.float16, device="cuda") for _ in range(2)]
        calls = []
        for i, (q, k, v) in enumerate(ins):
            if rank == 0:
                kd, vd = k.cuda(), v.cuda()
            else:
                kd, vd = kb[i % 2], vb[i % 2]
            out = torch.full((1, 1, Sq, D), float("nan"), dtype=torch.float16, device="cuda")
            calls.append((q[:, :, sh.start:sh.stop].contiguous().cuda(), kd, vd, D ** -0.5, out))
        outs = shard.attention_by_rows_pipelined(calls, Sq, src=0, reserve_sms=16)
        for (q, k, v), out in zip(ins, outs):
            full = gfx906_b200.attn(q.cuda(), k.cuda(), v.cuda(), D ** -0.5)
            errs.append(float((out.float() - full.float()).abs().max()))
        # copy engines: the same 3 calls, K/V pulled from rank 0's ring over
        # CUDA IPC while the previous kernel runs (fill writes each call's
        # K/V into the ring on rank 0); the kernel keeps every SM
        from gfx906_b200.peer import KVBroadcast

        bc = KVBroadcast((1, 1, Skv, D), src=0)
        dev_kv = [(k.cuda(), v.cuda()) for (_, k, v) in ins] if rank == 0 else None

        def fill(i, kk, vv):
            kk.copy_(dev_kv[i][0])
            vv.copy_(dev_kv[i][1])

        outs = [torch.full((1, 1, Sq, D), float("nan"), dtype=torch.float16, device="cuda") for _ in ins]
        shard.attention_by_rows_copy_engine([c[0] for c in calls], bc, D ** -0.5, Sq, outs, fill=fill)
        for (q, k, v), out in zip(ins, outs):
            full = gfx906_b200.attn(q.cuda(), k.cuda(), v.cuda(), D ** -0.5)
            errs.append(float((out.float() - full.float()).abs().max()))
        # and with the output rows pushed to every rank on the copy engines too
        from gfx906_b200.peer import RowGather

        rows = [(shard.row_shard(Sq, r, world).start, shard.row_shard(Sq, r, world).stop) for r in range(world)]
        rg = RowGather((1, 1, Sq, D), rows)
        got = {}
        shard.attention_by_rows_copy_engine([c[0] for c in calls], bc, D ** -0.5, Sq, fill=fill, rg=rg,
                                            consume=lambda i, o: got.__setitem__(i, o.clone()))
        last = shard.attention_by_rows_copy_engine([c[0] for c in calls], bc, D ** -0.5, Sq, fill=fill, rg=rg)
        for i, (q, k, v) in enumerate(ins):
            full = gfx906_b200.attn(q.cuda(), k.cuda(), v.cuda(), D ** -0.5)
            errs.append(float((got[i].float() - full.float()).abs().max()))
            if i == len(ins) - 1:
                errs.append(float((last.float() - full.float()).abs().max()))
        rg.close()
        bc.close()
        # a chain of pulls (each rank pulls from the previous one; a tree of
        # fanout 1): on 3+ ranks the non-source parents are exercised
        bc = KVBroadcast((1, 1, Skv, D), src=0, fanout=1)
        outs = [torch.full((1, 1, Sq, D), float("nan"), dtype=torch.float16, device="cuda") for _ in ins]
        for _ in range(2):  # call indices run on across uses
            shard.attention_by_rows_copy_engine([c[0] for c in calls], bc, D ** -0.5, Sq, outs, fill=fill)
        for (q, k, v), out in zip(ins, outs):
            full = gfx906_b200.attn(q.cuda(), k.cuda(), v.cuda(), D ** -0.5)
            errs.append(float((out.float() - full.float()).abs().max()))
        bc.close()
        torch.cuda.synchronize()
        if rank == 0:
            result_q.put(errs)
    finally:
        dist.destroy_process_group()


def test_sharded_attention_nccl():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 or more GPUs")
    world = min(n, 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_worker, args=(world, _free_port(), q), nprocs=world, start_method="spawn", join=True)
    errs = q.get(timeout=120)
    assert all(e <= 2e-3 for e in errs) and len(errs) == 16, errs
