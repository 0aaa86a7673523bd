"""The host-side call counters of the copy-engine transport (gfx906_b200.peer.Board)
on CPU: gloo ranks on one node, shared memory between them.

Checked: a wait returns only once every listed rank has published the call
(ranks publish in turn, each waiting on the previous one's index, so any
missed ordering would deadlock into the time limit); counters are per
channel; a wait for an index nobody publishes ends in TimeoutError within
its limit; the segment's name is gone once every rank has mapped it.
"""

import os
import time

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.test_shard import free_port


def _worker(rank, world, port, result_q):
    from gfx906_b200.peer import Board

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        board = Board(2, timeout_s=5.0)
        assert board.arr.shape == (2, world)
        dist.barrier()  # rank 0 unlinks the name right after the constructor's barrier
        assert not os.path.exists("/dev/shm/" + board._shm.name.lstrip("/"))
        # a relay: call i is published by rank i % world after it has seen
        # call i - 1 from the previous rank, on channel 0; channel 1 echoes
        for i in range(40):
            owner = i % world
            if rank == owner:
                if i > 0:
                    board.wait(0, [(owner - 1) % world], i - 1)
                board.publish(0, i)
                board.publish(1, i)
        board.wait(0, list(range(world)), 40 - world)  # everybody's last call
        assert all(board.arr[1, r] == board.arr[0, r] for r in range(world))
        dist.barrier()
        t0 = time.monotonic()
        board.timeout_s = 0.3
        with pytest.raises(TimeoutError):
            board.wait(1, [(rank + 1) % world], 10_000)
        waited = time.monotonic() - t0
        assert 0.25 < waited < 5.0, waited
        dist.barrier()
        board.close()
        if rank == 0:
            result_q.put("ok")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_board_orders_calls_across_processes(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_worker, args=(world, free_port(), q), nprocs=world, start_method="spawn", join=True)
    assert q.get(timeout=60) == "ok"
