"""Batch sharding over GPUs: the host logic on CPU (world-size-2 gloo ranks)
and the native multi-GPU runner on the GPU.

The CPU ranks stand in for GPUs: each rank takes its slice of one seeded
global batch by the library's shard plan, runs it through the numpy oracle
(test infrastructure standing in for a GPU's forward), and the slices are
gathered in rank order; the result must equal the unsharded run.
"""

import os
import socket

import numpy as np
import pytest

from conftest import TOL, rel_err
from nert_b200 import configs
from oracle import np_ref


def test_shard_plan_contiguous_and_ragged():
    from nert_b200.sharding import shard_plan

    assert shard_plan(256, 8) == [(32 * i, 32) for i in range(8)]
    assert shard_plan(5, 2) == [(0, 3), (3, 2)]
    assert shard_plan(3, 4) == [(0, 1), (1, 1), (2, 1), (3, 0)]
    for batch in (0, 1, 7, 64, 255):
        for n in (1, 2, 3, 8):
            plan = shard_plan(batch, n)
            assert sum(c for _, c in plan) == batch
            assert all(plan[i][0] + plan[i][1] == plan[i + 1][0] for i in range(n - 1))
            assert max(c for _, c in plan) - min(c for _, c in plan) <= 1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, batch, q, leave_after):
    """One CPU rank: its slice of the seeded batch through the oracle, then an
    all-gather of the slices in rank order."""
    import datetime

    import torch.distributed as dist

    from nert_b200.sharding import gather_rows, rank_slice

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        g = configs.resnet18(1)
        x = configs.resnet_input(batch)
        sl = rank_slice(batch, rank, world)
        outs = []
        for step in range(2):
            if leave_after is not None and rank == 1 and step == leave_after:
                return  # leaves between steps, with nothing in flight
            local = np.concatenate([np_ref.run(g, {"input": x[i:i + 1]})["fc_out"] for i in range(sl.start, sl.stop)]
                                   or [np.zeros((0, 1000), np.float32)])
            outs.append(gather_rows(local, batch, dist))
        if rank == 0:
            q.put(("ok", outs[-1]))
    except Exception as e:  # reported to the parent, which asserts on it
        if rank == 0:
            q.put(("error", repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _spawn(batch, leave_after=None):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, batch, q, leave_after)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        kind, val = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return kind, val


def test_two_rank_gather_equals_unsharded():
    batch = 3  # ragged: rank 0 takes two images, rank 1 one
    kind, got = _spawn(batch)
    assert kind == "ok", got
    g = configs.resnet18(batch)
    want = np_ref.run(g, {"input": configs.resnet_input(batch)})["fc_out"]
    np.testing.assert_array_equal(got, want)


def test_rank_leaving_between_steps_fails_the_next_collective():
    """Rank 1 leaves after one step; rank 0's next gather ends with an error
    within the process group's timeout instead of waiting for good."""
    kind, msg = _spawn(2, leave_after=1)
    assert kind == "error", msg


@pytest.mark.gpu
def test_sharded_runner_matches_oracle(cuda):
    """The native runner: a ragged split (3 + 2 images) of ResNet-18 over two
    shards (two GPUs when present, else both on GPU 0), each on its own host
    thread, equals the oracle on every image, on two runs in a row."""
    import torch

    from nert_b200.sharding import ShardedModel

    devices = [0, 1] if torch.cuda.device_count() > 1 else [0, 0]
    batch = 5
    g = configs.resnet18(batch)
    x = configs.resnet_input(batch)
    want = np_ref.run(g, {"input": x})["fc_out"]
    m = ShardedModel(configs.resnet18(1), {"input": list(x.shape)}, devices)
    try:
        assert [(s["offset"], s["count"]) for s in m.shards] == [(0, 3), (3, 2)]
        assert m.outputs[0]["shape"] == (batch, 1000)
        first = m.run({"input": x})["fc_out"]
        again = m.run({"input": x})["fc_out"]
    finally:
        m.close()
    np.testing.assert_array_equal(first, again)
    assert rel_err(first, want) <= TOL
