"""Data-parallel host logic on CPU: two gloo ranks average a gradient buffer and
take the max of their step times, as bench.py does over NCCL."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from atlas_b200 import dp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    r, w = dp.init("gloo")
    buf = torch.full((1000,), float(r + 1))
    dp.allreduce_mean_(buf)
    t = dp.max_over_ranks(10.0 * (r + 1))
    q.put((r, float(buf[0]), float(buf[-1]), t))
    torch.distributed.destroy_process_group()


def test_gloo_two_ranks_mean_and_max():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(60)
    assert [x[1] for x in res] == [1.5, 1.5] and [x[3] for x in res] == [20.0, 20.0]


def test_param_count_170m_and_59m():
    # exact counts of the reference LM at the BASELINE configs (model.py:271-305)
    assert dp.atlas_param_count() == 140685912
    assert dp.atlas_param_count(n_layer=8, n_embd=512, n_head=8) == 61042960
