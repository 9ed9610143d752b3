"""Failure detection between ranks, on CPU (gloo), made on the host: a rank that
never joins, and a rank that leaves between steps. The others must learn of it
through an error within a bounded time, never hang."""
from __future__ import annotations

import os
import socket
import time
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _lonely_rank(port, q):
    import torch.distributed as dist
    t0 = time.monotonic()
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=2,
                                timeout=timedelta(seconds=3))
        q.put(("joined", time.monotonic() - t0))
    except Exception as e:  # noqa: BLE001 - any error is the expected outcome
        q.put(("error", time.monotonic() - t0, type(e).__name__))


def test_init_times_out_when_a_rank_never_joins():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(_free_port(), q))
    p.start()
    p.join(120)
    if p.is_alive():
        p.kill()
        pytest.fail("process-group init hung with a missing rank")
    res = q.get(timeout=5)
    assert res[0] == "error", res
    assert res[1] < 60, res


def _ffn_rank(rank, world, port, q):
    import torch.distributed as dist
    from tests.test_tp_gloo import _oracle_matmul, _weights, M, H
    from oracle import gguf_oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    from vllm_webgpu_b200.tp import TensorParallelSwiGLU
    g, u, d = _weights()
    ffn = TensorParallelSwiGLU(g, u, d, rank=rank, world=world, matmul=_oracle_matmul)
    x = torch.from_numpy(O.make_activations(M, H, seed=3))
    ffn(x)  # step 1: everyone present
    if rank == 1:
        q.put((1, "left"))
        q.close()
        q.join_thread()  # the message is flushed before the abrupt exit
        os._exit(0)  # leaves between steps, with no collective in flight
    t0 = time.monotonic()
    try:
        ffn(x)  # step 2: the peer is gone
        q.put((0, "completed", time.monotonic() - t0))
    except Exception as e:  # noqa: BLE001
        q.put((0, "error", time.monotonic() - t0, type(e).__name__))


def test_collective_errors_when_a_rank_leaves_between_steps():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_ffn_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(180)
    for p in ps:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung after its peer left")
    res = {}
    while not q.empty():
        r = q.get()
        res[r[0]] = r
    assert res[1][1] == "left"
    assert res[0][1] == "error", res[0]
    assert res[0][2] < 60, res[0]
