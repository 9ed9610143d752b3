"""Tensor-parallel SwiGLU FFN: sharding + all-reduce on 2 CPU ranks (gloo),
checked against the unsharded FFN computed with the oracle."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import gguf_oracle as O

H, I, M = 512, 1024, 3


def _oracle_matmul(x: torch.Tensor, w, out_dtype=torch.float32):
    """CPU stand-in for ops.mul_mat (test only): x @ dequant(W)^T via the oracle."""
    y = O.matmul_ref(x.float().numpy(), w.data.numpy(), w.qtype, w.n, w.k)
    return torch.from_numpy(y).to(out_dtype)


def _weights():
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    g = GGUFQuantTensor(torch.from_numpy(O.make_weights(I, H, O.Q4_K, seed=1)), O.Q4_K, (I, H))
    u = GGUFQuantTensor(torch.from_numpy(O.make_weights(I, H, O.Q4_K, seed=2)), O.Q4_K, (I, H))
    d = GGUFQuantTensor(torch.from_numpy(O.make_weights(H, I, O.Q4_K, seed=3)), O.Q4_K, (H, I))
    return g, u, d


def _reference(x):
    g, u, d = _weights()
    gg = _oracle_matmul(x, g)
    uu = _oracle_matmul(x, u)
    a = torch.nn.functional.silu(gg) * uu
    return _oracle_matmul(a, d)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, x, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from vllm_webgpu_b200.tp import TensorParallelSwiGLU
        g, u, d = _weights()
        ffn = TensorParallelSwiGLU(g, u, d, rank=rank, world=world, matmul=_oracle_matmul)
        y = ffn(x)
        # the residual rides on rank 0's partial only: the sum carries it once
        res = torch.from_numpy(O.make_activations(M, H, seed=9))
        yr = ffn(x, residual=res)
        q.put((rank, (y.numpy(), yr.numpy())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_ffn_matches_unsharded(world):
    x = torch.from_numpy(O.make_activations(M, H, seed=5))
    ref = _reference(x).numpy()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, x, q)) for r in range(world)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res = O.make_activations(M, H, seed=9)
    for r in range(world):
        assert O.rel_err(outs[r][0], ref) < 1e-5
        assert O.rel_err(outs[r][1], ref + res) < 1e-5


def test_shard_ranges_and_errors():
    from vllm_webgpu_b200.tp import shard_ffn, shard_range
    assert shard_range(28672, 7, 8, 256) == (25088, 28672)
    with pytest.raises(ValueError):
        shard_range(1000, 0, 3, 1)
    with pytest.raises(ValueError):
        shard_range(1024, 0, 8, 256)  # 128-weight shards split a Q4_K superblock
    g, u, d = _weights()
    gl, ul, dl = shard_ffn(g, u, d, 1, 2)
    assert gl.shape == (I // 2, H) and dl.shape == (H, I // 2)
    full = O.dequantize(d.data.numpy(), O.Q4_K, H, I)
    assert np.array_equal(O.dequantize(dl.data.numpy(), O.Q4_K, H, I // 2), full[:, I // 2:])


# ---- the layer's seven projections split over ranks (TensorParallelLayerLinears) ----
LH, LI, LKV = 1024, 2048, 256  # hidden, intermediate, k/v width of a small Llama-like layer (splits stay
# superblock-aligned up to 4 ranks)


def _layer_weights():
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    shapes = {"q": (LH, LH), "k": (LKV, LH), "v": (LKV, LH), "o": (LH, LH), "gate": (LI, LH), "up": (LI, LH),
              "down": (LH, LI)}
    return {p: GGUFQuantTensor(torch.from_numpy(O.make_weights(n, k, O.Q4_K, seed=20 + i)), O.Q4_K, (n, k))
            for i, (p, (n, k)) in enumerate(shapes.items())}


def _layer_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from vllm_webgpu_b200.tp import TensorParallelLayerLinears
        ws = _layer_weights()
        tpl = TensorParallelLayerLinears(ws, rank=rank, world=world, matmul=_oracle_matmul)
        xs = {nm: torch.from_numpy(O.make_activations(2, k, seed=30 + j))
              for j, (nm, k) in enumerate((("normed", LH), ("attn", LH), ("ffn", LH), ("act", LI)))}
        h0, h1 = rank * LH // world, (rank + 1) * LH // world
        i0, i1 = rank * LI // world, (rank + 1) * LI // world
        bufs = {p: torch.empty((2, tpl.w[p].n), dtype=torch.float32) for p in ("q", "k", "v", "gate", "up")}
        bufs["o"] = torch.empty((2, LH), dtype=torch.float32)
        bufs["down"] = torch.empty((2, LH), dtype=torch.float32)
        tpl(xs["normed"], xs["attn"][:, h0:h1], xs["ffn"], xs["act"][:, i0:i1], bufs)
        q.put((rank, {p: b.numpy() for p, b in bufs.items()}))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_layer_linears_gloo(world):
    import queue
    import time as _t
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_layer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    got = {}
    deadline = _t.monotonic() + 240
    while len(got) < world:
        try:
            r, v = q.get(timeout=5)
            got[r] = v
        except queue.Empty:
            if any(p.exitcode not in (None, 0) for p in ps) or _t.monotonic() > deadline:
                for p in ps:
                    p.kill()
                pytest.fail(f"a rank failed: exit codes {[p.exitcode for p in ps]}")
    for p in ps:
        p.join(60)
    ws = _layer_weights()
    xs = {nm: O.make_activations(2, k, seed=30 + j)
          for j, (nm, k) in enumerate((("normed", LH), ("attn", LH), ("ffn", LH), ("act", LI)))}
    src = {"q": "normed", "k": "normed", "v": "normed", "o": "attn", "gate": "ffn", "up": "ffn", "down": "act"}
    for p, w in ws.items():
        ref = O.matmul_ref(xs[src[p]], w.data.numpy(), w.qtype, w.n, w.k)
        if p in ("o", "down"):  # all-reduced: every rank holds the full sum
            for r in range(world):
                assert O.rel_err(got[r][p], ref) <= 1e-5, (p, r)
        else:  # output-row slices, concatenated in rank order
            full = np.concatenate([got[r][p] for r in range(world)], axis=1)
            assert O.rel_err(full, ref) <= 1e-5, p
