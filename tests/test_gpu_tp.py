"""Tensor-parallel Q4_K SwiGLU FFN on the GPU (BASELINE config 5 shapes scaled
down): world 1 against the oracle FFN, and, when 2+ GPUs are visible, 2 NCCL
ranks (one process per GPU) against the same oracle."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O
from tests.helpers import TOL

pytestmark = pytest.mark.gpu
H, I = 1024, 2048
# The FFN chains three quantized matmuls through SwiGLU: each matmul meets the
# 2e-3 gate on its own (test_gpu_gemv / test_gpu_gemm); above M = 8 the chain runs
# on the fp16-operand GEMM and the errors of the three add up, so the composite
# output is held to 1.5x the single-matmul gate.
FFN_TOL = 1.5 * TOL
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _weights():
    return (O.make_weights(I, H, O.Q4_K, seed=1), O.make_weights(I, H, O.Q4_K, seed=2),
            O.make_weights(H, I, O.Q4_K, seed=3))


def _oracle_ffn(x: np.ndarray) -> np.ndarray:
    g, u, d = _weights()
    gg = O.matmul_ref(x, g, O.Q4_K, I, H)
    uu = O.matmul_ref(x, u, O.Q4_K, I, H)
    a = (gg / (1.0 + np.exp(-gg))) * uu
    return O.matmul_ref(a.astype(np.float32), d, O.Q4_K, H, I)


def _ffn(rank, world, group=None):
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    from vllm_webgpu_b200.tp import TensorParallelSwiGLU
    g, u, d = _weights()
    dev = torch.device("cuda", torch.cuda.current_device())
    t = lambda raw, n, k: GGUFQuantTensor(torch.from_numpy(raw).to(dev), O.Q4_K, (n, k))
    return TensorParallelSwiGLU(t(g, I, H), t(u, I, H), t(d, H, I), rank=rank, world=world, group=group)


@pytest.mark.parametrize("m", [1, 32])
def test_tp_ffn_world1(cuda, m):
    x = O.make_activations(m, H, seed=4)
    y = _ffn(0, 1)(torch.from_numpy(x).to(torch.bfloat16).cuda())
    torch.cuda.synchronize()
    xb = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert O.rel_err(y.cpu().numpy(), _oracle_ffn(xb)) <= FFN_TOL


WORKER = r"""
import os, sys, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, {root!r}); sys.path.insert(0, os.path.join({root!r}, "vllm-webgpu_b200"))
from tests.test_gpu_tp import _ffn, H
from oracle import gguf_oracle as O
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
x = O.make_activations(8, H, seed=4)
y = _ffn(rank, world)(torch.from_numpy(x).to(torch.bfloat16).cuda())
torch.cuda.synchronize()
if rank == 0:
    np.save(sys.argv[1], y.cpu().numpy())
dist.destroy_process_group()
"""


def test_tp_ffn_two_gpus_nccl(cuda, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "worker.py"
    script.write_text(WORKER.format(root=ROOT))
    out = tmp_path / "y.npy"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", GGUFMM_TP_FUSED="0")  # the NCCL all-reduce path
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr", "127.0.0.1", "--master-port", "29533", str(script), str(out)],
                       env=env, capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    x = O.make_activations(8, H, seed=4)
    xb = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert O.rel_err(np.load(out), _oracle_ffn(xb)) <= TOL


WORKER_FUSED = r"""
import os, sys, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, {root!r}); sys.path.insert(0, os.path.join({root!r}, "vllm-webgpu_b200"))
from tests.test_gpu_tp import _ffn, H
from oracle import gguf_oracle as O
from vllm_webgpu_b200 import _lib
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
ffn = _ffn(rank, world)
outs = []
for m, seed in ((1, 5), (8, 6), (1, 7)):  # three calls: both halves of the exchange buffers
    x = O.make_activations(m, H, seed=seed)
    y = ffn(torch.from_numpy(x).to(torch.bfloat16).cuda())
    torch.cuda.synchronize()
    outs.append(y.cpu().numpy())
assert ffn._exchange is not None, "the fused down-projection all-reduce did not run"
assert _lib.lib().ggufmm_device_status(1, None) == 0
np.savez(sys.argv[1] + f".{{rank}}.npz", *outs)
dist.destroy_process_group()
"""


def test_tp_ffn_two_gpus_fused_allreduce(cuda, tmp_path):
    """Decode TP FFN on 2 GPUs whose down projection and all-reduce are one kernel
    (partials exchanged through NVLink peer memory): both GPUs hold the same bits,
    equal to the oracle FFN within the matmul gate."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "worker_fused.py"
    script.write_text(WORKER_FUSED.format(root=ROOT))
    out = tmp_path / "y"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", GGUFMM_TP_FUSED="1")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr", "127.0.0.1", "--master-port", "29534", str(script), str(out)],
                       env=env, capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    y0, y1 = np.load(str(out) + ".0.npz"), np.load(str(out) + ".1.npz")
    for i, (m, seed) in enumerate(((1, 5), (8, 6), (1, 7))):
        a, b = y0[f"arr_{i}"], y1[f"arr_{i}"]
        assert np.array_equal(a, b)
        x = O.make_activations(m, H, seed=seed)
        xb = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
        assert O.rel_err(a, _oracle_ffn(xb)) <= TOL


def _peer_worker(rank, world, port, q):
    import os

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from vllm_webgpu_b200 import ops
        n = 4096
        ar = ops.PeerAllReduce(n, device=torch.device("cuda", rank))
        outs = []
        # eager calls, then the same call replayed from a CUDA graph (the generation
        # counter advances on the device)
        x = torch.empty(n, dtype=torch.float32, device="cuda")
        for it in range(3):
            x.copy_(torch.from_numpy(O.make_activations(1, n, seed=100 * it + rank)).reshape(n))
            outs.append(ar(x, out=torch.empty_like(x)).cpu().numpy())
        y = torch.empty_like(x)
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.graph(g, stream=s):
            ar(x, out=y)
        for it in range(3, 6):
            x.copy_(torch.from_numpy(O.make_activations(1, n, seed=100 * it + rank)).reshape(n))
            dist.barrier()
            g.replay()
            torch.cuda.synchronize()
            outs.append(y.cpu().numpy())
        from vllm_webgpu_b200 import _lib
        q.put((rank, outs, _lib.lib().ggufmm_device_status(1, None)))
    finally:
        dist.destroy_process_group()


def test_peer_allreduce_two_gpus_eager_and_graph(cuda):
    """ggufmm_allreduce on 2 GPUs: every rank receives the rank-ordered sum, bit-identical
    across ranks, eagerly and replayed from a CUDA graph."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict((r, (o, st)) for r, o, st in (q.get(timeout=240) for _ in range(2)))
    for p in ps:
        p.join(60)
    n = 4096
    for it in range(6):
        ref = sum(O.make_activations(1, n, seed=100 * it + r).reshape(n).astype(np.float32) for r in range(2))
        assert np.array_equal(res[0][0][it], res[1][0][it])
        assert np.allclose(res[0][0][it], ref, rtol=1e-6, atol=1e-6)
    assert res[0][1] == 0 and res[1][1] == 0


def _gather_worker(rank, world, port, q, dtype_name="float32"):
    import os

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from vllm_webgpu_b200 import _lib, ops
        from vllm_webgpu_b200.formats import GGUFQuantTensor
        m, n, k = (300, 2048, 1024) if dtype_name == "float32" else (1100, 2048, 1024)
        raw = O.make_weights(n, k, O.Q4_K, seed=77)
        w = GGUFQuantTensor(torch.from_numpy(raw).cuda(), O.Q4_K, (n, k))
        r0, r1 = rank * n // world, (rank + 1) * n // world
        g = ops.PeerGather(m, n, getattr(torch, dtype_name), device=torch.device("cuda", rank))
        outs = []
        for it in range(2):
            x = torch.from_numpy(O.make_activations(m, k, seed=5 + it)).to(torch.bfloat16).cuda()
            y = ops.gemm_allgather(x, w.rows(r0, r1), g)
            torch.cuda.synchronize()
            outs.append(y.float().cpu().numpy().copy())
        q.put((rank, outs, _lib.lib().ggufmm_device_status(1, None)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dtype_name", ["float32", "bfloat16"])
def test_gemm_allgather_two_gpus(cuda, dtype_name):
    """The N-split GEMM with the all-gather in its epilogue: each GPU computes half the
    output columns and stores them into both GPUs' outputs; after the device barrier
    both hold the full product (oracle, 2e-3; bf16 adds half an ulp of each value),
    bit-identical, twice in a row. bf16 at M = 1100: whole tiles go through the staged
    16-byte peer stores, the ragged last token tile through per-element stores."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_gather_worker, args=(r, 2, port, q, dtype_name)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict((r, (o, st)) for r, o, st in (q.get(timeout=240) for _ in range(2)))
    for p in ps:
        p.join(60)
    m, n, k = (300, 2048, 1024) if dtype_name == "float32" else (1100, 2048, 1024)
    raw = O.make_weights(n, k, O.Q4_K, seed=77)
    for it in range(2):
        x = torch.from_numpy(O.make_activations(m, k, seed=5 + it)).to(torch.bfloat16).float().numpy()
        ref = O.matmul_ref(x, raw, O.Q4_K, n, k)
        assert np.array_equal(res[0][0][it], res[1][0][it])
        if dtype_name == "float32":
            assert O.rel_err(res[0][0][it], ref) <= TOL
        else:
            rms = float(np.sqrt(np.mean(ref * ref)))
            assert bool(np.all(np.abs(res[0][0][it] - ref) <= TOL * rms + 2.0 ** -8 * np.abs(ref)))
    assert res[0][1] == 0 and res[1][1] == 0
