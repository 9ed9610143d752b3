"""Host <-> device staging by a kernel (ggufmm_stage_copy): byte-exact copies from and
to pinned host memory, ragged sizes, refusal of pageable memory, and the serving
graph's staged replay with the kernel copies against the copy-engine ones."""
from __future__ import annotations

import os

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nbytes", [16, 4096 + 16, 53248, 172032 + 48, 1 << 20])
def test_stage_copy_round_trip_exact(cuda, nbytes):
    from vllm_webgpu_b200 import ops
    g = torch.Generator().manual_seed(nbytes)
    host_in = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, generator=g).pin_memory()
    dev = torch.empty(nbytes, dtype=torch.uint8, device=cuda)
    host_out = torch.zeros(nbytes, dtype=torch.uint8).pin_memory()
    ops.stage_copy(dev, host_in)
    ops.stage_copy(host_out, dev)
    torch.cuda.synchronize()
    assert torch.equal(dev.cpu(), host_in)
    assert torch.equal(host_out, host_in)


def test_stage_copy_tail_bytes(cuda):
    """Sizes that are not a multiple of 16 bytes: the tail is copied, nothing past it."""
    from vllm_webgpu_b200 import _lib
    n = 1000 + 7
    src = torch.arange(n + 64, dtype=torch.int64).to(torch.uint8).pin_memory()
    dst = torch.full((n + 64,), 0xAB, dtype=torch.uint8, device=cuda)
    st = _lib.lib().ggufmm_stage_copy(dst.data_ptr(), src.data_ptr(), n, torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "ggufmm_stage_copy")
    got = dst.cpu()
    assert torch.equal(got[:n], src[:n])
    assert bool((got[n:] == 0xAB).all())


def test_stage_copy_refuses_pageable_and_misaligned(cuda):
    from vllm_webgpu_b200 import _lib, ops
    pageable = torch.zeros(4096, dtype=torch.uint8)
    dev = torch.empty(4096, dtype=torch.uint8, device=cuda)
    with pytest.raises(ValueError):
        ops.stage_copy(dev, pageable)
    lib = _lib.lib()
    pinned = torch.zeros(4096 + 16, dtype=torch.uint8).pin_memory()
    s = torch.cuda.current_stream().cuda_stream
    assert lib.ggufmm_stage_copy(dev.data_ptr(), pageable.data_ptr(), 4096, s) == _lib.ERR_ARG
    assert lib.ggufmm_stage_copy(dev.data_ptr(), pinned.data_ptr() + 8, 4096, s) == _lib.ERR_ALIGN
    torch.cuda.synchronize()


def test_stage_copy_in_graph_chained_with_kernels(cuda):
    """Captured in a CUDA graph between kernels: each replay moves the refilled host
    input in and the result out."""
    from vllm_webgpu_b200 import ops
    n = 8192
    hin = torch.zeros(n, dtype=torch.float32).pin_memory()
    hout = torch.zeros(n, dtype=torch.float32).pin_memory()
    din = torch.empty(n, dtype=torch.float32, device=cuda)
    dout = torch.empty(n, dtype=torch.float32, device=cuda)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ops.stage_copy(din, hin)
        torch.mul(din, 3.0, out=dout)
        ops.stage_copy(hout, dout)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        ops.stage_copy(din, hin)
        torch.mul(din, 3.0, out=dout)
        ops.stage_copy(hout, dout)
    for step in range(3):
        hin.copy_(torch.arange(n, dtype=torch.float32) + step)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(hout, 3.0 * hin)


def test_layer_graph_staged_by_kernel_matches_memcpy(cuda, monkeypatch):
    """The serving path's staged replay gives the same outputs with kernel staging
    and with copy-engine memcpy nodes."""
    from oracle import gguf_oracle as O
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    from vllm_webgpu_b200.models.llama import PROJ, LlamaB200Model
    h, it, kv = 512, 1792, 128
    shapes = {"q": (h, h), "k": (kv, h), "v": (kv, h), "o": (h, h), "gate": (it, h), "up": (it, h), "down": (h, it)}
    model = LlamaB200Model(None, device=cuda)
    for i, (p, (n, k)) in enumerate(shapes.items()):
        raw = O.make_weights(n, k, O.Q4_K, seed=70 + i)
        model.weights[f"model.layers.0.{PROJ[p]}"] = GGUFQuantTensor(torch.from_numpy(raw).cuda(), O.Q4_K, (n, k))
    ins = {"normed": h, "attn_out": h, "ffn_normed": h, "ffn_act": it}
    outs = {"q": h, "k": kv, "v": kv, "o": h, "gate": it, "up": it, "down": h}
    results = []
    for mode in ("1", "0"):
        monkeypatch.setenv("GGUFMM_STAGE_KERNEL", mode)
        hin = {nm: torch.randn((1, kk)).to(torch.bfloat16).pin_memory() for nm, kk in ins.items()}
        if results:
            for nm in hin:
                hin[nm].copy_(results[0][1][nm])
        din = {nm: torch.empty_like(t, device=cuda) for nm, t in hin.items()}
        bufs = {p: torch.empty((1, n), dtype=torch.float32, device=cuda) for p, n in outs.items()}
        hout = {p: torch.zeros((1, n), dtype=torch.float32).pin_memory() for p, n in outs.items()}
        model.layer_linears_graph(0, din["normed"], din["attn_out"], din["ffn_normed"], din["ffn_act"], bufs,
                                  stage_in=[(din[nm], hin[nm]) for nm in ins],
                                  stage_out=[(hout[p], bufs[p]) for p in outs])
        torch.cuda.synchronize()
        results.append(({p: hout[p].clone() for p in outs}, {nm: hin[nm].clone() for nm in ins}))
    for p in outs:
        assert torch.equal(results[0][0][p], results[1][0][p]), p
    assert os.environ.get("GGUFMM_STAGE_KERNEL") == "0"
