"""The Llama layer's projections through the model API (eager and graph-replayed)
against the oracle, on the GPU."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O
from tests.helpers import TOL

pytestmark = pytest.mark.gpu

# a scaled-down Llama layer: q/k/v/o over hidden 512, gate/up/down over intermediate 1792
SHAPES = {"q": (512, 512), "k": (128, 512), "v": (128, 512), "o": (512, 512), "gate": (1792, 512),
          "up": (1792, 512), "down": (512, 1792)}
INPUT = {"q": "normed", "k": "normed", "v": "normed", "o": "attn_out", "gate": "ffn_normed",
         "up": "ffn_normed", "down": "ffn_act"}


def _model(cuda):
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    from vllm_webgpu_b200.models.llama import PROJ, LlamaB200Model
    model = LlamaB200Model(None, device="cuda:0")
    raws = {}
    for i, (p, (n, k)) in enumerate(SHAPES.items()):
        raw = O.make_weights(n, k, O.Q4_K, seed=40 + i)
        raws[p] = raw
        model.weights[f"model.layers.0.{PROJ[p]}"] = GGUFQuantTensor(
            torch.from_numpy(np.ascontiguousarray(raw).reshape(n, -1)).cuda(), O.Q4_K, (n, k))
    return model, raws


@pytest.mark.parametrize("m", [1, 16, 64])
@pytest.mark.parametrize("graph", [False, True], ids=["eager", "graph"])
def test_layer_linears_match_oracle(cuda, graph, m):
    """M = 1: grouped decode GEMVs; M = 16 / 64 (batched decode): grouped fused-dequant GEMMs."""
    model, raws = _model(cuda)
    xs = {nm: torch.from_numpy(O.make_activations(m, k, seed=60 + j)).to(torch.bfloat16).cuda()
          for j, (nm, k) in enumerate((("normed", 512), ("attn_out", 512), ("ffn_normed", 512), ("ffn_act", 1792)))}
    bufs = {p: torch.empty((m, n), dtype=torch.float32, device="cuda") for p, (n, _) in SHAPES.items()}
    call = model.layer_linears_graph if graph else model.layer_linears
    for rep in range(3 if graph else 1):  # graph: captured on the first call, replayed after
        for nm in xs:  # refill the static inputs between replays
            xs[nm].copy_(torch.from_numpy(O.make_activations(m, xs[nm].shape[1], seed=70 + rep)).to(torch.bfloat16))
        call(0, xs["normed"], xs["attn_out"], xs["ffn_normed"], xs["ffn_act"], bufs)
        torch.cuda.synchronize()
        for p, (n, k) in SHAPES.items():
            ref = O.matmul_ref(xs[INPUT[p]].float().cpu().numpy(), raws[p], O.Q4_K, n, k)
            assert O.rel_err(bufs[p].cpu().numpy(), ref) <= TOL, (p, rep)


@pytest.mark.parametrize("m", [1, 16])
def test_layer_linears_graph_with_staged_host_copies(cuda, m):
    """The serving path: one replay copies the activations in from pinned host memory,
    runs the projections and copies the outputs back; the host buffers are refilled
    between replays."""
    model, raws = _model(cuda)
    dims = (("normed", 512), ("attn_out", 512), ("ffn_normed", 512), ("ffn_act", 1792))
    kin = sum(k for _, k in dims)
    hin = torch.empty((m, kin), dtype=torch.bfloat16).pin_memory()
    din = torch.empty((m, kin), dtype=torch.bfloat16, device="cuda")
    xs, off = {}, 0
    for nm, k in dims:
        xs[nm] = din[:, off:off + k]
        off += k
    nout = sum(n for n, _ in SHAPES.values())
    dout = torch.empty((m * nout,), dtype=torch.float32, device="cuda")
    hout = torch.empty_like(dout, device="cpu").pin_memory()
    bufs, off = {}, 0
    for p, (n, _) in SHAPES.items():
        bufs[p] = dout[off:off + m * n].view(m, n)
        off += m * n
    for rep in range(3):
        hin.copy_(torch.from_numpy(O.make_activations(m, kin, seed=90 + rep)).to(torch.bfloat16))
        model.layer_linears_graph(0, xs["normed"], xs["attn_out"], xs["ffn_normed"], xs["ffn_act"], bufs,
                                  stage_in=[(din, hin)], stage_out=[(hout, dout)])
        torch.cuda.current_stream().synchronize()
        off = 0
        hx = {}
        for nm, k in dims:
            hx[nm] = hin[:, off:off + k].float().numpy()
            off += k
        off = 0
        for p, (n, k) in SHAPES.items():
            got = hout[off:off + m * n].view(m, n).numpy()
            off += m * n
            ref = O.matmul_ref(hx[INPUT[p]], raws[p], O.Q4_K, n, k)
            assert O.rel_err(got, ref) <= TOL, (p, rep)
