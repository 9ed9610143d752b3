"""Decode GEMV with the residual add in its epilogue (ggufmm_gemv_residual), the
model's o / down projections and the TP FFN taking a residual, against the oracle
on the GPU."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O
from tests.helpers import QNAMES, TOL

pytestmark = pytest.mark.gpu


def _wt(raw, qt, n, k):
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    return GGUFQuantTensor(torch.from_numpy(np.ascontiguousarray(raw).reshape(n, -1)).cuda(), qt, (n, k))


@pytest.mark.parametrize("qt", [O.Q4_K, O.Q4_0], ids=lambda q: QNAMES[q])
@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (2, 4096, 14336), (4, 14336, 4096), (3, 1000, 2048),
                                   (8, 512, 1024)])
@pytest.mark.parametrize("yd", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_gemv_residual_matches_oracle(cuda, qt, m, n, k, yd):
    """y = x W^T + r on every GEMV shape (4-warp, the 2-CTA K split of the down
    projection, 8-warp) with ragged N; fp32 and bf16 outputs."""
    from vllm_webgpu_b200 import ops
    raw = O.make_weights(n, k, qt, seed=21)
    x = torch.from_numpy(O.make_activations(m, k, seed=22)).to(torch.bfloat16).cuda()
    r = torch.from_numpy(O.make_activations(m, n, seed=23)).to(yd).cuda()
    y = ops.gemv_residual(x, _wt(raw, qt, n, k), r)
    torch.cuda.synchronize()
    ref = O.matmul_ref(x.float().cpu().numpy(), raw, qt, n, k) + r.float().cpu().numpy()
    tol = TOL if yd == torch.float32 else 2e-2  # bf16 output rounding (2^-8 of the largest |y|)
    assert O.rel_err(y.float().cpu().numpy(), ref) <= tol


def test_gemv_residual_in_place(cuda):
    """out = residual (the reference's h = h + ffn_out): each element is read and
    then written by the same thread."""
    from vllm_webgpu_b200 import ops
    n, k, m = 4096, 14336, 2
    raw = O.make_weights(n, k, O.Q4_K, seed=24)
    x = torch.from_numpy(O.make_activations(m, k, seed=25)).to(torch.bfloat16).cuda()
    h = torch.from_numpy(O.make_activations(m, n, seed=26)).float().cuda()
    ref = O.matmul_ref(x.float().cpu().numpy(), raw, O.Q4_K, n, k) + h.cpu().numpy()
    out = ops.gemv_residual(x, _wt(raw, O.Q4_K, n, k), h, out=h)
    torch.cuda.synchronize()
    assert out.data_ptr() == h.data_ptr()
    assert O.rel_err(h.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("m", [1, 16])
def test_model_projections_with_residual(cuda, m):
    """project_o / project_down with residual=: fused at M = 1, projection + add at M = 16."""
    from vllm_webgpu_b200.models.llama import PROJ, LlamaB200Model
    model = LlamaB200Model(None, device="cuda:0")
    raws = {}
    for i, (p, (n, k)) in enumerate({"o": (512, 512), "down": (512, 1792)}.items()):
        raws[p] = (O.make_weights(n, k, O.Q4_K, seed=30 + i), n, k)
        model.weights[f"model.layers.0.{PROJ[p]}"] = _wt(raws[p][0], O.Q4_K, n, k)
    for p, fn in (("o", model.project_o), ("down", model.project_down)):
        raw, n, k = raws[p]
        x = torch.from_numpy(O.make_activations(m, k, seed=40)).to(torch.bfloat16).cuda()
        r = torch.from_numpy(O.make_activations(m, n, seed=41)).float().cuda()
        out = torch.empty((m, n), dtype=torch.float32, device="cuda")
        fn(0, x, out, residual=r)
        torch.cuda.synchronize()
        ref = O.matmul_ref(x.float().cpu().numpy(), raw, O.Q4_K, n, k) + r.cpu().numpy()
        assert O.rel_err(out.cpu().numpy(), ref) <= TOL, p


@pytest.mark.parametrize("m", [1, 32])
def test_tp_ffn_residual_single_gpu(cuda, m):
    """The TP FFN at world 1 with a residual: the down projection adds it in its
    epilogue at M = 1 (fp32 reduce dtype), after the GEMM at M = 32."""
    from vllm_webgpu_b200.tp import TensorParallelSwiGLU
    h, i = 1024, 2048
    g, u, d = (_wt(O.make_weights(i, h, O.Q4_K, seed=50), O.Q4_K, i, h),
               _wt(O.make_weights(i, h, O.Q4_K, seed=51), O.Q4_K, i, h),
               _wt(O.make_weights(h, i, O.Q4_K, seed=52), O.Q4_K, h, i))
    ffn = TensorParallelSwiGLU(g, u, d)
    x = torch.from_numpy(O.make_activations(m, h, seed=53)).to(torch.bfloat16).cuda()
    r = torch.from_numpy(O.make_activations(m, h, seed=54)).float().cuda()
    y0 = ffn(x).clone()
    y1 = ffn(x, residual=r)
    torch.cuda.synchronize()
    base = y0.cpu().numpy()
    assert O.rel_err(y1.cpu().numpy(), base + r.cpu().numpy()) <= TOL
