"""The FFN epilogues above the decode GEMV (and for the formats its fused forms do not
cover): SwiGLU of gate and up, and the residual add, in the GEMM's epilogue pass
(ggufmm_gemm_swiglu / ggufmm_gemm_residual) or after a grouped decode GEMV
(ggufmm_ffn_epilogue) -- against the oracle, through the ops and the model's calls.

Gate: max|y - y_ref| / rms(y_ref) <= 2e-3 on fp32 outputs; the SwiGLU is the product of
two matmuls, so its gate is 1.5 x 2e-3 (as for the FFN chain)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O
from tests.helpers import QNAMES, QTYPES, TOL

pytestmark = pytest.mark.gpu


def _wt(raw, qt, n, k):
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    return GGUFQuantTensor(torch.from_numpy(np.ascontiguousarray(raw).reshape(n, -1)).cuda(), qt, (n, k))


def _swiglu_ref(x, rg, ru, qt, n, k):
    g = O.matmul_ref(x, rg, qt, n, k)
    u = O.matmul_ref(x, ru, qt, n, k)
    return g / (1.0 + np.exp(-g)) * u


def _gemm_unsplit(x, w):
    """ops.gemm with a workspace that holds only the fp16 operands: the persistent
    GEMM then runs its last wave unsplit, as the epilogue path's GEMM does, so the
    two accumulate in the same order."""
    from vllm_webgpu_b200 import ops
    m = x.shape[0]
    ws = torch.empty(w.n * w.k * 2 + (m * w.k * 2 + 255) // 256 * 256, dtype=torch.uint8, device=x.device)
    return ops.gemm(x, w, out_dtype=torch.float32, workspace=ws)


def _check_swiglu(y, x, gate, up, rg, ru, qt, n, k):
    """Decode (M <= 8, the integer / fp16 GEMV): against the oracle SwiGLU at 1.5 x 2e-3.
    Above it the GEMM runs on fp16 operands, so each of gate and up is within 2e-3 of the
    oracle and their product can reach ~4e-3 of its rms: the epilogue is checked against
    silu(g) * u of the same GEMM's gate and up outputs (1e-5), and those against the
    oracle at 2e-3."""
    from vllm_webgpu_b200 import ops
    xn = x.float().cpu().numpy()
    if x.shape[0] <= ops.GEMV_MAX_M:
        assert O.rel_err(y.cpu().numpy(), _swiglu_ref(xn, rg, ru, qt, n, k)) <= 1.5 * TOL
        return
    g = _gemm_unsplit(x, gate)
    u = _gemm_unsplit(x, up)
    assert O.rel_err(g.cpu().numpy(), O.matmul_ref(xn, rg, qt, n, k)) <= TOL
    assert O.rel_err(u.cpu().numpy(), O.matmul_ref(xn, ru, qt, n, k)) <= TOL
    ref = (torch.nn.functional.silu(g.double()) * u.double()).cpu().numpy()
    # Q4_K runs the fused-dequant GEMM, whose K split can differ between the grouped
    # launch and the single-weight ones; the tensor core's fp32 accumulation is not
    # reassociation-exact, so those agree to ~1e-4 of the RMS rather than bit for bit
    assert O.rel_err(y.cpu().numpy(), ref) <= (1e-3 if qt == O.Q4_K else 1e-5)


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
@pytest.mark.parametrize("m", [2, 16, 64, 200, 1100])
def test_swiglu_any_m(cuda, qt, m):
    """M = 2: decode (fused integer GEMV for Q4_K / Q4_0, grouped GEMV + epilogue pass
    otherwise); M = 16 / 64 / 200: the fused-dequant GEMM's partials (Q4_K; 256-token
    tiles at 200) or the two-pass GEMM; M = 1100: the two-pass GEMM for every format,
    all with the SwiGLU in the epilogue."""
    from vllm_webgpu_b200 import ops
    n, k = 1536, 2048
    rg, ru = O.make_weights(n, k, qt, seed=1), O.make_weights(n, k, qt, seed=2)
    gate, up = _wt(rg, qt, n, k), _wt(ru, qt, n, k)
    x = torch.from_numpy(O.make_activations(m, k, seed=3)).to(torch.bfloat16).cuda()
    y = ops.swiglu(x, gate, up, out_dtype=torch.float32)
    _check_swiglu(y, x, gate, up, rg, ru, qt, n, k)


@pytest.mark.parametrize("qt", [O.Q4_K, O.Q8_0], ids=["Q4_K", "Q8_0"])
@pytest.mark.parametrize("m", [3, 32, 160, 600])
def test_residual_any_m_in_place(cuda, qt, m):
    from vllm_webgpu_b200 import ops
    n, k = 1024, 4096
    raw = O.make_weights(n, k, qt, seed=5)
    x = torch.from_numpy(O.make_activations(m, k, seed=6)).to(torch.bfloat16).cuda()
    h = torch.from_numpy(O.make_activations(m, n, seed=7)).cuda()
    h0 = h.cpu().numpy().astype(np.float64)
    ops.linear_residual(x, _wt(raw, qt, n, k), h, out=h)  # h = h + x W^T in place
    ref = O.matmul_ref(x.float().cpu().numpy(), raw, qt, n, k) + h0
    assert O.rel_err(h.cpu().numpy(), ref) <= TOL


def test_gemm_swiglu_matches_separate_projections_4096x14336(cuda):
    """Llama-3-8B FFN width at M = 64 through the fused-dequant partials (one launch for
    gate and up), against gate and up as separate GEMMs and the same SwiGLU."""
    from vllm_webgpu_b200 import ops
    from vllm_webgpu_b200.quant.pack import random_weights
    gate = random_weights(14336, 4096, O.Q4_K, seed=8, device=cuda)
    up = random_weights(14336, 4096, O.Q4_K, seed=9, device=cuda)
    x = torch.randn((64, 4096), device=cuda).to(torch.bfloat16)
    y = ops.gemm_swiglu(x, gate, up, out_dtype=torch.float32)
    g = ops.gemm(x, gate, out_dtype=torch.float32)
    u = ops.gemm(x, up, out_dtype=torch.float32)
    ref = (torch.nn.functional.silu(g) * u).double().cpu().numpy()
    # the grouped launch may split K differently from the single-weight launches (two
    # CTAs per SM when the launch is large), and the tensor core's fp32 accumulation is
    # not reassociation-exact, so the sums agree to ~1e-4 of their RMS, not bit for bit
    assert O.rel_err(y.cpu().numpy(), ref) <= 1e-3


@pytest.mark.parametrize("m", [16, 64])
def test_model_ffn_act_and_residual_projections_batched(cuda, m):
    """The model's project_ffn_act and project_o / project_down with out = residual at
    batched-decode M: native epilogues, and the residual is not lost when updated in place."""
    from vllm_webgpu_b200.models.llama import PROJ, LlamaB200Model
    h, it = 512, 1792
    model = LlamaB200Model(None, device=cuda)
    raws = {}
    for i, (p, (n, k)) in enumerate({"o": (h, h), "gate": (it, h), "up": (it, h), "down": (h, it)}.items()):
        raws[p] = O.make_weights(n, k, O.Q4_K, seed=60 + i)
        model.weights[f"model.layers.0.{PROJ[p]}"] = _wt(raws[p], O.Q4_K, n, k)
    xf = torch.from_numpy(O.make_activations(m, h, seed=11)).to(torch.bfloat16).cuda()
    act = torch.empty((m, it), dtype=torch.float32, device=cuda)
    model.project_ffn_act(0, xf, act)
    _check_swiglu(act, xf, model.weights[f"model.layers.0.{PROJ['gate']}"], model.weights[f"model.layers.0.{PROJ['up']}"],
                  raws["gate"], raws["up"], O.Q4_K, it, h)
    hid = torch.from_numpy(O.make_activations(m, h, seed=12)).cuda()
    h0 = hid.cpu().numpy().astype(np.float64)
    attn = torch.from_numpy(O.make_activations(m, h, seed=13)).to(torch.bfloat16).cuda()
    model.project_o(0, attn, hid, residual=hid)
    ref_o = O.matmul_ref(attn.float().cpu().numpy(), raws["o"], O.Q4_K, h, h) + h0
    assert O.rel_err(hid.cpu().numpy(), ref_o) <= TOL
    a16 = act.to(torch.bfloat16)
    h1 = hid.cpu().numpy().astype(np.float64)
    model.project_down(0, a16, hid, residual=hid)
    ref_d = O.matmul_ref(a16.float().cpu().numpy(), raws["down"], O.Q4_K, h, it) + h1
    assert O.rel_err(hid.cpu().numpy(), ref_d) <= TOL
