"""Fused SwiGLU decode GEMV (ggufmm_gemv_swiglu), the model's FFN activation and
LM head, and the TP FFN routing through it, against the oracle on the GPU."""
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


def _silu(v):
    return v / (1.0 + np.exp(-v))


@pytest.mark.parametrize("qt", [O.Q4_K, O.Q4_0], ids=lambda q: QNAMES[q])
@pytest.mark.parametrize("m,n,k", [(1, 14336, 4096), (1, 3584, 8192), (2, 1000, 4096), (3, 777, 2048),
                                   (8, 512, 1024), (1, 40, 14336)])
def test_gemv_swiglu_matches_oracle(cuda, qt, m, n, k):
    from vllm_webgpu_b200 import ops
    rg, ru = O.make_weights(n, k, qt, seed=11), O.make_weights(n, k, qt, seed=12)
    x = torch.from_numpy(O.make_activations(m, k, seed=13)).to(torch.bfloat16).cuda()
    y = ops.gemv_swiglu(x, _wt(rg, qt, n, k), _wt(ru, qt, n, k), out_dtype=torch.float32)
    torch.cuda.synchronize()
    xf = x.float().cpu().numpy()
    ref = _silu(O.matmul_ref(xf, rg, qt, n, k)) * O.matmul_ref(xf, ru, qt, n, k)
    assert O.rel_err(y.cpu().numpy(), ref) <= TOL


def test_gemv_swiglu_rejects_other_formats(cuda):
    from vllm_webgpu_b200 import ops
    n, k = 256, 1024
    raw = O.make_weights(n, k, O.Q8_0, seed=1)
    x = torch.zeros((1, k), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        ops.gemv_swiglu(x, _wt(raw, O.Q8_0, n, k), _wt(raw, O.Q8_0, n, k))


def test_model_ffn_act_and_lm_head(cuda):
    from vllm_webgpu_b200.models.llama import PROJ, LlamaB200Model
    model = LlamaB200Model(None, device="cuda:0")
    hid, inter, vocab = 1024, 2816, 5000
    raws = {}
    for i, (p, (n, k)) in enumerate({"gate": (inter, hid), "up": (inter, hid)}.items()):
        raws[p] = O.make_weights(n, k, O.Q4_K, seed=20 + i)
        model.weights[f"model.layers.0.{PROJ[p]}"] = _wt(raws[p], O.Q4_K, n, k)
    rl = O.make_weights(vocab, hid, O.Q6_K, seed=30)
    model.weights["lm_head.weight"] = _wt(rl, O.Q6_K, vocab, hid)
    x = torch.from_numpy(O.make_activations(1, hid, seed=31)).to(torch.bfloat16).cuda()
    act = torch.empty((1, inter), dtype=torch.float32, device="cuda")
    logits = torch.empty((1, vocab), dtype=torch.float32, device="cuda")
    model.project_ffn_act(0, x, act)
    model.project_lm_head(x, logits)
    torch.cuda.synchronize()
    xf = x.float().cpu().numpy()
    ref_act = _silu(O.matmul_ref(xf, raws["gate"], O.Q4_K, inter, hid)) * O.matmul_ref(xf, raws["up"], O.Q4_K, inter, hid)
    assert O.rel_err(act.cpu().numpy(), ref_act) <= TOL
    assert O.rel_err(logits.cpu().numpy(), O.matmul_ref(xf, rl, O.Q6_K, vocab, hid)) <= TOL
