"""The five BASELINE configurations at their exact shapes and dtypes, each checked
against the oracle (gguf-py's dequantize restated in numpy, then a float64 matmul).

1. Q8_0 matvec: W 4096 x 4096 quantized by gguf's own Q8_0 rule, x fp32 [1, 4096].
2. Q4_0 GEMV: N = 14336, K = 4096, M in {1, 4, 8}, x fp16.
3. Q4_K Llama-3-8B layer (q, k, v, o, gate, up, down) at M in {1, 16, 64}, x bf16,
   through the model's ``layer_linears`` (the reference's call sites).
4. Q4_K / Q6_K prefill GEMM: N = 14336, K = 4096, M in {512, 2048, 8192}, x bf16,
   bf16 output; sampled tokens x sampled weight rows against the oracle.
5. Q4_K SwiGLU FFN of Llama-3-70B (hidden 8192, intermediate 28672) at world 1,
   M in {1, 32, 2048}; sampled tokens and output features against the oracle FFN.

Gates: max|y - y_ref| / rms(y_ref) <= 2e-3 for fp32 outputs. A bf16 output adds its
own rounding, half a bf16 ulp of |y_ref| (at most 2^-8 relative) per element. The FFN is a
chain of three matmuls with an fp32 SwiGLU between them, so its gate is 1.5 x 2e-3.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O
from tests.helpers import TOL

pytestmark = pytest.mark.gpu

BF16_HALF_ULP = 2.0 ** -8  # half a bf16 ulp, relative to the value (worst case at a binade bottom)


def _wt(raw: np.ndarray, qt: int, n: int, k: int):
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    return GGUFQuantTensor(torch.from_numpy(np.ascontiguousarray(raw).reshape(n, -1)).cuda(), qt, (n, k))


def _deq(w, rows=None) -> np.ndarray:
    """Oracle dequantization (float32, exact) of a GGUFQuantTensor's rows."""
    raw = w.data.cpu().numpy() if rows is None else w.data[rows].cpu().numpy()
    n = raw.shape[0]
    return O.dequantize(raw, w.qtype, n, w.k)


def _mm(x: np.ndarray, w: np.ndarray, step: int = 2048) -> np.ndarray:
    """x @ w.T in float64, converting w a slab of rows at a time."""
    x = np.asarray(x, np.float64)
    return np.concatenate([x @ w[i:i + step].astype(np.float64).T for i in range(0, w.shape[0], step)], axis=1)


def _bf16_ok(y: np.ndarray, ref: np.ndarray) -> bool:
    rms = float(np.sqrt(np.mean(ref ** 2)))
    return bool(np.all(np.abs(y - ref) <= TOL * rms + BF16_HALF_ULP * np.abs(ref)))


# ---- config 1 -------------------------------------------------------------------------

def test_config1_q8_0_matvec_fp32(cuda):
    from vllm_webgpu_b200 import ops
    n = k = 4096
    raw = O.make_weights(n, k, O.Q8_0, seed=0)  # gguf's Q8_0 rule: d = max|w| / 127, q = round(w / d)
    x = O.make_activations(1, k, seed=1)        # fp32 ~ N(0, 1)
    y = ops.mul_mat(torch.from_numpy(x).cuda(), _wt(raw, O.Q8_0, n, k), out_dtype=torch.float32)
    ref = O.matmul_ref(x, raw, O.Q8_0, n, k)
    assert O.rel_err(y.cpu().numpy(), ref) <= TOL


# ---- config 2 -------------------------------------------------------------------------

@pytest.fixture(scope="module")
def q4_0_ffn_up():
    n, k = 14336, 4096
    raw = O.make_weights(n, k, O.Q4_0, seed=0)
    return raw, O.dequantize(raw, O.Q4_0, n, k)


@pytest.mark.parametrize("m", [1, 4, 8])
def test_config2_q4_0_gemv_fp16(cuda, q4_0_ffn_up, m):
    from vllm_webgpu_b200 import ops
    raw, wd = q4_0_ffn_up
    n, k = wd.shape
    x = torch.from_numpy(O.make_activations(m, k, seed=1)).to(torch.float16).cuda()
    y = ops.mul_mat(x, _wt(raw, O.Q4_0, n, k), out_dtype=torch.float32)
    ref = _mm(x.double().cpu().numpy(), wd)
    assert O.rel_err(y.cpu().numpy(), ref) <= TOL


# ---- config 3 -------------------------------------------------------------------------

LAYER = [("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
         ("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336)]


@pytest.fixture(scope="module")
def llama8b_layer(cuda):
    from vllm_webgpu_b200.models.llama import PROJ, LlamaB200Model
    from vllm_webgpu_b200.quant.pack import random_weights
    model = LlamaB200Model(None, device=cuda)
    deq = {}
    for i, (p, n, k) in enumerate(LAYER):
        w = random_weights(n, k, O.Q4_K, seed=300 + i, device=cuda)
        model.weights[f"model.layers.0.{PROJ[p]}"] = w
        deq[p] = _deq(w)
    return model, deq


@pytest.mark.parametrize("m", [1, 16, 64])
def test_config3_q4k_llama8b_layer(cuda, llama8b_layer, m):
    model, deq = llama8b_layer
    g = torch.Generator(device=cuda)
    g.manual_seed(40 + m)
    xs = {name: torch.randn((m, kk), generator=g, device=cuda).to(torch.bfloat16)
          for name, kk in (("normed", 4096), ("attn_out", 4096), ("ffn_normed", 4096), ("ffn_act", 14336))}
    bufs = {p: torch.empty((m, n), dtype=torch.float32, device=cuda) for p, n, _ in LAYER}
    model.layer_linears(0, xs["normed"], xs["attn_out"], xs["ffn_normed"], xs["ffn_act"], bufs)
    torch.cuda.synchronize()
    src = {"q": "normed", "k": "normed", "v": "normed", "o": "attn_out", "gate": "ffn_normed",
           "up": "ffn_normed", "down": "ffn_act"}
    for p, _, _ in LAYER:
        ref = _mm(xs[src[p]].double().cpu().numpy(), deq[p])
        err = O.rel_err(bufs[p].cpu().numpy(), ref)
        assert err <= TOL, (p, m, err)


# ---- config 4 -------------------------------------------------------------------------

@pytest.fixture(scope="module")
def prefill_weights(cuda):
    from vllm_webgpu_b200.quant.pack import random_weights
    return {qt: random_weights(14336, 4096, qt, seed=400 + qt, device=cuda) for qt in (O.Q4_K, O.Q6_K)}


@pytest.mark.parametrize("qt", [O.Q4_K, O.Q6_K], ids=["Q4_K", "Q6_K"])
@pytest.mark.parametrize("m", [512, 2048, 8192])
def test_config4_prefill_gemm_bf16(cuda, prefill_weights, qt, m):
    from vllm_webgpu_b200 import ops
    w = prefill_weights[qt]
    g = torch.Generator(device=cuda)
    g.manual_seed(50 + m)
    x = torch.randn((m, w.k), generator=g, device=cuda).to(torch.bfloat16)
    y16 = ops.gemm(x, w, out_dtype=torch.bfloat16)
    y32 = ops.gemm(x, w, out_dtype=torch.float32)
    torch.cuda.synchronize()
    rng = np.random.default_rng(m + qt)
    toks = np.sort(rng.choice(m, size=48, replace=False))
    rows = np.sort(rng.choice(w.n, size=384, replace=False))
    rows_t = torch.from_numpy(rows).cuda()
    ref = _mm(x[torch.from_numpy(toks).cuda()].double().cpu().numpy(), _deq(w, rows_t))
    got32 = y32[toks][:, rows].cpu().numpy()
    got16 = y16[toks][:, rows].float().cpu().numpy()
    assert O.rel_err(got32, ref) <= TOL
    assert _bf16_ok(got16, ref)


# ---- config 5 -------------------------------------------------------------------------

HID, INTER = 8192, 28672


@pytest.fixture(scope="module")
def ffn70b(cuda):
    from vllm_webgpu_b200.quant.pack import random_weights
    from vllm_webgpu_b200.tp import TensorParallelSwiGLU
    gate = random_weights(INTER, HID, O.Q4_K, seed=501, device=cuda)
    up = random_weights(INTER, HID, O.Q4_K, seed=502, device=cuda)
    down = random_weights(HID, INTER, O.Q4_K, seed=503, device=cuda)
    ffn = TensorParallelSwiGLU(gate, up, down, rank=0, world=1)
    out_rows = np.sort(np.random.default_rng(5).choice(HID, size=256, replace=False))
    return ffn, _deq(gate), _deq(up), out_rows, _deq(down, torch.from_numpy(out_rows).cuda())


@pytest.mark.parametrize("m", [1, 32, 2048])
def test_config5_swiglu_ffn_70b_world1(cuda, ffn70b, m):
    ffn, wg, wu, out_rows, wd_rows = ffn70b
    g = torch.Generator(device=cuda)
    g.manual_seed(60 + m)
    x = torch.randn((m, HID), generator=g, device=cuda).to(torch.bfloat16)
    y = ffn(x)
    torch.cuda.synchronize()
    toks = np.sort(np.random.default_rng(m).choice(m, size=min(m, 6), replace=False))
    xs = x[torch.from_numpy(toks).cuda()].double().cpu().numpy()
    gs, us = _mm(xs, wg), _mm(xs, wu)
    act = gs / (1.0 + np.exp(-gs)) * us
    ref = _mm(act, wd_rows)
    got = y.float()[torch.from_numpy(toks).cuda()][:, torch.from_numpy(out_rows).cuda()].cpu().numpy()
    assert O.rel_err(got, ref) <= 1.5 * TOL
