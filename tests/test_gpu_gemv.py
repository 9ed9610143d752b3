"""Decode GEMV (M <= 8) against the fp32 dequantize-then-matmul oracle.

Gate: max|y - y_ref| / rms(y_ref) <= 2e-3 (the tolerance of the north star)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O
from tests.helpers import QTYPES, QNAMES, TOL, bf16_round, golden

pytestmark = pytest.mark.gpu


def _wt(raw, qt, n, k):
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    return GGUFQuantTensor(torch.from_numpy(np.ascontiguousarray(raw).reshape(n, -1)).cuda(), qt, (n, k))


def _run(qt, m, n, k, xdtype=torch.bfloat16, ydtype=torch.float32, seed=0):
    from vllm_webgpu_b200 import ops
    raw = O.make_weights(n, k, qt, seed=seed)
    x = O.make_activations(m, k, seed=seed + 1)
    xt = torch.from_numpy(x).to(xdtype).cuda()
    y = ops.gemv(xt, _wt(raw, qt, n, k), out_dtype=ydtype)
    torch.cuda.synchronize()
    ref = O.matmul_ref(xt.float().cpu().numpy(), raw, qt, n, k)
    return y.float().cpu().numpy(), ref


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
@pytest.mark.parametrize("m", [1, 2, 3, 4, 8])
def test_gemv_llama_shapes(cuda, qt, m):
    y, ref = _run(qt, m, 4096, 4096)
    assert O.rel_err(y, ref) <= TOL


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
@pytest.mark.parametrize("n,k", [(14336, 4096), (4096, 14336), (1024, 4096)])
def test_gemv_layer_shapes_m1(cuda, qt, n, k):
    y, ref = _run(qt, 1, n, k)
    assert O.rel_err(y, ref) <= TOL


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
@pytest.mark.parametrize("n,k,m", [(1, 2048, 1), (5, 2048, 3), (7, 6144, 2), (13, 18432, 1), (9, 32768, 1),
                                   (3, 65536, 1), (18, 1024, 2), (33, 8192, 1), (40, 12288, 1), (21, 256, 8)])
def test_gemv_ragged_and_wide(cuda, qt, n, k, m):
    """N not a multiple of the row tile (row groups copied whole, partly filled);
    K in one piece, in several pieces, and with a short last piece."""
    y, ref = _run(qt, m, n, k)
    assert O.rel_err(y, ref) <= TOL


@pytest.mark.parametrize("xd", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("yd", [torch.float32, torch.float16, torch.bfloat16])
def test_gemv_dtypes(cuda, xd, yd):
    y, ref = _run(O.Q4_K, 2, 2048, 4096, xdtype=xd, ydtype=yd)
    tol = TOL if yd == torch.float32 else (5e-3 if yd == torch.float16 else 2e-2)
    assert O.rel_err(y, ref) <= tol


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
def test_gemv_golden_case(cuda, qt):
    from vllm_webgpu_b200 import ops
    g = golden(qt)
    m, n, k = (int(v) for v in g["mm_shape"])
    y = ops.gemv(torch.from_numpy(g["mm_x"]).cuda(), _wt(g["mm_w"], qt, n, k))
    assert O.rel_err(y.cpu().numpy(), g["mm_y32"]) <= TOL


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
def test_gemv_linearity(cuda, qt):
    """W(a x1 + x2) == a W x1 + W x2 (fp32 activations)."""
    from vllm_webgpu_b200 import ops
    n, k = 512, 4096
    w = _wt(O.make_weights(n, k, qt, seed=9), qt, n, k)
    rng = np.random.default_rng(4)
    x1 = torch.from_numpy(rng.standard_normal((1, k), dtype=np.float32)).cuda()
    x2 = torch.from_numpy(rng.standard_normal((1, k), dtype=np.float32)).cuda()
    lhs = ops.gemv(2.0 * x1 + x2, w)
    rhs = 2.0 * ops.gemv(x1, w) + ops.gemv(x2, w)
    assert O.rel_err(lhs.cpu().numpy(), rhs.cpu().numpy()) <= 1e-4


def test_gemv_zero_and_strided_input(cuda):
    from vllm_webgpu_b200 import ops
    n, k = 256, 4096
    raw = O.make_weights(n, k, O.Q4_K, seed=1)
    w = _wt(raw, O.Q4_K, n, k)
    z = ops.gemv(torch.zeros((3, k), dtype=torch.bfloat16, device="cuda"), w)
    assert torch.count_nonzero(z).item() == 0
    big = torch.randn((4, 2 * k), device="cuda").to(torch.bfloat16)
    xs = big[:, :k]  # row stride 2K
    y = ops.gemv(xs, w, out_dtype=torch.float32)
    ref = O.matmul_ref(xs.float().cpu().numpy(), raw, O.Q4_K, n, k)
    assert O.rel_err(y.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("n,k,m", [(4096, 5120, 1), (1024, 3584, 2), (4096, 1536, 1), (33, 8960, 3), (17, 2560, 8),
                                   (64, 1280, 1)])
def test_gemv_q6k_rows_not_16_byte_multiples(cuda, n, k, m):
    """Q6_K rows of K/256 not a multiple of 8 (K = 5120: 4200 bytes) start at every
    2-byte offset mod 16: staged by the fp16 tensor-core GEMV, not refused."""
    from vllm_webgpu_b200 import ops
    assert O.row_bytes(O.Q6_K, k) % 16
    raw = O.make_weights(n, k, O.Q6_K, seed=5)
    assert ops.gemv_kernel(m, _wt(raw, O.Q6_K, n, k)) == ops.GEMV_F16
    y, ref = _run(O.Q6_K, m, n, k, seed=5)
    assert O.rel_err(y, ref) <= TOL


def test_gemv_no_device_timeouts(cuda):
    from vllm_webgpu_b200 import _lib
    assert _lib.lib().ggufmm_device_status(1, None) == 0


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
@pytest.mark.parametrize("m", [1, 3])
def test_gemv_grouped_qkv_and_gate_up(cuda, qt, m):
    """Fused q/k/v (4096, 1024, 1024 rows) and gate/up in one launch each, checked
    per weight against the oracle."""
    from vllm_webgpu_b200 import ops
    k = 4096
    for ns in ((4096, 1024, 1024), (2048, 2048)):
        raws = [O.make_weights(n, k, qt, seed=31 + i) for i, n in enumerate(ns)]
        ws = [_wt(r, qt, n, k) for r, n in zip(raws, ns)]
        x = torch.from_numpy(O.make_activations(m, k, seed=7)).to(torch.bfloat16).cuda()
        ys = ops.gemv_grouped(x, ws, out_dtype=torch.float32)
        torch.cuda.synchronize()
        for r, n, y in zip(raws, ns, ys):
            assert y.shape == (m, n)
            assert O.rel_err(y.cpu().numpy(), O.matmul_ref(x.float().cpu().numpy(), r, qt, n, k)) <= TOL


def test_gemv_grouped_ragged_and_fallback(cuda):
    """Segments whose N is not a multiple of 16, and 5 fp32 tokens (10 fp16 hi/lo
    columns: more than one n8 tile, so one GEMV per weight is launched instead)."""
    from vllm_webgpu_b200 import ops
    for qt, k, ns, m, xd in ((O.Q4_K, 2048, (37, 5, 300), 2, torch.bfloat16), (O.Q8_0, 2048, (64, 19), 5, torch.float32)):
        raws = [O.make_weights(n, k, qt, seed=5 + i) for i, n in enumerate(ns)]
        ws = [_wt(r, qt, n, k) for r, n in zip(raws, ns)]
        x = torch.from_numpy(O.make_activations(m, k, seed=9)).to(xd).cuda()
        ys = ops.gemv_grouped(x, ws, out_dtype=torch.float32)
        torch.cuda.synchronize()
        for r, n, y in zip(raws, ns, ys):
            assert O.rel_err(y.cpu().numpy(), O.matmul_ref(x.float().cpu().numpy(), r, qt, n, k)) <= TOL


@pytest.mark.parametrize("m", [2, 4, 8])
@pytest.mark.parametrize("n,k", [(14336, 4096), (4096, 14336)])
def test_mul_mat_decode_routing_q4k(cuda, n, k, m):
    """Q4_K decode through mul_mat, which takes the integer GEMV (one 8-warp CTA
    per SM when the row blocks fill the GPU, the 2-CTA K split when they do not)
    or, where only the streaming GEMV would fit, the tcgen05 GEMM."""
    from vllm_webgpu_b200 import ops
    raw = O.make_weights(n, k, O.Q4_K, seed=3)
    x = O.make_activations(m, k, seed=4)
    xt = torch.from_numpy(x).to(torch.bfloat16).cuda()
    w = _wt(raw, O.Q4_K, n, k)
    kind = ops.gemv_kernel(m, w, xt.dtype)
    assert kind in (ops.GEMV_INT8, ops.GEMV_F16, ops.GEMV_STREAM)
    assert ops.gemv_preferred(m, w, xt.dtype) == (kind != ops.GEMV_STREAM)
    y = ops.mul_mat(xt, w, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ref = O.matmul_ref(xt.float().cpu().numpy(), raw, O.Q4_K, n, k)
    assert O.rel_err(y.float().cpu().numpy(), ref) <= TOL


def test_gemv_kernel_kinds(cuda):
    """The headline decode shapes take the integer tensor-core GEMV."""
    from vllm_webgpu_b200 import ops
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    for n, k, m in [(14336, 4096, 1), (4096, 14336, 1), (14336, 4096, 8)]:
        w = GGUFQuantTensor(torch.empty((n, k // 256 * 144), dtype=torch.uint8, device="cuda"), O.Q4_K, (n, k))
        assert ops.gemv_kernel(m, w) == ops.GEMV_INT8, (n, k, m)
