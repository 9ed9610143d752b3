"""Tensor-core (tcgen05) GEMM against the fp32 dequantize-then-matmul oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O
from tests.helpers import QTYPES, QNAMES, TOL, golden

pytestmark = pytest.mark.gpu


def _wt(raw, qt, n, k):
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    return GGUFQuantTensor(torch.from_numpy(np.ascontiguousarray(raw).reshape(n, -1)).cuda(), qt, (n, k))


def _check(qt, m, n, k, seed=0, rows=None, ydtype=torch.float32):
    from vllm_webgpu_b200 import ops
    raw = O.make_weights(n, k, qt, seed=seed)
    x = torch.from_numpy(O.make_activations(m, k, seed=seed + 1)).to(torch.bfloat16).cuda()
    y = ops.gemm(x, _wt(raw, qt, n, k), out_dtype=ydtype)
    torch.cuda.synchronize()
    y = y.float().cpu().numpy()
    xf = x.float().cpu().numpy()
    if rows is not None:  # check a sample of output columns (weight rows)
        idx = np.random.default_rng(seed).choice(n, size=rows, replace=False)
        idx.sort()
        ref = O.matmul_ref(xf, raw[idx], qt, rows, k)
        return O.rel_err(y[:, idx], ref)
    return O.rel_err(y, O.matmul_ref(xf, raw, qt, n, k))


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
@pytest.mark.parametrize("m", [9, 16, 33, 64, 100, 256, 300])
def test_gemm_small(cuda, qt, m):
    assert _check(qt, m, 1024, 4096) <= TOL


@pytest.mark.parametrize("m,n,k", [(129, 1000, 2048), (700, 300, 4096), (1024, 1152, 1024), (1025, 640, 1024)])
def test_gemm_fused_prefill_tiles(cuda, m, n, k):
    """Q4_K above one 128-token tile: 256-token tiles of the fused-dequant GEMM (each
    CTA dequantizes its weight tile for its own token tile) up to M = 1024, ragged token
    and weight-row tails; M = 1025 takes the two-pass path."""
    assert _check(O.Q4_K, m, n, k, seed=4) <= TOL


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
@pytest.mark.parametrize("n,k", [(200, 512), (130, 2048), (4096, 14336)])
def test_gemm_ragged(cuda, qt, n, k):
    assert _check(qt, 77, n, k) <= TOL


@pytest.mark.parametrize("qt", [O.Q4_K, O.Q6_K], ids=lambda q: QNAMES[q])
@pytest.mark.parametrize("m", [512, 2048])
def test_gemm_prefill_config(cuda, qt, m):
    """BASELINE config 4 (K=4096, N=14336), 384 sampled weight rows checked."""
    assert _check(qt, m, 14336, 4096, rows=384) <= TOL


def _tail_plan(tiles, nk, sms):
    """K slices of the tiles left after the full waves (1: no split), and the tiles run whole."""
    rest = tiles % sms
    sl = min(sms // rest, nk // 8) if rest else 1
    if sl < 2:
        return 1, tiles
    kper = -(-nk // sl)
    sl = -(-nk // kper)
    return (sl, tiles - rest) if sl >= 2 else (1, tiles)


def _persistent_plan(n, m, k, sms=148):
    """The persistent GEMM's token-tile width and tail split: min over widths of
    waves x (width + 192), the split tail counted as 1/slices + 0.15 of a wave."""
    nt, nk = (n + 127) // 128, (k + 63) // 64
    best = None
    for bn in (256, 224, 192, 160, 128):
        tiles = ((m + bn - 1) // bn) * nt
        sl, _ = _tail_plan(tiles, nk, sms)
        waves = tiles // sms + 1 / sl + 0.15 if sl > 1 else -(-tiles // sms)
        cost = waves * (bn + 192)
        if best is None or cost < best[1] * 0.999:
            best = (bn, cost, sl)
    return best[0], best[2]


@pytest.mark.parametrize("n,m,bn,slices", [
    (14336, 1000, 256, 4),   # full waves + a tail of 4 tiles cut in 4 K slices
    (20000, 194, 224, 4),    # ragged weight tiles, a tail of 9 tiles
    (4096, 647, 192, 1),     # no split: the tiles fill whole waves
    (4096, 300, 160, 2),     # less than one wave: every tile split
    (1024, 300, 128, 4),
    (14336, 301, 160, 1),
])
def test_gemm_persistent_widths_and_tail_split(cuda, n, m, bn, slices):
    """Every token-tile width of the persistent GEMM (two accumulators at a
    power-of-two TMEM stride, ragged last token tile) and its K-split tail
    (fp32 partial tiles summed in order by the reduce pass); K = 2048."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert _persistent_plan(n, m, 2048, sms) == (bn, slices)
    assert _check(O.Q4_K, m, n, 2048, rows=256) <= TOL


def test_gemm_tail_split_deterministic_and_matches_unsplit(cuda):
    """The split tail sums its slices in a fixed order: identical bits on every
    call, and within fp32 rounding of the same GEMM without the split (a
    workspace too small for the partials)."""
    from vllm_webgpu_b200 import _lib, ops
    m, n, k = 1000, 14336, 2048
    raw = O.make_weights(n, k, O.Q4_K, seed=3)
    w = _wt(raw, O.Q4_K, n, k)
    x = torch.from_numpy(O.make_activations(m, k, seed=4)).to(torch.bfloat16).cuda()
    full = int(_lib.lib().ggufmm_gemm_workspace_size(O.Q4_K, m, n, k))
    base = n * k * 2 + m * k * 2
    assert full > base  # this shape splits its tail
    y1 = ops.gemm(x, w, out_dtype=torch.float32)
    y2 = ops.gemm(x, w, out_dtype=torch.float32)
    ws = torch.empty(base, dtype=torch.uint8, device="cuda")
    y0 = ops.gemm(x, w, out_dtype=torch.float32, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    rms = y0.float().pow(2).mean().sqrt()
    assert float((y1 - y0).abs().max() / rms) < 1e-4


@pytest.mark.parametrize("qt", [O.Q4_K, O.Q8_0], ids=lambda q: QNAMES[q])
def test_gemm_many_tiles_per_cta_ragged(cuda, qt):
    """785 tiles (5 token tiles x 157 weight tiles, both ragged): several tiles per
    CTA of the persistent GEMM, both TMEM accumulators reused."""
    assert _check(qt, 1100, 20000, 512, rows=512) <= TOL


@pytest.mark.parametrize("xd", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("m", [100, 300])
def test_gemm_strided_unaligned_x(cuda, xd, m):
    """Activations as a column slice of a wider buffer (base off 16-byte alignment,
    odd row stride) take the element-wise cast; aligned ones the vector cast."""
    from vllm_webgpu_b200 import ops
    qt, n, k = O.Q4_K, 512, 1024
    raw = O.make_weights(n, k, qt, seed=3)
    xs = torch.from_numpy(O.make_activations(m, k, seed=4)).to(xd)
    wide = torch.zeros((m, k + 3), dtype=xd)
    wide[:, 1:k + 1] = xs
    x = wide.cuda()[:, 1:k + 1]
    y = ops.gemm(x, _wt(raw, qt, n, k), out_dtype=torch.float32)
    torch.cuda.synchronize()
    ref = O.matmul_ref(xs.float().numpy(), raw, qt, n, k)
    assert O.rel_err(y.cpu().numpy(), ref) <= TOL


def test_gemm_prefill_8192_sampled(cuda):
    assert _check(O.Q4_K, 8192, 14336, 4096, rows=128) <= TOL


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
def test_gemm_golden_case(cuda, qt):
    from vllm_webgpu_b200 import ops
    g = golden(qt)
    m, n, k = (int(v) for v in g["mm_shape"])
    y = ops.gemm(torch.from_numpy(g["mm_x"]).cuda(), _wt(g["mm_w"], qt, n, k))
    assert O.rel_err(y.cpu().numpy(), g["mm_y32"]) <= TOL


def test_gemm_matches_gemv_at_m8(cuda):
    from vllm_webgpu_b200 import ops
    n, k = 2048, 4096
    w = _wt(O.make_weights(n, k, O.Q4_K, seed=2), O.Q4_K, n, k)
    x = torch.randn((8, k), device="cuda").to(torch.bfloat16)
    a = ops.gemm(x, w, out_dtype=torch.float32)
    b = ops.gemv(x, w, out_dtype=torch.float32)
    assert O.rel_err(a.cpu().numpy(), b.cpu().numpy().astype(np.float64)) <= TOL


def test_mul_mat_dispatch_and_shape(cuda):
    from vllm_webgpu_b200 import ops
    n, k = 512, 4096
    raw = O.make_weights(n, k, O.Q4_K, seed=3)
    w = _wt(raw, O.Q4_K, n, k)
    for m in (1, 8, 9, 40):
        x = torch.randn((2, m, k), device="cuda").to(torch.bfloat16)
        y = ops.mul_mat(x, w, out_dtype=torch.float32)
        assert y.shape == (2, m, n)
        ref = O.matmul_ref(x.float().reshape(-1, k).cpu().numpy(), raw, O.Q4_K, n, k)
        assert O.rel_err(y.reshape(-1, n).cpu().numpy(), ref) <= TOL


def test_gemm_no_device_timeouts(cuda):
    from vllm_webgpu_b200 import _lib
    assert _lib.lib().ggufmm_device_status(1, None) == 0


@pytest.mark.parametrize("m,n,k,yd", [(1, 1000, 4096, torch.bfloat16), (8, 4096, 14336, torch.float32),
                                      (128, 1000, 8192, torch.float16), (40, 8192, 28672, torch.float32)])
def test_gemm_fused_ksplit_ragged(cuda, m, n, k, yd):
    """Q4_K at M <= 128 on few weight-row tiles: K is split across CTAs (fp32
    partials, then an ordered sum); N not a multiple of the 128-row tile."""
    rows = 256 if n * k > 64 * 2**20 else None
    # fp16 / bf16 outputs carry their own rounding (2^-11 / 2^-8 of the largest |y|)
    tol = TOL if yd == torch.float32 else (5e-3 if yd == torch.float16 else 2e-2)
    assert _check(O.Q4_K, m, n, k, seed=5, rows=rows, ydtype=yd) <= tol


def test_gemm_fused_ksplit_deterministic(cuda):
    """The K split adds its partial sums in a fixed order: repeated calls are
    bit-identical."""
    from vllm_webgpu_b200 import ops
    n, k, m = 4096, 14336, 16
    w = _wt(O.make_weights(n, k, O.Q4_K, seed=6), O.Q4_K, n, k)
    x = torch.from_numpy(O.make_activations(m, k, seed=7)).to(torch.bfloat16).cuda()
    y0 = ops.gemm(x, w, out_dtype=torch.float32)
    for _ in range(3):
        assert torch.equal(ops.gemm(x, w, out_dtype=torch.float32), y0)


@pytest.mark.parametrize("qt", [O.Q4_K, O.Q8_0], ids=["Q4_K", "Q8_0"])
@pytest.mark.parametrize("m,shapes", [(16, [(4096, 4096), (1024, 4096), (1024, 4096)]),
                                      (33, [(1000, 2048), (300, 2048)]),
                                      (128, [(640, 1024), (640, 1024), (130, 1024), (257, 1024)]),
                                      (200, [(512, 1024), (384, 1024)])])
def test_gemm_grouped(cuda, qt, m, shapes):
    """Weights sharing the activations in one call: Q4_K at M <= 128 is one fused
    launch over every weight's row tiles (ragged N per weight, K split across CTAs);
    other types and M > 128 run one GEMM per weight."""
    from vllm_webgpu_b200 import ops
    k = shapes[0][1]
    raws = [O.make_weights(n, k, qt, seed=20 + i) for i, (n, _) in enumerate(shapes)]
    ws = [_wt(r, qt, n, k) for r, (n, _) in zip(raws, shapes)]
    x = torch.from_numpy(O.make_activations(m, k, seed=30)).to(torch.bfloat16).cuda()
    ys = ops.gemm_grouped(x, ws, out_dtype=torch.float32)
    torch.cuda.synchronize()
    xf = x.float().cpu().numpy()
    for y, r, (n, _) in zip(ys, raws, shapes):
        assert O.rel_err(y.cpu().numpy(), O.matmul_ref(xf, r, qt, n, k)) <= TOL, n
