"""The CPU oracle against the golden vectors made by gguf-py (CPU only)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import gguf_oracle as O
from tests.helpers import QTYPES, QNAMES, golden, same_bits


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
def test_dequant_matches_golden_random_blocks(qt):
    g = golden(qt)
    assert same_bits(O.dequantize(g["blocks_rand"], qt), g["deq_rand"])


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
def test_dequant_matches_golden_edge_blocks(qt):
    g = golden(qt)
    with np.errstate(invalid="ignore", over="ignore"):
        assert same_bits(O.dequantize(g["blocks_edge"], qt), g["deq_edge"])


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
def test_matmul_ref_matches_golden(qt):
    g = golden(qt)
    m, n, k = (int(v) for v in g["mm_shape"])
    y = O.matmul_ref(g["mm_x"], g["mm_w"], qt, n, k)
    # golden is numpy fp32 (the reference's own precision); ours sums in f64
    assert O.rel_err(y, g["mm_y32"]) < 1e-5


@pytest.mark.parametrize("qt", [O.Q8_0, O.Q4_0], ids=lambda q: QNAMES[q])
def test_quantize_matches_gguf_golden(qt):
    g = golden(qt)
    assert np.array_equal(O.quantize(g["quant_w"], qt).reshape(-1), g["quant_q"].reshape(-1))


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
def test_quantizer_roundtrip_error(qt):
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((16, 1024)) * 0.02).astype(np.float32)
    q = O.quantize(w, qt)
    assert q.shape == (16, O.row_bytes(qt, 1024))
    wd = O.dequantize(q, qt, 16, 1024)
    # 4-bit formats: max error well under one quant step of the widest block
    bound = {O.Q8_0: 0.03, O.Q4_0: 0.35, O.Q4_K: 0.35, O.Q6_K: 0.1}[qt]
    assert np.abs(wd - w).max() / 0.02 < bound


def test_rel_err_gate_definition():
    y = np.array([1.0, -1.0, 1.0, -1.0])
    assert O.rel_err(y + 0.001, y) == pytest.approx(0.001)


gguf = pytest.importorskip("gguf")


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
def test_oracle_equals_live_gguf_on_seeded_weights(qt):
    """Where gguf-py is importable, cross-check seeded BASELINE-shaped blocks live."""
    from gguf.quants import dequantize as gd
    q = O.make_weights(64, 4096, qt, seed=0)
    assert same_bits(O.dequantize(q, qt), gd(q, gguf.GGMLQuantizationType(qt)))
