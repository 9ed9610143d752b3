"""The product-side torch quantizer emits the same bytes as the oracle packers
(and, for Q8_0 / Q4_0, as gguf-py's quantize). CPU tensors; the same torch ops
run on CUDA."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O
from tests.helpers import QTYPES, QNAMES, golden


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
def test_pack_matches_oracle(qt):
    from vllm_webgpu_b200.quant.pack import quantize
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((24, 1024)) * 0.02).astype(np.float32)
    w[0, :256] = 0.0          # all-zero blocks
    w[1, :256] = 0.01         # constant positive blocks
    w[2, :32] *= 1000.0       # huge outlier block
    got = quantize(torch.from_numpy(w), qt)
    assert got.shape == (24, 1024)
    assert np.array_equal(got.data.numpy(), O.quantize(w, qt))


@pytest.mark.parametrize("qt", [O.Q8_0, O.Q4_0], ids=lambda q: QNAMES[q])
def test_pack_matches_gguf_golden(qt):
    from vllm_webgpu_b200.quant.pack import quantize
    g = golden(qt)
    got = quantize(torch.from_numpy(g["quant_w"]), qt)
    assert np.array_equal(got.data.numpy().reshape(-1), g["quant_q"].reshape(-1))


def test_random_weights_shape_and_determinism():
    from vllm_webgpu_b200.quant.pack import random_weights
    a = random_weights(8, 512, "Q4_K", seed=1, device="cpu")
    b = random_weights(8, 512, "Q4_K", seed=1, device="cpu")
    assert a.data.shape == (8, 288) and torch.equal(a.data, b.data)
    wd = O.dequantize(a.data.numpy(), O.Q4_K, 8, 512)
    assert 0.01 < wd.std() < 0.03


def test_quant_tensor_splits():
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    from vllm_webgpu_b200.quant.pack import quantize
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((16, 1024)) * 0.02).astype(np.float32)
    q = quantize(torch.from_numpy(w), "Q6_K")
    full = O.dequantize(q.data.numpy(), O.Q6_K, 16, 1024)
    r = q.rows(4, 12)
    assert np.array_equal(O.dequantize(r.data.numpy(), O.Q6_K, 8, 1024), full[4:12])
    c = q.cols(256, 768)
    assert np.array_equal(O.dequantize(c.data.numpy(), O.Q6_K, 16, 512), full[:, 256:768])
    with pytest.raises(ValueError):
        q.cols(100, 512)
    with pytest.raises(ValueError):
        GGUFQuantTensor(q.data[:, :10], O.Q6_K, (16, 1024))
