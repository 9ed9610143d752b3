"""GPU dequantization is bit-identical to gguf-py (golden vectors) and to the
oracle on seeded BASELINE-shaped weights."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O
from tests.helpers import QTYPES, QNAMES, golden, same_bits

pytestmark = pytest.mark.gpu


def _gpu_deq(raw: np.ndarray, qt: int, n: int, k: int, dtype=torch.float32) -> np.ndarray:
    from vllm_webgpu_b200 import ops
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    w = GGUFQuantTensor(torch.from_numpy(np.ascontiguousarray(raw).reshape(n, -1)).cuda(), qt, (n, k))
    out = ops.dequantize(w, out_dtype=dtype)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
@pytest.mark.parametrize("which", ["rand", "edge"])
def test_dequant_golden_bit_exact(cuda, qt, which):
    g = golden(qt)
    blk = g[f"blocks_{which}"]
    bs = O.block_size(qt)
    out = _gpu_deq(blk, qt, blk.shape[0], bs)
    assert same_bits(out, g[f"deq_{which}"])


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
@pytest.mark.parametrize("n,k", [(1, 256), (37, 768), (1024, 4096), (256, 14336)])
def test_dequant_seeded_bit_exact(cuda, qt, n, k):
    raw = O.make_weights(n, k, qt, seed=n + k)
    assert same_bits(_gpu_deq(raw, qt, n, k), O.dequantize(raw, qt, n, k))


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
def test_dequant_fp16_is_one_rounding(cuda, qt):
    raw = O.make_weights(64, 4096, qt, seed=5)
    ref = O.dequantize(raw, qt, 64, 4096).astype(np.float16).astype(np.float32)
    assert same_bits(_gpu_deq(raw, qt, 64, 4096, torch.float16), ref)


def test_dequant_full_config_size(cuda):
    """BASELINE config 4 weight (14336 x 4096 Q4_K): exact on a sampled slab,
    and the fp32 checksum of the whole matrix matches the oracle's."""
    qt, n, k = O.Q4_K, 14336, 4096
    raw = O.make_weights(n, k, qt, seed=0)
    gpu = _gpu_deq(raw, qt, n, k)
    ref = O.dequantize(raw, qt, n, k)
    assert same_bits(gpu, ref)
