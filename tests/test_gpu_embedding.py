"""Quantized embedding lookup (ggufmm_embedding) against the oracle: rows of a GGUF
table dequantized bit-exactly (fp32) or rounded once (f16 / bf16), through the op
and the model's embedding_lookup dispatch; out-of-range ids are reported."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O
from tests.helpers import QNAMES, QTYPES, bf16_round, same_bits

pytestmark = pytest.mark.gpu


def _table(qt, vocab, hidden, seed):
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    raw = O.make_weights(vocab, hidden, qt, seed=seed)
    return raw, GGUFQuantTensor(torch.from_numpy(raw).cuda(), qt, (vocab, hidden))


@pytest.mark.parametrize("qt", QTYPES, ids=lambda q: QNAMES[q])
@pytest.mark.parametrize("hidden", [4096, 5120])
def test_embedding_bit_exact(cuda, qt, hidden):
    from vllm_webgpu_b200 import ops
    vocab = 1000
    raw, t = _table(qt, vocab, hidden, seed=3)
    ids = np.array([0, vocab - 1, 7, 7, 512, 999, 3, 250], dtype=np.int64)
    full = O.dequantize(raw, qt, vocab, hidden)
    got = ops.embedding(torch.from_numpy(ids).cuda(), t, out_dtype=torch.float32)
    assert same_bits(got.cpu().numpy(), full[ids])
    g16 = ops.embedding(torch.from_numpy(ids).cuda(), t, out_dtype=torch.float16)
    assert np.array_equal(g16.cpu().numpy(), full[ids].astype(np.float16))
    gbf = ops.embedding(torch.from_numpy(ids).cuda(), t, out_dtype=torch.bfloat16)
    assert np.array_equal(gbf.float().cpu().numpy(), bf16_round(full[ids]))


def test_embedding_llama3_vocab_and_dispatch(cuda):
    """Llama-3 shape (128256 x 4096, Q6_K as in Q4_K_M files) through the model's
    embedding_lookup dispatch; a strided output row layout."""
    from vllm_webgpu_b200.models.llama import LlamaB200Model
    from vllm_webgpu_b200.quant.pack import random_weights
    vocab, hidden = 128256, 4096
    t = random_weights(vocab, hidden, O.Q6_K, seed=11, device=cuda)
    model = LlamaB200Model(None, device=cuda)
    model.weights["model.embed_tokens.weight"] = t
    ids = torch.tensor([128255, 0, 42, 100000, 5], dtype=torch.int32, device=cuda)
    buf = torch.empty((5, 2 * hidden), dtype=torch.bfloat16, device=cuda)
    out = buf[:, :hidden]
    model.embed_tokens(ids, out)
    rows = t.data[ids.long()].cpu().numpy()
    ref = O.dequantize(rows, O.Q6_K, 5, hidden)
    assert np.array_equal(out.float().cpu().numpy(), bf16_round(ref))


def test_embedding_out_of_range_is_reported(cuda):
    from vllm_webgpu_b200 import _lib, ops
    raw, t = _table(O.Q4_K, 64, 512, seed=5)
    lib = _lib.lib()
    assert lib.ggufmm_device_status(1, None) == 0
    got = ops.embedding(torch.tensor([3, 64, -1], dtype=torch.int32, device="cuda"), t, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert lib.ggufmm_device_status(1, None) == 2
    assert torch.count_nonzero(got[1:]).item() == 0
    full = O.dequantize(raw, O.Q4_K, 64, 512)
    assert same_bits(got[0].cpu().numpy(), full[3])
    assert lib.ggufmm_device_status(0, None) == 0
