"""GGUF file -> CUDA -> kernels, on a GPU: a file written by gguf-py with the
mixed block types of a Q4_K_M-style Llama-3-8B layer is loaded with
``load_gguf_weights(path, device="cuda")`` (the reference's loader API,
vllm_webgpu/quant/gguf_loader.py:137-162, which uploaded flat bytes and lost the
block type), and the layer's projections run from it against the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O
from tests.helpers import TOL

pytestmark = pytest.mark.gpu
gguf = pytest.importorskip("gguf")

# GGUF tensor name -> (HF projection key, N, K, block type)
LAYER = {
    "blk.0.attn_q.weight": ("q", 4096, 4096, O.Q4_K),
    "blk.0.attn_k.weight": ("k", 1024, 4096, O.Q8_0),
    "blk.0.attn_v.weight": ("v", 1024, 4096, O.Q6_K),
    "blk.0.attn_output.weight": ("o", 4096, 4096, O.Q4_0),
    "blk.0.ffn_gate.weight": ("gate", 14336, 4096, O.Q4_K),
    "blk.0.ffn_up.weight": ("up", 14336, 4096, O.Q4_K),
    "blk.0.ffn_down.weight": ("down", 4096, 14336, O.Q6_K),
}


@pytest.fixture(scope="module")
def gguf_layer(cuda, tmp_path_factory):
    from vllm_webgpu_b200.quant.pack import random_weights
    path = tmp_path_factory.mktemp("gguf") / "layer.gguf"
    raws = {}
    wr = gguf.GGUFWriter(str(path), "llama")
    wr.add_block_count(1)
    wr.add_embedding_length(4096)
    wr.add_feed_forward_length(14336)
    wr.add_head_count(32)
    wr.add_head_count_kv(8)
    wr.add_context_length(8192)
    wr.add_rope_freq_base(500000.0)
    for i, (name, (_, n, k, qt)) in enumerate(LAYER.items()):
        raw = random_weights(n, k, qt, seed=700 + i, device=cuda).data.cpu().numpy()
        raws[name] = raw
        wr.add_tensor(name, raw, raw_dtype=gguf.GGMLQuantizationType(qt))
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    return path, raws


def test_gguf_file_to_cuda_keeps_blocks(cuda, gguf_layer):
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    from vllm_webgpu_b200.models.llama import PROJ
    from vllm_webgpu_b200.quant.gguf_loader import load_gguf_weights
    path, raws = gguf_layer
    w = load_gguf_weights(str(path), device="cuda")
    for name, (p, n, k, qt) in LAYER.items():
        t = w[f"model.layers.0.{PROJ[p]}"]
        assert isinstance(t, GGUFQuantTensor) and t.data.is_cuda
        assert t.qtype == qt and t.shape == (n, k)
        assert np.array_equal(t.data.cpu().numpy(), raws[name])


@pytest.mark.parametrize("m", [1, 16])
def test_gguf_file_layer_linears(cuda, gguf_layer, m):
    from vllm_webgpu_b200.models.llama import LlamaB200Model
    from vllm_webgpu_b200.quant.gguf_loader import load_gguf_weights
    path, raws = gguf_layer
    model = LlamaB200Model(None, device=cuda)
    model.weights = load_gguf_weights(str(path), device="cuda")
    g = torch.Generator(device=cuda)
    g.manual_seed(80 + m)
    xs = {nm: torch.randn((m, kk), generator=g, device=cuda).to(torch.bfloat16)
          for nm, kk in (("normed", 4096), ("attn_out", 4096), ("ffn_normed", 4096), ("ffn_act", 14336))}
    bufs = {p: torch.empty((m, n), dtype=torch.float32, device=cuda) for p, n, _, _ in LAYER.values()}
    model.layer_linears(0, xs["normed"], xs["attn_out"], xs["ffn_normed"], xs["ffn_act"], bufs)
    torch.cuda.synchronize()
    src = {"q": "normed", "k": "normed", "v": "normed", "o": "attn_out", "gate": "ffn_normed",
           "up": "ffn_normed", "down": "ffn_act"}
    for name, (p, n, k, qt) in LAYER.items():
        ref = O.matmul_ref(xs[src[p]].float().cpu().numpy(), raws[name], qt, n, k)
        err = O.rel_err(bufs[p].cpu().numpy(), ref)
        assert err <= TOL, (p, O.QTYPES[qt][0], m, err)
