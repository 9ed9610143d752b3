"""Gemma 4 call sites on the GPU: attention width heads x head_dim != hidden (q/k/v
and o), gate/up/down, and the LM head tied to the quantized embedding table --
all against the oracle."""
from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O
from tests.helpers import TOL

pytestmark = pytest.mark.gpu

CFG = SimpleNamespace(hidden_size=2560, num_attention_heads=8, num_key_value_heads=2, head_dim=256,
                      intermediate_size=10240, vocab_size=4096, num_hidden_layers=1)


def _model(cuda):
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    from vllm_webgpu_b200.models.gemma4 import build_model
    from vllm_webgpu_b200.models.llama import PROJ
    model = build_model("Gemma3ForCausalLM", CFG, device=cuda)
    h, qd, kvd, it = CFG.hidden_size, model.q_dim, model.kv_dim, CFG.intermediate_size
    shapes = {"q": (qd, h, O.Q4_K), "k": (kvd, h, O.Q4_K), "v": (kvd, h, O.Q6_K), "o": (h, qd, O.Q4_K),
              "gate": (it, h, O.Q4_K), "up": (it, h, O.Q4_K), "down": (h, it, O.Q6_K)}
    raws = {}
    for i, (p, (n, k, qt)) in enumerate(shapes.items()):
        raws[p] = (O.make_weights(n, k, qt, seed=900 + i), qt, n, k)
        model.weights[f"model.layers.0.{PROJ[p]}"] = GGUFQuantTensor(torch.from_numpy(raws[p][0]).cuda(), qt, (n, k))
    emb = O.make_weights(CFG.vocab_size, h, O.Q6_K, seed=950)
    model.weights["model.embed_tokens.weight"] = GGUFQuantTensor(torch.from_numpy(emb).cuda(), O.Q6_K,
                                                                 (CFG.vocab_size, h))
    return model, raws, emb


@pytest.mark.parametrize("m", [1, 4, 32])
def test_gemma4_layer_projections(cuda, m):
    model, raws, _ = _model(cuda)
    assert model.q_dim == 2048 != CFG.hidden_size
    g = torch.Generator(device=cuda)
    g.manual_seed(m)
    xs = {"normed": torch.randn((m, CFG.hidden_size), generator=g, device=cuda).to(torch.bfloat16),
          "attn_out": torch.randn((m, model.q_dim), generator=g, device=cuda).to(torch.bfloat16),
          "ffn_normed": torch.randn((m, CFG.hidden_size), generator=g, device=cuda).to(torch.bfloat16),
          "ffn_act": torch.randn((m, CFG.intermediate_size), generator=g, device=cuda).to(torch.bfloat16)}
    bufs = {p: torch.empty((m, raws[p][2]), dtype=torch.float32, device=cuda) for p in raws}
    model.layer_linears(0, xs["normed"], xs["attn_out"], xs["ffn_normed"], xs["ffn_act"], bufs)
    torch.cuda.synchronize()
    src = {"q": "normed", "k": "normed", "v": "normed", "o": "attn_out", "gate": "ffn_normed",
           "up": "ffn_normed", "down": "ffn_act"}
    for p, (raw, qt, n, k) in raws.items():
        ref = O.matmul_ref(xs[src[p]].float().cpu().numpy(), raw, qt, n, k)
        assert O.rel_err(bufs[p].cpu().numpy(), ref) <= TOL, p


@pytest.mark.parametrize("m", [1, 8])
def test_gemma4_lm_head_tied_to_quantized_embedding(cuda, m):
    """No lm_head.weight: the logits come from the quantized token_embd table, and the
    same table serves the embedding lookup."""
    model, _, emb = _model(cuda)
    assert "lm_head.weight" not in model.weights
    x = torch.from_numpy(O.make_activations(m, CFG.hidden_size, seed=4)).to(torch.bfloat16).cuda()
    logits = torch.empty((m, CFG.vocab_size), dtype=torch.float32, device=cuda)
    model.project_lm_head(x, logits)
    ref = O.matmul_ref(x.float().cpu().numpy(), emb, O.Q6_K, CFG.vocab_size, CFG.hidden_size)
    assert O.rel_err(logits.cpu().numpy(), ref) <= TOL
    ids = torch.tensor([1, 4095, 77], dtype=torch.int32, device=cuda)
    e = torch.empty((3, CFG.hidden_size), dtype=torch.float32, device=cuda)
    model.embed_tokens(ids, e)
    full = O.dequantize(emb, O.Q6_K, CFG.vocab_size, CFG.hidden_size)
    assert np.array_equal(e.cpu().numpy(), full[[1, 4095, 77]])
