"""The Gemma 4 layer's quantized projections, called the way the reference's
``Gemma4WebGPUModel`` calls them (vllm_webgpu/models/gemma4.py:203-210 q/k/v,
:259-264 o, :274-291 gate/up/down, :151-156 LM head), each through
``_dispatch("matmul_quant", ...)``.

On the matmul path Gemma 4 differs from Llama in two ways, both kept here:
* the attention width is ``num_attention_heads * head_dim``, which need not equal
  the hidden size (q: hidden -> q_dim, k/v: hidden -> kv_dim, o: q_dim -> hidden);
* the LM head falls back to the tied embedding table when the file has no
  ``lm_head.weight`` (gemma4.py:152) -- in a GGUF file that is the quantized
  ``token_embd.weight``, which the GEMV / GEMM read directly.
The reference's FFN activation shader for Gemma is the same gelu_mul
(silu(gate) * up, shaders/generic/gelu_mul.wgsl:14-20) as Llama's, so the fused
SwiGLU paths apply unchanged. The per-head norms, PLE block and logit softcap
are outside the quantized-matmul path.
"""
from __future__ import annotations

import torch

from .llama import LlamaB200Model


class Gemma4B200Model(LlamaB200Model):
    """Gemma 4 projections on the B200 kernels (same call sites as the Llama model)."""

    def __init__(self, model_config, device: torch.device | str | None = None) -> None:
        super().__init__(model_config, device)
        cfg = model_config
        if cfg is not None:
            self.hidden_size = cfg.hidden_size
            self.num_q_heads = cfg.num_attention_heads
            self.num_kv_heads = cfg.num_key_value_heads
            self.head_dim = getattr(cfg, "head_dim", cfg.hidden_size // cfg.num_attention_heads)
            self.q_dim = self.num_q_heads * self.head_dim
            self.kv_dim = self.num_kv_heads * self.head_dim

    def lm_head_weight(self):
        """``lm_head.weight`` or, as in the reference (gemma4.py:152), the tied embedding table."""
        return self.weights.get("lm_head.weight", self.weights["model.embed_tokens.weight"])

    def project_lm_head(self, hidden: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
        return self._linear(hidden, self.lm_head_weight(), logits)


# reference: vllm_webgpu/v1/model_runner.py ARCH_MAP (architecture -> model family)
ARCH_MAP = {
    "LlamaForCausalLM": "llama", "MistralForCausalLM": "llama", "Qwen2ForCausalLM": "llama",
    "Qwen3ForCausalLM": "llama", "Gemma3ForCausalLM": "gemma4",
}


def build_model(arch: str, model_config, device: torch.device | str | None = None):
    """The B200 model class for an architecture name, as the reference's
    ``_build_model`` picks its WebGPU model (vllm_webgpu/v1/model_runner.py:42-53);
    NotImplementedError for architectures outside the map."""
    family = ARCH_MAP.get(arch)
    if family == "llama":
        return LlamaB200Model(model_config, device)
    if family == "gemma4":
        return Gemma4B200Model(model_config, device)
    raise NotImplementedError(f"Architecture {arch!r} is not supported. Supported: {sorted(ARCH_MAP)}")
