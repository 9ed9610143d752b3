"""Weight loading for the B200 path -- same functions and names as the
reference loader (vllm_webgpu/quant/gguf_loader.py), with two fixes the
quantized kernels need:

* GGUF tensors keep their quantization type and logical [N, K] shape
  (the reference uploads flat u8 and drops both, gguf_loader.py:152-159);
* everything lands in CUDA device memory as torch tensors instead of WebGPU
  storage buffers (vllm_webgpu/webgpu/buffer.py:30-36).

Quantized 2-D weights become :class:`GGUFQuantTensor` (raw GGUF blocks,
byte-identical to the file); F32/F16/BF16 tensors become dense tensors.
"""
from __future__ import annotations

import json
import logging
import struct
from pathlib import Path

import numpy as np
import torch

from ..formats import QUANT_SIZES, GGUFQuantTensor

logger = logging.getLogger(__name__)

_GGUF_MAGIC = b"GGUF"


def detect_weight_format(path: str) -> str:
    """"safetensors" | "safetensors_sharded" | "gguf" (reference gguf_loader.py:13-31)."""
    p = Path(path)
    if p.is_dir():
        if (p / "model.safetensors.index.json").exists():
            return "safetensors_sharded"
        return "safetensors"
    if p.suffix == ".gguf":
        return "gguf"
    if p.suffix in {".safetensors", ".bin"}:
        return "safetensors"
    with open(p, "rb") as f:
        magic = f.read(4)
    return "gguf" if magic == _GGUF_MAGIC else "safetensors"


def _device(device) -> torch.device:
    return torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())


def load_safetensors_weights(path: str, device=None, quantize: str | None = None) -> dict:
    """Load a safetensors file to ``device``.

    Like the reference (gguf_loader.py:51-92), BF16 and F32 tensors are cast
    to F16 with a clip to +-65504. With ``quantize`` set (e.g. "Q4_K"), every
    2-D ``*_proj.weight`` is packed into that GGUF format on the device.
    """
    dev = _device(device)
    with open(path, "rb") as f:
        header_len = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(header_len))
        raw_data = f.read()
    weights: dict = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        dtype_str = meta["dtype"]
        shape = tuple(meta["shape"])
        start, end = meta["data_offsets"]
        raw = raw_data[start:end]
        if dtype_str == "F16":
            arr = np.frombuffer(raw, dtype=np.float16).reshape(shape)
        elif dtype_str == "BF16":
            u16 = np.frombuffer(raw, dtype=np.uint16)
            f32 = (u16.astype(np.uint32) << 16).view(np.float32)
            arr = np.clip(f32, -65504.0, 65504.0).reshape(shape).astype(np.float16)
        elif dtype_str == "F32":
            arr = np.clip(np.frombuffer(raw, dtype=np.float32), -65504.0, 65504.0).reshape(shape).astype(np.float16)
        else:
            logger.warning("Unsupported dtype %s for tensor %s, skipping", dtype_str, name)
            continue
        t = torch.from_numpy(np.ascontiguousarray(arr)).to(dev)
        if quantize and t.dim() == 2 and name.endswith("_proj.weight"):
            from .pack import quantize as pack
            t = pack(t, quantize)
        weights[name] = t
    logger.info("Loaded %d tensors from %s", len(weights), path)
    return weights


def load_safetensors_weights_sharded(model_dir: str, device=None, quantize: str | None = None) -> dict:
    """Multi-shard safetensors via model.safetensors.index.json (reference :34-48)."""
    index_path = Path(model_dir) / "model.safetensors.index.json"
    with open(index_path) as f:
        index = json.load(f)
    weights: dict = {}
    for shard in sorted(set(index["weight_map"].values())):
        weights.update(load_safetensors_weights(str(Path(model_dir) / shard), device, quantize))
    return weights


# GGUF -> HuggingFace tensor names. The table has to name the same tensors as
# the reference's (gguf_loader.py:95-134) so models find their weights.
_GGUF_TOP = {
    "token_embd.weight": "model.embed_tokens.weight",
    "output.weight": "lm_head.weight",
    "output_norm.weight": "model.norm.weight",
}
_GGUF_BLK = {
    "attn_q.weight": "self_attn.q_proj.weight",
    "attn_k.weight": "self_attn.k_proj.weight",
    "attn_v.weight": "self_attn.v_proj.weight",
    "attn_output.weight": "self_attn.o_proj.weight",
    "attn_norm.weight": "input_layernorm.weight",
    "ffn_gate.weight": "mlp.gate_proj.weight",
    "ffn_up.weight": "mlp.up_proj.weight",
    "ffn_down.weight": "mlp.down_proj.weight",
    "ffn_norm.weight": "post_attention_layernorm.weight",
    "attn_q_norm.weight": "self_attn.q_norm.weight",
    "attn_k_norm.weight": "self_attn.k_norm.weight",
    "post_attention_norm.weight": "post_attention_layernorm.weight",
    "post_ffw_norm.weight": "post_feedforward_layernorm.weight",
    "layer_output_scale.weight": "self_attn.layer_scale",
}


def _gguf_to_hf_name(gguf_name: str) -> str | None:
    if gguf_name in _GGUF_TOP:
        return _GGUF_TOP[gguf_name]
    if gguf_name.startswith("blk."):
        parts = gguf_name.split(".", 2)
        if len(parts) == 3 and parts[2] in _GGUF_BLK:
            return f"model.layers.{parts[1]}.{_GGUF_BLK[parts[2]]}"
    return None


def load_gguf_weights(path: str, device=None) -> dict:
    """Load a GGUF file with HF-style names (reference gguf_loader.py:137-162).

    Quantized tensors of a supported type (Q4_0, Q8_0, Q4_K, Q6_K) become
    GGUFQuantTensor([N, row_bytes] uint8 blocks, qtype, (N, K)); F32/F16/BF16
    tensors become dense tensors in their logical shape. Any other quantized
    type raises ValueError naming it (the B200 kernels cannot read it).
    """
    try:
        import gguf
    except ImportError as e:  # same message as the reference
        raise ImportError("Install the 'gguf' package to load GGUF files.") from e
    dev = _device(device)
    reader = gguf.GGUFReader(path)
    weights: dict = {}
    skipped = 0
    for tensor in reader.tensors:
        hf_name = _gguf_to_hf_name(tensor.name)
        if hf_name is None:
            skipped += 1
            continue
        qt = int(tensor.tensor_type)
        shape = tuple(int(v) for v in reversed(list(tensor.shape)))  # GGML ne[] is innermost-first
        if qt in QUANT_SIZES:
            n = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
            k = shape[-1]
            data = np.require(np.asarray(tensor.data).view(np.uint8), requirements=["C", "W"]).reshape(n, -1)
            weights[hf_name] = GGUFQuantTensor(torch.from_numpy(data).to(dev), qt, (n, k))
        elif qt in (int(gguf.GGMLQuantizationType.F32), int(gguf.GGMLQuantizationType.F16),
                    int(gguf.GGMLQuantizationType.BF16)):
            arr = np.asarray(tensor.data)
            if qt == int(gguf.GGMLQuantizationType.BF16):
                arr = (arr.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
            weights[hf_name] = torch.from_numpy(np.require(arr, requirements=["C", "W"]).reshape(shape)).to(dev)
        else:
            raise ValueError(f"{tensor.name}: GGUF type {gguf.GGMLQuantizationType(qt).name} is not "
                             f"supported by the B200 kernels (supported: Q4_0, Q8_0, Q4_K, Q6_K, F32, F16, BF16)")
    logger.info("Loaded %d GGUF tensors (%d skipped) from %s", len(weights), skipped, path)
    return weights


def gguf_read_config(path: str) -> dict:
    """Model configuration from GGUF metadata (reference gguf_loader.py:165-228):
    same keys and defaults."""
    try:
        import gguf
    except ImportError as e:
        raise ImportError("Install the 'gguf' package.") from e
    reader = gguf.GGUFReader(path)

    def _get(key):
        if key not in reader.fields:
            return None
        v = reader.fields[key].parts[-1].tolist()
        if isinstance(v, list) and len(v) == 1:
            return v[0]
        return v

    def _get_str(key):
        v = _get(key)
        return bytes(v).decode("utf-8", errors="replace") if isinstance(v, list) else v

    arch = _get("general.architecture")
    p = bytes(arch).decode() if isinstance(arch, list) else str(arch)
    cfg = {
        "architectures": [_get_str("general.name") or "LlamaForCausalLM"],
        "hidden_size": _get(f"{p}.embedding_length") or 4096,
        "num_hidden_layers": _get(f"{p}.block_count") or 32,
        "num_attention_heads": _get(f"{p}.attention.head_count") or 32,
        "num_key_value_heads": _get(f"{p}.attention.head_count_kv") or 8,
        "intermediate_size": _get(f"{p}.feed_forward_length") or 14336,
        "vocab_size": 151936,
        "rope_theta": _get(f"{p}.rope.freq_base") or 10000.0,
        "head_dim": _get(f"{p}.attention.key_length"),
        "max_position_embeddings": _get(f"{p}.context_length") or 8192,
        "tie_word_embeddings": False,
        "final_logit_softcapping": _get(f"{p}.final_logit_softcapping"),
        "_gguf_arch_prefix": p,
    }
    if cfg["head_dim"] is None:
        cfg["head_dim"] = cfg["hidden_size"] // cfg["num_attention_heads"]
    arch_map = {"llama": "LlamaForCausalLM", "qwen3": "Qwen3ForCausalLM", "qwen2": "Qwen2ForCausalLM",
                "gemma3": "Gemma3ForCausalLM", "gemma4": "Gemma3ForCausalLM"}
    cfg["architectures"] = [arch_map.get(p, "LlamaForCausalLM")]
    return cfg
