"""Host-side mirror of the reference API: GGUF loading keeps qtype + shape,
format detection, config reading, platform registration, _dispatch errors."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O

gguf = pytest.importorskip("gguf")


def _write_gguf(path, tensors: dict, arch="llama"):
    w = gguf.GGUFWriter(str(path), arch)
    w.add_block_count(1)
    w.add_embedding_length(512)
    w.add_feed_forward_length(1024)
    w.add_head_count(8)
    w.add_head_count_kv(2)
    w.add_context_length(4096)
    w.add_rope_freq_base(500000.0)
    for name, (arr, qt) in tensors.items():
        if qt is None:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=gguf.GGMLQuantizationType(qt))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@pytest.fixture
def gguf_file(tmp_path):
    q = O.make_weights(64, 512, O.Q4_K, seed=0)       # attn_q: N=64, K=512
    d6 = O.make_weights(512, 256, O.Q6_K, seed=1)     # ffn_down: N=512, K=256
    q8 = O.make_weights(32, 512, O.Q8_0, seed=2)
    norm = np.linspace(0.5, 1.5, 512).astype(np.float32)
    p = tmp_path / "tiny.gguf"
    _write_gguf(p, {"blk.0.attn_q.weight": (q, O.Q4_K), "blk.0.ffn_down.weight": (d6, O.Q6_K),
                    "blk.0.attn_k.weight": (q8, O.Q8_0), "blk.0.attn_norm.weight": (norm, None),
                    "rope_freqs": (norm[:4], None)})
    return p, q, d6, q8, norm


def test_load_gguf_keeps_type_and_shape(gguf_file):
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    from vllm_webgpu_b200.quant.gguf_loader import detect_weight_format, load_gguf_weights
    p, q, d6, q8, norm = gguf_file
    assert detect_weight_format(str(p)) == "gguf"
    w = load_gguf_weights(str(p), device="cpu")
    wq = w["model.layers.0.self_attn.q_proj.weight"]
    assert isinstance(wq, GGUFQuantTensor) and wq.qtype == O.Q4_K and wq.shape == (64, 512)
    assert np.array_equal(wq.data.numpy(), q)
    wd = w["model.layers.0.mlp.down_proj.weight"]
    assert wd.qtype == O.Q6_K and wd.shape == (512, 256) and np.array_equal(wd.data.numpy(), d6)
    assert w["model.layers.0.self_attn.k_proj.weight"].qtype == O.Q8_0
    assert torch.allclose(w["model.layers.0.input_layernorm.weight"], torch.from_numpy(norm))
    assert "rope_freqs" not in w and len(w) == 4  # unmapped tensors skipped, as in the reference


def test_gguf_read_config(gguf_file):
    from vllm_webgpu_b200.quant.gguf_loader import gguf_read_config
    cfg = gguf_read_config(str(gguf_file[0]))
    assert cfg["hidden_size"] == 512 and cfg["intermediate_size"] == 1024
    assert cfg["num_key_value_heads"] == 2 and cfg["head_dim"] == 64
    assert cfg["architectures"] == ["LlamaForCausalLM"]


def test_unsupported_gguf_type_is_refused(tmp_path):
    from vllm_webgpu_b200.quant.gguf_loader import load_gguf_weights
    raw = np.zeros((4, 176), np.uint8)  # Q5_K: 256 weights / 176 bytes
    p = tmp_path / "q5k.gguf"
    _write_gguf(p, {"blk.0.attn_v.weight": (raw, int(gguf.GGMLQuantizationType.Q5_K))})
    with pytest.raises(ValueError, match="Q5_K"):
        load_gguf_weights(str(p), device="cpu")


def test_detect_formats(tmp_path):
    from vllm_webgpu_b200.quant.gguf_loader import detect_weight_format
    (tmp_path / "m").mkdir()
    (tmp_path / "m" / "model.safetensors.index.json").write_text("{}")
    assert detect_weight_format(str(tmp_path / "m")) == "safetensors_sharded"
    f = tmp_path / "blob"
    f.write_bytes(b"GGUF\x03\x00")
    assert detect_weight_format(str(f)) == "gguf"
    assert detect_weight_format(str(tmp_path / "x.safetensors")) == "safetensors"


def test_safetensors_quantize_on_load(tmp_path):
    import json
    import struct
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    from vllm_webgpu_b200.quant.gguf_loader import load_safetensors_weights
    w = (np.random.default_rng(0).standard_normal((32, 512)) * 0.02).astype(np.float16)
    hdr = {"model.layers.0.mlp.up_proj.weight": {"dtype": "F16", "shape": [32, 512],
                                                 "data_offsets": [0, w.nbytes]}}
    hb = json.dumps(hdr).encode()
    p = tmp_path / "m.safetensors"
    p.write_bytes(struct.pack("<Q", len(hb)) + hb + w.tobytes())
    out = load_safetensors_weights(str(p), device="cpu", quantize="Q4_K")
    t = out["model.layers.0.mlp.up_proj.weight"]
    assert isinstance(t, GGUFQuantTensor) and t.shape == (32, 512)
    assert np.array_equal(t.data.numpy(), O.quantize(w.astype(np.float32), O.Q4_K))


def test_platform_without_gpu_and_register():
    import vllm_webgpu_b200
    from vllm_webgpu_b200.platform import B200Platform
    if torch.cuda.is_available():
        pytest.skip("CPU-only expectations")
    assert B200Platform.is_available() is False
    assert vllm_webgpu_b200.register() is None
    assert B200Platform.get_device_count() == 0
    assert B200Platform.device_type == "cuda"
    with pytest.raises(ValueError):
        B200Platform.set_device(1)
    B200Platform.verify_quantization("q4_k_m")
    with pytest.raises(ValueError):
        B200Platform.verify_quantization("awq")


def test_dispatch_boundary_errors():
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    from vllm_webgpu_b200.models.base import BaseB200Model
    m = BaseB200Model(None, device="cpu")
    with pytest.raises(NotImplementedError):
        m._dispatch("rms_norm", [], {}, (1, 1, 1))
    w = GGUFQuantTensor(torch.zeros((4, 144), dtype=torch.uint8), O.Q4_K, (4, 256))
    x = torch.zeros((1, 256))
    with pytest.raises(ValueError, match="N=8"):
        m._dispatch("matmul_quant", [x, w, None, torch.zeros((1, 8))], {"K": 256, "N": 8, "USE_QUANT": 1})
    with pytest.raises(ValueError, match="CUDA"):  # right shapes, but the kernels run on CUDA tensors only
        m._dispatch("matmul_quant", [x, w, None, torch.zeros((1, 4))], {"K": 256, "N": 4, "USE_QUANT": 1})


def test_build_model_follows_the_reference_arch_map():
    """Architecture -> model family as the reference's ARCH_MAP
    (vllm_webgpu/v1/model_runner.py:32-53)."""
    from types import SimpleNamespace

    from vllm_webgpu_b200.models.gemma4 import ARCH_MAP, Gemma4B200Model, build_model
    from vllm_webgpu_b200.models.llama import LlamaB200Model
    cfg = SimpleNamespace(hidden_size=2560, num_attention_heads=8, num_key_value_heads=2, head_dim=256)
    assert type(build_model("LlamaForCausalLM", None, device="cpu")) is LlamaB200Model
    assert type(build_model("Qwen2ForCausalLM", None, device="cpu")) is LlamaB200Model
    g = build_model("Gemma3ForCausalLM", cfg, device="cpu")
    assert isinstance(g, Gemma4B200Model) and g.q_dim == 2048 and g.kv_dim == 512
    assert set(ARCH_MAP) == {"LlamaForCausalLM", "MistralForCausalLM", "Qwen2ForCausalLM", "Qwen3ForCausalLM",
                             "Gemma3ForCausalLM"}
    with pytest.raises(NotImplementedError):
        build_model("GPT2LMHeadModel", None, device="cpu")
