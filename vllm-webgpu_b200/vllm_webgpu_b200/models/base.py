"""Model base with the reference's dispatch boundary, backed by CUDA.

``BaseB200Model._dispatch`` keeps the signature of the reference's
``BaseWebGPUModel._dispatch(shader_name, bindings, constants, workgroups,
shader_subdir)`` (vllm_webgpu/models/base.py:62-100) so the model code's
linear call sites (vllm_webgpu/models/llama.py:276-283, 328-332, 343-348,
355-359) run unchanged; the "matmul_quant" shader is served by the sm_100a
kernels of libggufmm instead of a WGSL pipeline. Buffers are torch CUDA
tensors; the caller owns them, including the output, exactly as in the
reference (scratch buffers are pre-allocated, llama.py:58-102).

``_batched_dispatch`` mirrors the reference's one-submit-per-layer block
(base.py:28-44): dispatches inside the block are captured into a CUDA graph
and the graph is launched only when the block exits cleanly, so a Python
exception half-way through a layer launches nothing (the reference's reason
for submitting only on clean exit).
"""
from __future__ import annotations

import logging
from contextlib import contextmanager

import torch

from .. import ops
from ..formats import GGUFQuantTensor

logger = logging.getLogger(__name__)


class BaseB200Model:
    def __init__(self, model_config, device: torch.device | str | None = None) -> None:
        self.model_config = model_config
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.weights: dict[str, GGUFQuantTensor | torch.Tensor] = {}
        self._graph_block = False

    @contextmanager
    def _batched_dispatch(self, capture: bool = True):
        """Record every _dispatch() in the block; launch them only on clean exit."""
        if not capture:
            yield
            return
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        self._graph_block = True
        try:
            with torch.cuda.graph(graph, stream=side):
                yield
        finally:
            self._graph_block = False
        graph.replay()  # not reached when the block raised
        torch.cuda.current_stream(self.device).wait_stream(side)
        self._last_graph = graph  # keep the graph (and its memory) alive until replaced

    def load_weights(self, path: str) -> None:
        from ..quant.gguf_loader import (detect_weight_format, load_gguf_weights, load_safetensors_weights,
                                         load_safetensors_weights_sharded)
        fmt = detect_weight_format(path)
        if fmt == "safetensors":
            self.weights = load_safetensors_weights(path, self.device)
        elif fmt == "safetensors_sharded":
            self.weights = load_safetensors_weights_sharded(path, self.device)
        elif fmt == "gguf":
            self.weights = load_gguf_weights(path, self.device)
        else:
            raise ValueError(f"Unknown weight format for {path}")
        logger.info("Loaded %d weight tensors (%s format)", len(self.weights), fmt)

    def _dispatch(self, shader_name: str, bindings: list, constants: dict, workgroups: tuple = (1, 1, 1),
                  shader_subdir: str = "generic") -> None:
        """Run one kernel. The quantized matmul and the embedding lookup are on this path:

        ``matmul_quant``: bindings = [x, W, scales|unused, out], constants =
        {K, N, USE_QUANT}. x is [tokens, K]; out is a caller-owned [tokens, N]
        tensor written in place. W is a GGUFQuantTensor (any of Q4_0, Q8_0,
        Q4_K, Q6_K) or, with USE_QUANT=0, a dense [N, K] fp16/bf16 tensor.
        ``embedding_lookup``: bindings = [table, ids, out], constants =
        {HIDDEN_DIM}; the table is a GGUFQuantTensor (rows dequantized by
        ggufmm_embedding) or a dense [vocab, hidden] tensor.
        ``workgroups`` is accepted for signature compatibility; the launch
        geometry is the kernels' own.
        """
        if shader_name == "embedding_lookup":
            # bindings = [table, token ids, out] (vllm_webgpu/models/llama.py:170-178)
            table, ids, out = bindings
            hidden = int(constants["HIDDEN_DIM"])
            if isinstance(table, GGUFQuantTensor):
                if table.k != hidden:
                    raise ValueError(f"embedding_lookup: table rows are {table.k} wide, HIDDEN_DIM={hidden}")
                ops.embedding(ids, table, out=out.reshape(-1, hidden))
            else:
                out.reshape(-1, hidden).copy_(table[ids.reshape(-1).long()])
            return
        if shader_name != "matmul_quant":
            raise NotImplementedError(
                f"{shader_subdir}/{shader_name}: only the quantized matmul and embedding run on the B200 path")
        x, w, _scales, out = bindings
        k, n = int(constants["K"]), int(constants["N"])
        if isinstance(w, GGUFQuantTensor):
            if w.shape != (n, k):
                raise ValueError(f"matmul_quant: weight is {w.shape}, constants say N={n}, K={k}")
            ops.mul_mat(x.reshape(-1, k), w, out=out.reshape(-1, n))
            return
        if int(constants.get("USE_QUANT", 0)):
            raise ValueError("matmul_quant: USE_QUANT=1 needs a GGUFQuantTensor weight")
        if tuple(w.shape) != (n, k):
            raise ValueError(f"matmul_quant: weight is {tuple(w.shape)}, constants say N={n}, K={k}")
        y = torch.matmul(x.reshape(-1, k).to(w.dtype), w.t())
        # copy_ writes into `out` whatever its strides (out.reshape of a non-contiguous
        # tensor would be a temporary copy, and the result would be lost)
        out.copy_(y.reshape(out.shape))

    def forward(self, input_ids, positions, attn_metadata):  # pragma: no cover - out of scope
        raise NotImplementedError("attention / norm / rope are outside the quantized-matmul path")
