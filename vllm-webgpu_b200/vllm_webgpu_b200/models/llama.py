"""The Llama layer's quantized projections, called the way the reference's
``LlamaWebGPUModel._transformer_layer`` calls them
(vllm_webgpu/models/llama.py:276-283 q/k/v, :328-332 o, :343-348 gate/up,
:355-359 down), each through ``_dispatch("matmul_quant", ...)``. In decode
(M <= 8) the projections that share an input -- q/k/v and gate/up -- run as
one grouped launch (ggufmm_gemv_grouped), as vLLM fuses QKV and gate_up.

The reference picks ``USE_QUANT = 0 if q_proj.weight is present`` and so never
runs its quantized branch (llama.py:258); here the branch is chosen by the
weight's type, so GGUF blocks always take the quantized kernels.
Attention, norms and RoPE between the projections are outside this path.
"""
from __future__ import annotations

import torch

from .. import _lib, ops
from ..formats import GGUFQuantTensor
from .base import BaseB200Model

PROJ = {
    "q": "self_attn.q_proj.weight", "k": "self_attn.k_proj.weight", "v": "self_attn.v_proj.weight",
    "o": "self_attn.o_proj.weight", "gate": "mlp.gate_proj.weight", "up": "mlp.up_proj.weight",
    "down": "mlp.down_proj.weight",
}


def _overlaps(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Whether two tensors share any bytes of storage."""
    if a.device != b.device or a.untyped_storage().data_ptr() != b.untyped_storage().data_ptr():
        return False
    a0, b0 = a.data_ptr(), b.data_ptr()
    a1 = a0 + (a.numel() and (sum((s - 1) * st for s, st in zip(a.shape, a.stride())) + 1) * a.element_size())
    b1 = b0 + (b.numel() and (sum((s - 1) * st for s, st in zip(b.shape, b.stride())) + 1) * b.element_size())
    return a0 < b1 and b0 < a1


class LlamaB200Model(BaseB200Model):
    """Holds the weights and runs a layer's seven projections."""

    def _w(self, layer: int, proj: str):
        return self.weights[f"model.layers.{layer}.{PROJ[proj]}"]

    def _linear(self, x: torch.Tensor, w, out: torch.Tensor) -> torch.Tensor:
        n, k = (w.shape if isinstance(w, GGUFQuantTensor) else tuple(w.shape))
        use_quant = 1 if isinstance(w, GGUFQuantTensor) else 0
        self._dispatch("matmul_quant", [x, w, None, out], {"K": k, "N": n, "USE_QUANT": use_quant},
                       ((n + 255) // 256, 1, 1))
        return out

    def _fused(self, x: torch.Tensor, ws: list, bufs: list) -> bool:
        """One grouped launch for projections that read the same input (all
        GGUF-quantized with one qtype): the grouped decode GEMV where it is the
        faster path, else the grouped GEMM; False if not applicable."""
        m = x.reshape(-1, x.shape[-1]).shape[0]
        if (not all(isinstance(w, GGUFQuantTensor) for w in ws) or len({w.qtype for w in ws}) != 1
                or len({b.dtype for b in bufs}) != 1 or not x.is_cuda):
            return False
        outs = [b.reshape(-1, w.n) for b, w in zip(bufs, ws)]
        if ops.gemv_preferred(m, ws[0], x.dtype):
            ops.gemv_grouped(x, ws, outs=outs)
        else:
            ops.gemm_grouped(x, ws, outs=outs)
        return True

    def project_qkv(self, layer: int, normed: torch.Tensor, q_buf, k_buf, v_buf):
        ws = [self._w(layer, p) for p in ("q", "k", "v")]
        if not self._fused(normed, ws, [q_buf, k_buf, v_buf]):
            for buf, w in zip((q_buf, k_buf, v_buf), ws):
                self._linear(normed, w, buf)
        return q_buf, k_buf, v_buf

    def _linear_residual(self, x: torch.Tensor, w, out: torch.Tensor, residual):
        """out = x W^T (+ residual): the reference's projection followed by its add
        shader (llama.py:329-335, 357-363), here one native call: the decode GEMV with
        the add in its epilogue, or the GEMM with the add in its epilogue pass (the sum
        rounded once). ``out`` may be ``residual`` (h = h + proj in place)."""
        if residual is None:
            return self._linear(x, w, out)
        if isinstance(w, GGUFQuantTensor) and out.dtype == residual.dtype and x.is_cuda:
            ops.linear_residual(x.reshape(-1, w.k), w, residual.reshape(-1, w.n), out=out.reshape(-1, w.n))
            return out
        # dense (USE_QUANT=0) weights
        if out.data_ptr() == residual.data_ptr() or _overlaps(out, residual):
            tmp = torch.empty_like(out)
            self._linear(x, w, tmp)
            torch.add(tmp, residual, out=out)
            return out
        self._linear(x, w, out)
        out.add_(residual)
        return out

    def project_o(self, layer: int, attn_out: torch.Tensor, out: torch.Tensor, residual=None):
        return self._linear_residual(attn_out, self._w(layer, "o"), out, residual)

    def project_gate_up(self, layer: int, ffn_normed: torch.Tensor, gate_buf, up_buf):
        ws = [self._w(layer, "gate"), self._w(layer, "up")]
        if not self._fused(ffn_normed, ws, [gate_buf, up_buf]):
            self._linear(ffn_normed, ws[0], gate_buf)
            self._linear(ffn_normed, ws[1], up_buf)
        return gate_buf, up_buf

    def project_down(self, layer: int, ffn_act: torch.Tensor, out: torch.Tensor, residual=None):
        return self._linear_residual(ffn_act, self._w(layer, "down"), out, residual)

    def project_ffn_act(self, layer: int, ffn_normed: torch.Tensor, act_buf: torch.Tensor) -> torch.Tensor:
        """The FFN activation silu(gate) * up into ``act_buf``, where the reference runs
        the gate and up dispatches and its gelu_mul SwiGLU shader (llama.py:343-352):
        one native call -- the fused decode GEMV (M <= 8) or the GEMM with the SwiGLU in
        its epilogue pass."""
        gate, up = self._w(layer, "gate"), self._w(layer, "up")
        if isinstance(gate, GGUFQuantTensor) and isinstance(up, GGUFQuantTensor) and gate.qtype == up.qtype:
            return ops.swiglu(ffn_normed, gate, up, out=act_buf.reshape(-1, gate.n))
        g = torch.empty_like(act_buf, dtype=torch.float32)
        u = torch.empty_like(act_buf, dtype=torch.float32)
        self.project_gate_up(layer, ffn_normed, g, u)
        act_buf.copy_(torch.nn.functional.silu(g) * u)  # dense (USE_QUANT=0) weights
        return act_buf

    def embed_tokens(self, input_ids: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Token embeddings into ``out`` [tokens, hidden] from ``model.embed_tokens.weight``
        (GGUF ``token_embd.weight``, quantized in a GGUF file), as the reference's
        ``_dispatch("embedding_lookup", [table, ids, x], {HIDDEN_DIM})`` (llama.py:170-178)."""
        table = self.weights["model.embed_tokens.weight"]
        hidden = table.k if isinstance(table, GGUFQuantTensor) else table.shape[1]
        self._dispatch("embedding_lookup", [table, input_ids, out], {"HIDDEN_DIM": hidden},
                       (input_ids.numel(), 1, 1))
        return out

    def project_lm_head(self, hidden: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
        """Logits from the final hidden state on the GGUF output weight (``lm_head.weight``,
        GGUF ``output.weight``), quantized like the other projections (the reference
        forces an f16 head, llama.py:228-235)."""
        return self._linear(hidden, self.weights["lm_head.weight"], logits)

    def layer_linears(self, layer: int, normed, attn_out, ffn_normed, ffn_act, bufs: dict) -> dict:
        """All seven projections of one layer into caller-owned ``bufs``
        (keys q, k, v, o, gate, up, down)."""
        self.project_qkv(layer, normed, bufs["q"], bufs["k"], bufs["v"])
        self.project_o(layer, attn_out, bufs["o"])
        self.project_gate_up(layer, ffn_normed, bufs["gate"], bufs["up"])
        self.project_down(layer, ffn_act, bufs["down"])
        return bufs

    def layer_linears_graph(self, layer: int, normed, attn_out, ffn_normed, ffn_act, bufs: dict,
                            stage_in: list | None = None, stage_out: list | None = None) -> dict:
        """``layer_linears`` replayed from a CUDA graph, the decode serving path:
        the launches are captured once per (layer, buffer addresses) and then
        replayed with one host call. The inputs and ``bufs`` must be the same
        tensors (static buffers the caller refills) on every call; the replay is
        ordered on the current stream.

        ``stage_in`` / ``stage_out``: optional (destination, source) pairs of
        host <-> device copies captured into the same graph, before and after the
        projections -- pinned host buffers the caller refills / reads, so one
        replay moves a decode step's activations in and its outputs out."""
        stage_in, stage_out = list(stage_in or ()), list(stage_out or ())
        for dst, src in stage_in + stage_out:
            host = src if src.device.type == "cpu" else dst
            if not host.is_pinned():
                raise ValueError("staged host buffers must be pinned")
        key = (layer, normed.data_ptr(), attn_out.data_ptr(), ffn_normed.data_ptr(), ffn_act.data_ptr(),
               tuple((k, b.data_ptr()) for k, b in sorted(bufs.items())),
               tuple((d.data_ptr(), s.data_ptr()) for d, s in stage_in + stage_out))
        graphs = self.__dict__.setdefault("_layer_graphs", {})
        g = graphs.get(key)
        cur = torch.cuda.current_stream(self.device)

        def body():
            for dst, src in stage_in:
                ops.staged_copy(dst, src)
            self.layer_linears(layer, normed, attn_out, ffn_normed, ffn_act, bufs)
            for dst, src in stage_out:
                ops.staged_copy(dst, src)
        if g is None:
            side = torch.cuda.Stream(self.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                body()  # warm-up
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                body()
            cur.wait_stream(side)
            graphs[key] = g
        g.replay()
        return bufs
