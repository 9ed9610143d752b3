"""PyTorch-facing operators over libggufmm (CUDA tensors in, CUDA tensors out).

These are the calls the model linear layers make in place of the reference's
``_dispatch("matmul_quant", [x, W, scales, out], {K, N, USE_QUANT}, ...)``
(vllm_webgpu/models/base.py:62-100, vllm_webgpu/models/llama.py:276-283).
Every function launches hand-written sm_100a kernels on the current CUDA
stream and returns without synchronizing. There is no CPU path: tensors must
live on a CUDA device and the native library must be present.
"""
from __future__ import annotations

import torch

from . import _lib
from .formats import GGUFQuantTensor

_DTYPE_CODE = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}

GEMV_MAX_M = 8


def _code(dtype: torch.dtype) -> int:
    if dtype not in _DTYPE_CODE:
        raise ValueError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16")
    return _DTYPE_CODE[dtype]


def _require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if t.device.type != "cuda":
            raise ValueError("libggufmm operates on CUDA tensors only (no CPU fallback)")
        if t.device != dev:
            raise ValueError(f"tensors on different devices: {t.device} vs {dev}")
    return dev


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _as_2d(x: torch.Tensor, k: int) -> torch.Tensor:
    if x.shape[-1] != k:
        raise ValueError(f"activation last dim {x.shape[-1]} != K={k}")
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2


def _out(x2: torch.Tensor, n: int, out: torch.Tensor | None, out_dtype: torch.dtype | None) -> torch.Tensor:
    m = x2.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype or x2.dtype, device=x2.device)
    else:
        if out.dim() != 2 or out.shape[0] != m or out.shape[1] != n or out.stride(1) != 1:
            raise ValueError(f"out must be a row-major [{m}, {n}] tensor")
    return out


def dequantize(w: GGUFQuantTensor, out_dtype: torch.dtype = torch.float32,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """[N, K] dequantized weights; float32 output is bit-identical to
    gguf.quants.dequantize (the reference loader's decoder)."""
    dev = _require_cuda(w.data)
    n, k = w.shape
    if out is None:
        out = torch.empty((n, k), dtype=out_dtype, device=dev)
    elif out.shape != (n, k) or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous [{n}, {k}] tensor")
    with torch.cuda.device(dev):
        st = _lib.lib().ggufmm_dequantize(w.data.data_ptr(), w.qtype, n, k, out.data_ptr(),
                                          _code(out.dtype), _stream(dev))
    _lib.check(st, "ggufmm_dequantize")
    return out


def embedding(ids: torch.Tensor, table: GGUFQuantTensor, out: torch.Tensor | None = None,
              out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Rows ``ids`` of a GGUF-quantized embedding table, dequantized: out[t, :] =
    table[ids[t], :]. Replaces the reference's ``embedding_lookup`` dispatch
    (vllm_webgpu/models/llama.py:170-178), which copied rows of an f16 table.
    float32 output is bit-identical to gguf.quants.dequantize of the row. An id
    outside the table gives a zero row and sets bit 2 of the device status word."""
    dev = _require_cuda(ids, table.data)
    ids32 = ids.reshape(-1)
    if ids32.dtype != torch.int32 or not ids32.is_contiguous():
        ids32 = ids32.to(torch.int32).contiguous()
    n_ids = ids32.numel()
    if out is None:
        out = torch.empty((n_ids, table.k), dtype=out_dtype, device=dev)
    elif out.dim() != 2 or out.shape != (n_ids, table.k) or out.stride(1) != 1:
        raise ValueError(f"out must be a row-major [{n_ids}, {table.k}] tensor")
    with torch.cuda.device(dev):
        st = _lib.lib().ggufmm_embedding(table.data.data_ptr(), table.qtype, table.n, table.k, ids32.data_ptr(),
                                         n_ids, out.data_ptr(), _code(out.dtype), out.stride(0), _stream(dev))
    _lib.check(st, "ggufmm_embedding")
    return out


def stage_copy(dst: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """dst <- src by a kernel, where one side is page-locked host memory and the other
    a CUDA tensor (both contiguous, same byte size, 16-byte aligned): the decode step's
    host <-> device staging on the SMs instead of a copy engine, chained with the
    projections by programmatic dependent launch. Replaces the reference's buffer
    upload / staging readback (vllm_webgpu/webgpu/buffer.py:34, :46-63). Ordered on
    the CUDA tensor's device's current stream."""
    dev = dst.device if dst.is_cuda else src.device
    if not dev.type == "cuda":
        raise ValueError("stage_copy needs a CUDA tensor on one side")
    host = src if dst.is_cuda else dst
    if host.device.type == "cpu" and not host.is_pinned():
        raise ValueError("the host side of stage_copy must be pinned")
    if not (dst.is_contiguous() and src.is_contiguous()):
        raise ValueError("stage_copy needs contiguous tensors")
    nbytes = dst.numel() * dst.element_size()
    if nbytes != src.numel() * src.element_size():
        raise ValueError("stage_copy: byte sizes differ")
    with torch.cuda.device(dev):
        st = _lib.lib().ggufmm_stage_copy(dst.data_ptr(), src.data_ptr(), nbytes, _stream(dev))
    _lib.check(st, "ggufmm_stage_copy")
    return dst


def staged_copy(dst: torch.Tensor, src: torch.Tensor) -> None:
    """The serving graphs' host <-> device copy: ``stage_copy`` where its conditions
    hold (GGUFMM_STAGE_KERNEL=0 keeps the copy-engine memcpy), else ``dst.copy_``."""
    import os
    if (os.environ.get("GGUFMM_STAGE_KERNEL", "1") != "0" and dst.is_contiguous() and src.is_contiguous()
            and dst.data_ptr() % 16 == 0 and src.data_ptr() % 16 == 0 and dst.dtype == src.dtype
            and dst.numel() == src.numel() and (dst.is_cuda != src.is_cuda)):
        stage_copy(dst, src)
    else:
        dst.copy_(src, non_blocking=True)


def gemv(x: torch.Tensor, w: GGUFQuantTensor, out: torch.Tensor | None = None,
         out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Decode GEMV, M <= 8 tokens: out[m, n] = sum_k x[m, k] W[n, k]."""
    dev = _require_cuda(x, w.data)
    x2 = _as_2d(x, w.k)
    y = _out(x2, w.n, out, out_dtype)
    with torch.cuda.device(dev):
        st = _lib.lib().ggufmm_gemv(w.data.data_ptr(), w.qtype, w.n, w.k, x2.data_ptr(), _code(x2.dtype),
                                    x2.shape[0], x2.stride(0), y.data_ptr(), _code(y.dtype), y.stride(0),
                                    _stream(dev))
    _lib.check(st, "ggufmm_gemv")
    return y


GEMV_STREAM, GEMV_F16, GEMV_INT8 = 0, 1, 2
_gemv_kernels: dict = {}


def gemv_kernel(m: int, w: GGUFQuantTensor, x_dtype: torch.dtype = torch.bfloat16) -> int:
    """Which decode GEMV kernel ``gemv`` launches for M tokens against ``w`` on the
    weight's device: GEMV_INT8, GEMV_F16 or GEMV_STREAM (the CUDA-core fallback), or
    ``_lib.ERR_ALIGN`` when no decode GEMV can stage the weight's rows."""
    dev = _require_cuda(w.data)
    key = (dev.index, w.qtype, w.n, w.k, m, x_dtype)
    kind = _gemv_kernels.get(key)
    if kind is None:
        with torch.cuda.device(dev):
            kind = int(_lib.lib().ggufmm_gemv_kernel(w.qtype, w.n, w.k, m, _code(x_dtype)))
        if kind != _lib.ERR_ALIGN:  # ERR_ALIGN: no decode GEMV can stage these rows
            _lib.check(min(kind, 0), "ggufmm_gemv_kernel")
        _gemv_kernels[key] = kind
    return kind


def gemv_preferred(m: int, w: GGUFQuantTensor, x_dtype: torch.dtype = torch.bfloat16) -> bool:
    """Whether the decode GEMV is the faster path for M tokens: M <= 8, and for
    Q4_K a tensor-core GEMV fits the shape (where only the streaming fallback
    does, as for M = 8 at K = 14336, the tcgen05 GEMM with fused dequantization
    is 2-4x faster)."""
    if not 1 <= m <= GEMV_MAX_M:
        return False
    kind = gemv_kernel(m, w, x_dtype)
    return kind >= 0 and (w.qtype != 12 or kind != GEMV_STREAM)


def gemv_grouped(x: torch.Tensor, ws: list[GGUFQuantTensor], outs: list[torch.Tensor] | None = None,
                 out_dtype: torch.dtype | None = None) -> list[torch.Tensor]:
    """Decode GEMV of up to 4 weights sharing the activations (fused q/k/v or
    gate/up) in one launch; returns one [M, N_i] output per weight."""
    if not 1 <= len(ws) <= 4:
        raise ValueError("gemv_grouped takes 1 to 4 weights")
    k, qt = ws[0].k, ws[0].qtype
    if any(w.k != k or w.qtype != qt for w in ws):
        raise ValueError("grouped weights must share K and the quantization type")
    dev = _require_cuda(x, *[w.data for w in ws])
    x2 = _as_2d(x, k)
    if outs is None:
        outs = [None] * len(ws)
    ys = [_out(x2, w.n, o, out_dtype) for w, o in zip(ws, outs)]
    if len({y.dtype for y in ys}) != 1:
        raise ValueError("grouped outputs must share a dtype")
    import ctypes
    nseg = len(ws)
    qs = (ctypes.c_void_p * nseg)(*[w.data.data_ptr() for w in ws])
    ns = (ctypes.c_int64 * nseg)(*[w.n for w in ws])
    yp = (ctypes.c_void_p * nseg)(*[y.data_ptr() for y in ys])
    ld = (ctypes.c_int64 * nseg)(*[y.stride(0) for y in ys])
    with torch.cuda.device(dev):
        st = _lib.lib().ggufmm_gemv_grouped(nseg, qs, ns, qt, k, x2.data_ptr(), _code(x2.dtype), x2.shape[0],
                                            x2.stride(0), yp, _code(ys[0].dtype), ld, _stream(dev))
    _lib.check(st, "ggufmm_gemv_grouped")
    return ys


def swiglu_fusable(x: torch.Tensor, gate: GGUFQuantTensor, up: GGUFQuantTensor) -> bool:
    """Whether gemv_swiglu handles these operands (decode M, Q4_K / Q4_0, K % 256 == 0,
    and the activations fit the integer GEMV's shared memory)."""
    m = x.numel() // max(x.shape[-1], 1)
    return (x.is_cuda and 1 <= m <= GEMV_MAX_M and gate.qtype == up.qtype and gate.qtype in (2, 12)
            and gate.shape == up.shape and gate.k % 256 == 0 and x.shape[-1] == gate.k
            and gemv_kernel(m, gate, x.dtype) == GEMV_INT8)


def gemv_swiglu(x: torch.Tensor, gate: GGUFQuantTensor, up: GGUFQuantTensor, out: torch.Tensor | None = None,
                out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Fused FFN input for decode (M <= 8): out = silu(x gate^T) * (x up^T), one launch
    (the gate and up GEMVs and the SwiGLU of the reference's three dispatches)."""
    if gate.shape != up.shape or gate.qtype != up.qtype:
        raise ValueError("gate and up must share shape and quantization type")
    dev = _require_cuda(x, gate.data, up.data)
    x2 = _as_2d(x, gate.k)
    y = _out(x2, gate.n, out, out_dtype)
    with torch.cuda.device(dev):
        st = _lib.lib().ggufmm_gemv_swiglu(gate.data.data_ptr(), up.data.data_ptr(), gate.qtype, gate.n, gate.k,
                                           x2.data_ptr(), _code(x2.dtype), x2.shape[0], x2.stride(0),
                                           y.data_ptr(), _code(y.dtype), y.stride(0), _stream(dev))
    _lib.check(st, "ggufmm_gemv_swiglu")
    return y


def residual_fusable(x: torch.Tensor, w: GGUFQuantTensor) -> bool:
    """Whether gemv_residual handles these operands (decode M on the integer GEMV)."""
    m = x.numel() // max(x.shape[-1], 1)
    return (x.is_cuda and w.qtype in (2, 12) and w.k % 256 == 0 and x.shape[-1] == w.k
            and gemv_preferred(m, w, x.dtype) and gemv_kernel(m, w, x.dtype) == GEMV_INT8)


def gemv_residual(x: torch.Tensor, w: GGUFQuantTensor, residual: torch.Tensor,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Decode GEMV with the residual add fused: out = x W^T + residual, one launch,
    the sum rounded once into out's dtype (= residual's). ``out`` may be
    ``residual`` itself (in place)."""
    dev = _require_cuda(x, w.data, residual)
    x2 = _as_2d(x, w.k)
    r2 = residual.reshape(-1, w.n) if residual.dim() != 2 else residual
    if r2.shape != (x2.shape[0], w.n) or r2.stride(1) != 1:
        raise ValueError(f"residual must be [{x2.shape[0]}, {w.n}] with unit column stride")
    y = _out(x2, w.n, out, r2.dtype)
    if y.dtype != r2.dtype:
        raise ValueError("out and residual must share a dtype")
    with torch.cuda.device(dev):
        st = _lib.lib().ggufmm_gemv_residual(w.data.data_ptr(), w.qtype, w.n, w.k, x2.data_ptr(), _code(x2.dtype),
                                             x2.shape[0], x2.stride(0), y.data_ptr(), _code(y.dtype), y.stride(0),
                                             r2.data_ptr(), r2.stride(0), _stream(dev))
    _lib.check(st, "ggufmm_gemv_residual")
    return y


_ffn_workspaces: dict = {}


def _ffn_workspace(w: GGUFQuantTensor, m: int, swiglu: bool) -> torch.Tensor:
    need = int(_lib.lib().ggufmm_gemm_ffn_workspace_size(w.qtype, m, w.n, w.k, int(swiglu)))
    idx = w.data.device.index
    ws = _ffn_workspaces.get(idx)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device=w.data.device)
        _ffn_workspaces[idx] = ws
    return ws


def gemm_swiglu(x: torch.Tensor, gate: GGUFQuantTensor, up: GGUFQuantTensor, out: torch.Tensor | None = None,
                out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """out = silu(x gate^T) * (x up^T) at any M through the tensor-core GEMM with the
    SwiGLU in its epilogue pass (ggufmm_gemm_swiglu), replacing the reference's gate and
    up dispatches and its gelu_mul shader (vllm_webgpu/models/llama.py:343-352)."""
    if gate.shape != up.shape or gate.qtype != up.qtype:
        raise ValueError("gate and up must share shape and quantization type")
    dev = _require_cuda(x, gate.data, up.data)
    x2 = _as_2d(x, gate.k)
    y = _out(x2, gate.n, out, out_dtype)
    ws = _ffn_workspace(gate, x2.shape[0], True)
    with torch.cuda.device(dev):
        st = _lib.lib().ggufmm_gemm_swiglu(gate.data.data_ptr(), up.data.data_ptr(), gate.qtype, gate.n, gate.k,
                                           x2.data_ptr(), _code(x2.dtype), x2.shape[0], x2.stride(0), y.data_ptr(),
                                           _code(y.dtype), y.stride(0), ws.data_ptr(), ws.numel(), _stream(dev))
    _lib.check(st, "ggufmm_gemm_swiglu")
    return y


def gemm_residual(x: torch.Tensor, w: GGUFQuantTensor, residual: torch.Tensor,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """out = x W^T + residual at any M, the add in the GEMM's epilogue pass
    (ggufmm_gemm_residual); ``out`` may be ``residual`` (in place)."""
    dev = _require_cuda(x, w.data, residual)
    x2 = _as_2d(x, w.k)
    r2 = residual.reshape(-1, w.n) if residual.dim() != 2 else residual
    if r2.shape != (x2.shape[0], w.n) or r2.stride(1) != 1:
        raise ValueError(f"residual must be [{x2.shape[0]}, {w.n}] with unit column stride")
    y = _out(x2, w.n, out, r2.dtype)
    if y.dtype != r2.dtype:
        raise ValueError("out and residual must share a dtype")
    ws = _ffn_workspace(w, x2.shape[0], False)
    with torch.cuda.device(dev):
        st = _lib.lib().ggufmm_gemm_residual(w.data.data_ptr(), w.qtype, w.n, w.k, x2.data_ptr(), _code(x2.dtype),
                                             x2.shape[0], x2.stride(0), y.data_ptr(), _code(y.dtype), y.stride(0),
                                             r2.data_ptr(), r2.stride(0), ws.data_ptr(), ws.numel(), _stream(dev))
    _lib.check(st, "ggufmm_gemm_residual")
    return y


def ffn_epilogue(sums: torch.Tensor, n: int, out: torch.Tensor, swiglu: bool,
                 residual: torch.Tensor | None = None) -> torch.Tensor:
    """The epilogue pass over fp32 sums (ggufmm_ffn_epilogue): swiglu, sums [M, 2n] (gate |
    up) -> out = silu(gate) * up; else sums [M, n] -> out = sums + residual."""
    dev = _require_cuda(sums, out)
    if sums.dtype != torch.float32 or not sums.is_contiguous():
        raise ValueError("sums must be contiguous float32")
    m = sums.shape[0]
    r = residual.reshape(m, n) if residual is not None else None
    with torch.cuda.device(dev):
        st = _lib.lib().ggufmm_ffn_epilogue(sums.data_ptr(), m, n, int(swiglu), r.data_ptr() if r is not None else None,
                                            r.stride(0) if r is not None else 0, out.data_ptr(), _code(out.dtype),
                                            out.stride(0), _stream(dev))
    _lib.check(st, "ggufmm_ffn_epilogue")
    return out


def swiglu(x: torch.Tensor, gate: GGUFQuantTensor, up: GGUFQuantTensor, out: torch.Tensor | None = None,
           out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """silu(x gate^T) * (x up^T) on the fastest native path: the one-launch integer decode
    GEMV where it serves the shape; other decode shapes run the grouped decode GEMV into
    fp32 sums and the epilogue pass; above the GEMV the GEMM with the SwiGLU epilogue."""
    x2 = _as_2d(x, gate.k)
    m = x2.shape[0]
    if swiglu_fusable(x2, gate, up):
        try:
            return gemv_swiglu(x2, gate, up, out=out, out_dtype=out_dtype)
        except ValueError as exc:
            if not _lib.is_align_refusal(exc):
                raise
    if gemv_preferred(m, gate, x2.dtype) and gate.shape == up.shape and gate.qtype == up.qtype:
        sums = torch.empty((m, 2 * gate.n), dtype=torch.float32, device=x2.device)
        gemv_grouped(x2, [gate, up], outs=[sums[:, :gate.n], sums[:, gate.n:]])
        y = _out(x2, gate.n, out, out_dtype)
        return ffn_epilogue(sums, gate.n, y, swiglu=True)
    return gemm_swiglu(x2, gate, up, out=out, out_dtype=out_dtype)


def linear_residual(x: torch.Tensor, w: GGUFQuantTensor, residual: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """x W^T + residual on the fastest native path: the integer decode GEMV with the add in
    its epilogue, other decode shapes as a GEMV into fp32 plus the epilogue pass, above
    the GEMV the GEMM with the add in its epilogue pass."""
    x2 = _as_2d(x, w.k)
    m = x2.shape[0]
    if residual_fusable(x2, w):
        try:
            return gemv_residual(x2, w, residual, out=out)
        except ValueError as exc:
            if not _lib.is_align_refusal(exc):
                raise
    if gemv_preferred(m, w, x2.dtype):
        sums = gemv(x2, w, out_dtype=torch.float32)
        r2 = residual.reshape(m, w.n)
        y = _out(x2, w.n, out, r2.dtype)
        return ffn_epilogue(sums, w.n, y, swiglu=False, residual=r2)
    return gemm_residual(x2, w, residual, out=out)


class PeerExchange:
    """Exchange buffers for ``gemv_allreduce`` on every GPU of a process group:
    one symmetric-memory allocation per GPU (``torch.distributed._symmetric_memory``,
    CUDA IPC between the GPUs of one node), zero-filled, with the peer addresses
    and the epoch counter the kernel needs. Creating it is a collective."""

    def __init__(self, n: int, m_max: int, group=None, device: torch.device | None = None):
        import ctypes

        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        group = group or dist.group.WORLD
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.n, self.m_max = n, m_max
        nbytes = int(_lib.lib().ggufmm_gemv_allreduce_buffer_bytes(n, m_max, self.world))
        if nbytes == 0:
            raise ValueError(f"no peer exchange for n={n}, m_max={m_max}, world={self.world}")
        device = device or torch.device("cuda", torch.cuda.current_device())
        try:
            symm_mem.enable_symm_mem_for_group(group.group_name)
        except Exception:  # already enabled, or not needed by this torch
            pass
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, group.group_name)
        torch.cuda.synchronize(device)
        dist.barrier(group)  # every buffer is zero before any GPU publishes into it
        self.ptrs = (ctypes.c_void_p * self.world)(*self.handle.buffer_ptrs)
        self.epoch = 0


class PeerAllReduce:
    """One-shot fp32 all-reduce over NVLink peer memory (ggufmm_allreduce) for vectors of
    up to 65536 values: one symmetric-memory exchange buffer per GPU of the group
    (``torch.distributed._symmetric_memory``), zero-filled. Creating it is a collective;
    calls must be made by every rank in the same order, and may be captured in a CUDA
    graph (the call's generation counter lives in device memory)."""

    MAX_N = 1 << 16

    def __init__(self, n: int, group=None, device: torch.device | None = None):
        import ctypes

        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        group = group or dist.group.WORLD
        self.world, self.rank, self.n = dist.get_world_size(group), dist.get_rank(group), n
        nbytes = int(_lib.lib().ggufmm_allreduce_buffer_bytes(n, self.world))
        if nbytes == 0:
            raise ValueError(f"no peer all-reduce for n={n} (a multiple of 4, at most {self.MAX_N} values)")
        device = device or torch.device("cuda", torch.cuda.current_device())
        try:
            symm_mem.enable_symm_mem_for_group(group.group_name)
        except Exception:  # already enabled, or not needed by this torch
            pass
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, group.group_name)
        torch.cuda.synchronize(device)
        dist.barrier(group)  # every buffer is zero before any GPU publishes into it
        self.ptrs = (ctypes.c_void_p * self.world)(*self.handle.buffer_ptrs)

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None,
                 residual: torch.Tensor | None = None) -> torch.Tensor:
        """out = the sum of every rank's x (+ residual), identical on every rank; x, out
        and residual fp32, contiguous, n values; out may be x."""
        if x.dtype != torch.float32 or not x.is_contiguous() or x.numel() != self.n:
            raise ValueError(f"x must be a contiguous float32 tensor of {self.n} values")
        out = x if out is None else out
        dev = x.device
        with torch.cuda.device(dev):
            st = _lib.lib().ggufmm_allreduce(x.data_ptr(), out.data_ptr(), self.n, self.ptrs, self.world, self.rank,
                                             residual.data_ptr() if residual is not None else None, _stream(dev))
        _lib.check(st, "ggufmm_allreduce")
        return out


class PeerGather:
    """Output buffers for the N-split GEMM whose epilogue all-gathers over NVLink
    (``gemm_allgather``): on every GPU of the group one symmetric-memory buffer holding
    the device barrier's flags and the full [m, n_total] output. Creating it is a
    collective. ``y`` is this GPU's full output (valid after ``gemm_allgather``)."""

    def __init__(self, m: int, n_total: int, dtype: torch.dtype = torch.bfloat16, group=None,
                 device: torch.device | None = None):
        import ctypes

        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        group = group or dist.group.WORLD
        self.world, self.rank, self.m, self.n_total, self.dtype = (dist.get_world_size(group),
                                                                   dist.get_rank(group), m, n_total, dtype)
        es = torch.empty((), dtype=dtype).element_size()
        device = device or torch.device("cuda", torch.cuda.current_device())
        try:
            symm_mem.enable_symm_mem_for_group(group.group_name)
        except Exception:  # already enabled, or not needed by this torch
            pass
        self.hdr = int(_lib.lib().ggufmm_allreduce_buffer_bytes(0, self.world))  # the barrier's flags
        self.buf = symm_mem.empty(self.hdr + m * n_total * es, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, group.group_name)
        torch.cuda.synchronize(device)
        dist.barrier(group)
        self.ptrs = (ctypes.c_void_p * self.world)(*self.handle.buffer_ptrs)
        self.y_ptrs = (ctypes.c_void_p * self.world)(*[p + self.hdr for p in self.handle.buffer_ptrs])
        self.y = self.buf[self.hdr:].view(dtype).view(m, n_total)


def gemm_allgather(x: torch.Tensor, w_local: GGUFQuantTensor, gather: PeerGather) -> torch.Tensor:
    """x @ W^T for a weight split by output rows over the gather's GPUs: this rank's slice
    ``w_local`` (n_total / world rows) is multiplied and every value is stored into every
    GPU's output at its column (the all-gather in the GEMM's epilogue); a device-side
    barrier then makes the full [M, n_total] output ``gather.y`` valid on every GPU."""
    dev = _require_cuda(x, w_local.data)
    x2 = _as_2d(x, w_local.k)
    m = x2.shape[0]
    if m != gather.m or w_local.n * gather.world != gather.n_total:
        raise ValueError("activations / weight slice do not match the gather buffers")
    ws = workspace_for(w_local, m)
    with torch.cuda.device(dev):
        lib = _lib.lib()
        st = lib.ggufmm_gemm_allgather(w_local.data.data_ptr(), w_local.qtype, w_local.n, w_local.k, x2.data_ptr(),
                                       _code(x2.dtype), m, x2.stride(0), gather.y_ptrs, gather.world,
                                       gather.rank * w_local.n, _code(gather.dtype), gather.n_total, ws.data_ptr(),
                                       ws.numel(), _stream(dev))
        _lib.check(st, "ggufmm_gemm_allgather")
        st = lib.ggufmm_peer_barrier(gather.ptrs, gather.world, gather.rank, _stream(dev))
    _lib.check(st, "ggufmm_peer_barrier")
    return gather.y


def gemv_allreduce(x: torch.Tensor, w: GGUFQuantTensor, exchange: PeerExchange, out: torch.Tensor | None = None,
                   out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Decode GEMV summed over the exchange's GPUs in the same kernel (NVLink peer
    memory): every GPU of the group calls it with its own W slice and receives
    the full sum. Replaces GEMV + NCCL all-reduce for the TP down projection."""
    dev = _require_cuda(x, w.data)
    x2 = _as_2d(x, w.k)
    if x2.shape[0] > exchange.m_max or w.n != exchange.n:
        raise ValueError("activations or output width do not match the exchange buffers")
    y = _out(x2, w.n, out, out_dtype)
    exchange.epoch += 1
    with torch.cuda.device(dev):
        st = _lib.lib().ggufmm_gemv_allreduce(w.data.data_ptr(), w.qtype, w.n, w.k, x2.data_ptr(), _code(x2.dtype),
                                              x2.shape[0], x2.stride(0), y.data_ptr(), _code(y.dtype), y.stride(0),
                                              exchange.ptrs, exchange.world, exchange.rank, exchange.m_max,
                                              exchange.epoch, _stream(dev))
    if st != 0:
        exchange.epoch -= 1  # nothing was launched
    _lib.check(st, "ggufmm_gemv_allreduce")
    return y


_workspaces: dict[int, torch.Tensor] = {}


def workspace_for(w: GGUFQuantTensor, m: int) -> torch.Tensor:
    """A cached per-device scratch buffer large enough for ggufmm_gemm (and for
    ggufmm_gemm_grouped when w is the group's weight with the largest N)."""
    need = int(_lib.lib().ggufmm_gemm_workspace_size(w.qtype, m, w.n, w.k))
    idx = w.data.device.index
    ws = _workspaces.get(idx)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device=w.data.device)
        _workspaces[idx] = ws
    return ws


def gemm(x: torch.Tensor, w: GGUFQuantTensor, out: torch.Tensor | None = None,
         out_dtype: torch.dtype | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Tensor-core (tcgen05) GEMM, any M: out[m, n] = sum_k x[m, k] W[n, k]."""
    dev = _require_cuda(x, w.data)
    x2 = _as_2d(x, w.k)
    y = _out(x2, w.n, out, out_dtype)
    ws = workspace if workspace is not None else workspace_for(w, x2.shape[0])
    with torch.cuda.device(dev):
        st = _lib.lib().ggufmm_gemm(w.data.data_ptr(), w.qtype, w.n, w.k, x2.data_ptr(), _code(x2.dtype),
                                    x2.shape[0], x2.stride(0), y.data_ptr(), _code(y.dtype), y.stride(0),
                                    ws.data_ptr(), ws.numel(), _stream(dev))
    _lib.check(st, "ggufmm_gemm")
    return y


def gemm_grouped(x: torch.Tensor, ws: list[GGUFQuantTensor], outs: list[torch.Tensor] | None = None,
                 out_dtype: torch.dtype | None = None) -> list[torch.Tensor]:
    """GEMM of up to 4 weights sharing the activations (q/k/v or gate/up) at any M;
    Q4_K at M <= 1024 is one fused-dequant launch over all of them."""
    if not 1 <= len(ws) <= 4:
        raise ValueError("gemm_grouped takes 1 to 4 weights")
    k, qt = ws[0].k, ws[0].qtype
    if any(w.k != k or w.qtype != qt for w in ws):
        raise ValueError("grouped weights must share K and the quantization type")
    dev = _require_cuda(x, *[w.data for w in ws])
    x2 = _as_2d(x, k)
    if outs is None:
        outs = [None] * len(ws)
    ys = [_out(x2, w.n, o, out_dtype) for w, o in zip(ws, outs)]
    if len({y.dtype for y in ys}) != 1:
        raise ValueError("grouped outputs must share a dtype")
    import ctypes
    nseg = len(ws)
    wsp = workspace_for(max(ws, key=lambda w: w.n), x2.shape[0])
    qs = (ctypes.c_void_p * nseg)(*[w.data.data_ptr() for w in ws])
    ns = (ctypes.c_int64 * nseg)(*[w.n for w in ws])
    yp = (ctypes.c_void_p * nseg)(*[y.data_ptr() for y in ys])
    ld = (ctypes.c_int64 * nseg)(*[y.stride(0) for y in ys])
    with torch.cuda.device(dev):
        st = _lib.lib().ggufmm_gemm_grouped(nseg, qs, ns, qt, k, x2.data_ptr(), _code(x2.dtype), x2.shape[0],
                                            x2.stride(0), yp, _code(ys[0].dtype), ld, wsp.data_ptr(), wsp.numel(),
                                            _stream(dev))
    _lib.check(st, "ggufmm_gemm_grouped")
    return ys


def mul_mat(x: torch.Tensor, w: GGUFQuantTensor, out: torch.Tensor | None = None,
            out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """y = x @ W^T: GEMV for M <= 8 where gemv_preferred holds, tensor-core GEMM otherwise.

    Same contract as vLLM's ``fused_mul_mat_gguf(x, qweight, qweight_type)``
    (vllm/model_executor/layers/quantization/gguf.py:198-230); the leading
    dimensions of ``x`` are preserved.
    """
    lead = x.shape[:-1]
    x2 = _as_2d(x, w.k)
    m = x2.shape[0]
    if x2.is_cuda and gemv_preferred(m, w, x2.dtype):
        try:
            y = gemv(x2, w, out=out, out_dtype=out_dtype)
        except ValueError as exc:
            if not _lib.is_align_refusal(exc):
                raise
            # unaligned operands: the GEMM path has no 16-byte alignment requirement
            y = gemm(x2, w, out=out, out_dtype=out_dtype)
    else:
        y = gemm(x2, w, out=out, out_dtype=out_dtype)
    return y.reshape(*lead, w.n)
