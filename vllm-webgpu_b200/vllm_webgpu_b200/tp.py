"""Tensor-parallel Q4_K SwiGLU FFN over NCCL.

The reference has no multi-GPU path at all: one device, gloo-only distributed
init, custom all-reduce disabled (vllm_webgpu/platform.py:83-84,112,133-135,
vllm_webgpu/v1/worker.py:56-59). This module is the B200 addition:

* gate and up are split by OUTPUT rows (each rank owns intermediate/P rows,
  a row slice of the GGUF byte matrix -- no re-quantization);
* down is split by INPUT columns over the same intermediate range (a
  superblock-aligned column slice of the GGUF bytes; 28672/8 = 3584 = 14
  superblocks);
* each rank computes silu(x Wg_r^T) * (x Wu_r^T) and its partial
  y_r = a_r Wd_r^T with the sm_100a kernels, then ONE all-reduce (sum) of the
  [M, hidden] partials joins the ranks: the one-shot peer-memory all-reduce
  (ops.PeerAllReduce) for decode-sized partials, NCCL above; or (opt-in,
  GGUFMM_TP_FUSED=1, decode M <= 8) one kernel that computes the down projection
  and exchanges the partials through NVLink peer memory (ops.gemv_allreduce).
* TensorParallelLayerLinears splits all seven projections of a layer the same
  way, with the o / down GEMV and its all-reduce in one kernel in decode.

The matmul callable is injectable so the sharding and the collective can be
tested on CPU ranks (gloo) against the oracle; on GPUs it is always
``ops.mul_mat``.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from . import _lib
from .formats import QUANT_SIZES, GGUFQuantTensor


def shard_range(total: int, rank: int, world: int, align: int) -> tuple[int, int]:
    """[start, stop) of rank's equal share of ``total``, aligned to ``align``."""
    if total % world:
        raise ValueError(f"{total} does not split evenly over {world} ranks")
    per = total // world
    if per % align:
        raise ValueError(f"shard of {per} is not a multiple of the {align}-weight block")
    return rank * per, (rank + 1) * per


def shard_ffn(gate: GGUFQuantTensor, up: GGUFQuantTensor, down: GGUFQuantTensor, rank: int,
              world: int) -> tuple[GGUFQuantTensor, GGUFQuantTensor, GGUFQuantTensor]:
    """This rank's gate/up row slices and down column slice (byte slices of the GGUF blocks)."""
    inter, hidden = gate.shape
    if up.shape != (inter, hidden) or down.shape != (hidden, inter):
        raise ValueError(f"inconsistent FFN shapes: gate {gate.shape}, up {up.shape}, down {down.shape}")
    block = QUANT_SIZES[down.qtype][1]
    i0, i1 = shard_range(inter, rank, world, block)
    return gate.rows(i0, i1), up.rows(i0, i1), down.cols(i0, i1)


class TensorParallelSwiGLU:
    """y = down(silu(gate(x)) * up(x)), intermediate dimension split over ranks."""

    def __init__(self, gate: GGUFQuantTensor, up: GGUFQuantTensor, down: GGUFQuantTensor, rank: int = 0,
                 world: int = 1, group=None, matmul: Callable | None = None, presharded: bool = False,
                 reduce_dtype: torch.dtype = torch.float32):
        if presharded:
            self.gate, self.up, self.down = gate, up, down
        else:
            self.gate, self.up, self.down = shard_ffn(gate, up, down, rank, world)
        self.rank, self.world, self.group = rank, world, group
        # the fused gate/up/SwiGLU GEMV serves decode unless a custom matmul is injected
        self.fused_swiglu = matmul is None
        if matmul is None:
            from .ops import mul_mat
            matmul = mul_mat
        self.matmul = matmul
        self.reduce_dtype = reduce_dtype
        # decode down projection + all-reduce fused over NVLink peer memory: opt-in
        # (GGUFMM_TP_FUSED=1); at 2 GPUs it measures 73.7 us per M=1 step of the 70B FFN
        # against 72.3 us for the GEMV + the one-shot peer all-reduce, the default
        import os
        self.fused_allreduce = self.fused_swiglu and reduce_dtype == torch.float32 and \
            os.environ.get("GGUFMM_TP_FUSED", "0") == "1"
        self._exchange = None

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """The FFN output, plus ``residual`` when given (the reference's final add,
        llama.py:362-363): rank 0 adds it to its partial before the all-reduce, so the
        sum carries it once -- in the down projection's epilogue when that GEMV runs on
        the integer tensor cores with the residual in the reduce dtype."""
        if self.fused_swiglu and x.is_cuda:
            from . import ops
            # gate, up and SwiGLU in one native call (fp32 activation): the decode GEMV or
            # the GEMM with the SwiGLU epilogue
            act = ops.swiglu(x, self.gate, self.up, out_dtype=torch.float32)
        else:
            g = self.matmul(x, self.gate, out_dtype=torch.float32)
            u = self.matmul(x, self.up, out_dtype=torch.float32)
            act = torch.nn.functional.silu(g) * u  # injected (CPU test) matmul: fp32 SwiGLU
        if self.world > 1 and self.fused_allreduce and act.is_cuda and act.shape[0] <= 8:
            y = self._down_allreduce(act)
            if y is not None:
                return y if residual is None else y.add_(residual)
        add_here = residual is not None and self.rank == 0
        if add_here and self.fused_swiglu and residual.dtype == self.reduce_dtype and act.is_cuda:
            from . import ops
            y = ops.linear_residual(act, self.down, residual)  # the add in the GEMV / GEMM epilogue
        else:
            y = self.matmul(act, self.down, out_dtype=self.reduce_dtype)
            if add_here:
                y.add_(residual)
        if self.world > 1:
            self._allreduce(y)
        return y

    def _allreduce(self, t: torch.Tensor) -> None:
        """Sum over the ranks: the one-shot peer-memory kernel for decode-sized fp32
        partials, NCCL otherwise (or with GGUFMM_TP_ALLREDUCE=nccl)."""
        import os
        if (self.fused_swiglu and t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()
                and t.numel() <= 1 << 16 and t.numel() % 4 == 0
                and os.environ.get("GGUFMM_TP_ALLREDUCE", "peer") != "nccl"):
            from . import ops
            peers = self.__dict__.setdefault("_peer", {})
            if t.numel() not in peers:
                peers[t.numel()] = ops.PeerAllReduce(t.numel(), self.group, t.device)
            peers[t.numel()](t)
            return
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def _down_allreduce(self, act: torch.Tensor):
        """Decode: the down projection and the all-reduce in one kernel over NVLink
        peer memory (ggufmm_gemv_allreduce); None when the shape is not served."""
        from . import ops
        try:
            if self._exchange is None:
                self._exchange = ops.PeerExchange(self.down.n, 8, self.group, act.device)
            return ops.gemv_allreduce(act, self.down, self._exchange, out_dtype=torch.float32)
        except _lib.GGUFMMValueError as e:
            # only a shape / alignment the fused kernel does not serve falls back (to
            # NCCL from now on); a dtype or argument refusal is a caller bug
            if e.status not in (_lib.ERR_SHAPE, _lib.ERR_ALIGN, _lib.ERR_QTYPE):
                raise
            self.fused_allreduce = False
            return None

    __call__ = forward


class TensorParallelLayerLinears:
    """The seven projections of one Llama layer split over ``world`` ranks (the
    Megatron split that keeps attention and the SwiGLU local to a rank):

    * q, k, v and gate, up by OUTPUT rows (a row slice of each GGUF byte matrix:
      rank r owns heads / intermediate features [r N/P, (r+1) N/P));
    * o and down by INPUT columns over the same ranges (superblock-aligned
      column slices), so each rank's o / down partial is summed by ONE
      all-reduce each (NCCL over NVLink, fp32: a bf16 partial would round each
      rank's sum by up to 2^-9 relative, the size of the 2e-3 gate itself).

    The reference calls these projections one dispatch each on a single device
    (vllm_webgpu/models/llama.py:276-283, 328-332, 343-348, 355-359); with
    world = 1 this class runs exactly those calls. ``forward`` takes the
    rank-local activations: ``attn_local`` is this rank's slice of the attention
    output (its heads), ``act_local`` its slice of the SwiGLU activation.
    """

    NAMES = ("q", "k", "v", "o", "gate", "up", "down")

    def __init__(self, weights: dict, rank: int = 0, world: int = 1, group=None, matmul: Callable | None = None):
        self.rank, self.world, self.group = rank, world, group
        self.matmul = matmul  # injectable (CPU tests); the GPU path uses the grouped kernels
        self.collective = True  # False leaves out the all-reduces (measuring what they cost)
        self._graphs: dict = {}
        # the o / down all-reduces: the one-shot peer-memory kernel (ggufmm_allreduce) for
        # decode-sized partials (3.9 us for 16 KB on 2 GPUs against 18.6 us for NCCL's, in
        # a CUDA graph), NCCL above 65536 values or with GGUFMM_TP_ALLREDUCE=nccl
        import os
        self.peer_allreduce = matmul is None and os.environ.get("GGUFMM_TP_ALLREDUCE", "peer") != "nccl"
        # o / down GEMV and all-reduce in one kernel in decode (35.6 against 37.6 us per layer
        # step on 2 GPUs); GGUFMM_TP_FUSED=0 runs the GEMV and ggufmm_allreduce separately
        self.fused_allreduce = matmul is None and os.environ.get("GGUFMM_TP_FUSED", "1") != "0"
        self._peer: dict = {}
        w = {}
        for p in ("q", "k", "v", "gate", "up"):
            n = weights[p].n
            r0, r1 = shard_range(n, rank, world, 16)
            w[p] = weights[p] if world == 1 else weights[p].rows(r0, r1)
        for p in ("o", "down"):
            k = weights[p].k
            block = QUANT_SIZES[weights[p].qtype][1]
            c0, c1 = shard_range(k, rank, world, block)
            w[p] = weights[p] if world == 1 else weights[p].cols(c0, c1)
        self.w = w

    def _mm(self, x, w, out) -> None:
        if self.matmul is not None:
            out.copy_(self.matmul(x, w, out_dtype=out.dtype).reshape(out.shape))
            return
        from . import ops
        ops.mul_mat(x, w, out=out)

    def _grouped(self, x: torch.Tensor, ps, outs) -> None:
        if self.matmul is not None:
            for p, o in zip(ps, outs):
                self._mm(x, self.w[p], o)
            return
        from . import ops
        ws = [self.w[p] for p in ps]
        m = x.reshape(-1, x.shape[-1]).shape[0]
        if len({w.qtype for w in ws}) == 1 and ops.gemv_preferred(m, ws[0], x.dtype):
            ops.gemv_grouped(x, ws, outs=outs)
        elif len({w.qtype for w in ws}) == 1:
            ops.gemm_grouped(x, ws, outs=outs)
        else:
            for w, o in zip(ws, outs):
                ops.mul_mat(x, w, out=o)

    def _allreduce(self, t: torch.Tensor) -> None:
        if self.world == 1 or not self.collective:
            return
        if (self.peer_allreduce and t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()
                and t.numel() <= 1 << 16 and t.numel() % 4 == 0):
            from . import ops
            key = t.numel()
            if key not in self._peer:
                self._peer[key] = ops.PeerAllReduce(key, self.group, t.device)
            self._peer[key](t)
            return
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def _mm_allreduce(self, x, p: str, out) -> None:
        """out = the all-reduced x W_p^T: in decode (M <= 8 on the integer GEMV) one kernel
        that also all-reduces through NVLink peer memory (ggufmm_gemv_allreduce), else the
        projection and a separate all-reduce."""
        w = self.w[p]
        if self.world > 1 and self.collective and self.fused_allreduce and x.is_cuda and out.dtype == torch.float32:
            from . import ops
            m = x.reshape(-1, x.shape[-1]).shape[0]
            if m <= 8 and w.qtype in (2, 12) and ops.gemv_kernel(m, w, x.dtype) == ops.GEMV_INT8:
                ex = self._peer.get(("x", p))
                if ex is None:
                    ex = self._peer[("x", p)] = ops.PeerExchange(w.n, 8, self.group, x.device)
                ops.gemv_allreduce(x, w, ex, out=out)
                return
        self._mm(x, w, out)
        self._allreduce(out)

    def forward(self, normed, attn_local, ffn_normed, act_local, bufs: dict) -> dict:
        """bufs: q, k, v, gate, up (this rank's output slices) and o, down (full
        width, fp32: the all-reduced sums)."""
        self._grouped(normed, ("q", "k", "v"), [bufs["q"], bufs["k"], bufs["v"]])
        self._mm_allreduce(attn_local, "o", bufs["o"])
        self._grouped(ffn_normed, ("gate", "up"), [bufs["gate"], bufs["up"]])
        self._mm_allreduce(act_local, "down", bufs["down"])
        return bufs

    __call__ = forward

    def graph_step(self, normed, attn_local, ffn_normed, act_local, bufs: dict, stage_in=(), stage_out=()) -> dict:
        """``forward`` replayed from a CUDA graph (captured on the first call for these
        buffers), with optional (destination, source) host <-> device copies of pinned
        buffers captured before and after it: the decode serving loop, one replay per
        step (the NCCL all-reduces are captured with the launches)."""
        from . import ops
        stage_in, stage_out = list(stage_in), list(stage_out)
        key = (normed.data_ptr(), attn_local.data_ptr(), ffn_normed.data_ptr(), act_local.data_ptr(),
               tuple((k, b.data_ptr()) for k, b in sorted(bufs.items())),
               tuple((d.data_ptr(), s.data_ptr()) for d, s in stage_in + stage_out))
        g = self._graphs.get(key)

        def body():
            for dst, src in stage_in:
                ops.staged_copy(dst, src)
            self.forward(normed, attn_local, ffn_normed, act_local, bufs)
            for dst, src in stage_out:
                ops.staged_copy(dst, src)
        if g is None:
            cur = torch.cuda.current_stream()
            side = torch.cuda.Stream()
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                body()  # warm-up
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                body()
            cur.wait_stream(side)
            self._graphs[key] = g
        g.replay()
        return bufs
