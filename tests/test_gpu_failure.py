"""Failure detection on the GPU, made without faulting it: a bounded wait that can
never complete (a peer GPU that never publishes its partials) must give up, report
the timeout through ggufmm_device_status, and leave the context usable.

The fused down-projection + all-reduce kernel is launched on ONE GPU as rank 0 of a
2-GPU group whose two exchange buffers are both local: rank 1 never runs, so its
flags are never set. The wait limit is lowered first so the kernel gives up within
milliseconds instead of seconds."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O
from tests.helpers import TOL

pytestmark = pytest.mark.gpu


def test_peer_wait_times_out_and_context_survives(cuda):
    from vllm_webgpu_b200 import _lib, ops
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    lib = _lib.lib()
    n, k, m, world = 512, 1024, 1, 2
    raw = O.make_weights(n, k, O.Q4_K, seed=21)
    w = GGUFQuantTensor(torch.from_numpy(raw).cuda(), O.Q4_K, (n, k))
    x = torch.from_numpy(O.make_activations(m, k, seed=22)).to(torch.bfloat16).cuda()
    y = torch.full((m, n), 7.0, dtype=torch.float32, device=cuda)
    nbytes = int(lib.ggufmm_gemv_allreduce_buffer_bytes(n, 8, world))
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=cuda) for _ in range(world)]
    ptrs = (ctypes.c_void_p * world)(*[b.data_ptr() for b in bufs])
    stream = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    assert lib.ggufmm_device_status(1, None) == 0
    assert lib.ggufmm_set_wait_limit(4096) == 0
    try:
        st = lib.ggufmm_gemv_allreduce(w.data.data_ptr(), O.Q4_K, n, k, x.data_ptr(), _lib.BF16, m, k,
                                       y.data_ptr(), _lib.F32, n, ptrs, world, 0, 8, 1, stream)
        assert st == 0  # the launch itself is valid
        torch.cuda.synchronize()  # returns: the kernel gave up instead of hanging
        assert lib.ggufmm_device_status(1, None) == 1  # the timeout is reported ...
        assert lib.ggufmm_device_status(0, None) == 0  # ... and cleared
    finally:
        assert lib.ggufmm_set_wait_limit(0) == 0
    # no sum was stored: the unfinished all-reduce left y as it was
    assert torch.all(y == 7.0)
    # this rank's own partials did land in both (local) exchange buffers
    assert torch.count_nonzero(bufs[0]).item() > 0 and torch.count_nonzero(bufs[1]).item() > 0
    # the context is still usable: a normal call is correct and raises no timeout
    y2 = ops.gemv(x, w, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ref = O.matmul_ref(x.float().cpu().numpy(), raw, O.Q4_K, n, k)
    assert O.rel_err(y2.cpu().numpy(), ref) <= TOL
    assert lib.ggufmm_device_status(0, None) == 0
